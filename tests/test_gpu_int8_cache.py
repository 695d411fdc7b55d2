"""int8 KV cache on the engine against the CPU oracle and the reference fixture.

Quantising append, dequantisation (``get``) and beam reorder are integer /
exactly-rounded work and must match bit for bit (nn/cache.py:47-123).  The
fused-dequant decode computes ``k_scale * (q . k8)`` and ``p * v_scale`` in
fp32 where the reference first rounds ``k8 * k_scale`` to the compute dtype, so
it is compared with the oracle's attention over the dequantised cache at the
decode tolerances (fp32: rtol 1e-4 / atol 2e-5; fp16 / bf16: max-abs 2e-2 of
max(1, max|ref|)).
"""

import numpy as np
import pytest

import oracle
from helpers import assert_close, to_np, torch_dtype

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import tensorsmith_b200 as ts  # noqa: E402
from tensorsmith_b200 import _lib, engine, nn  # noqa: E402


def host_round(x: np.ndarray, name: str) -> np.ndarray:
    """Round to the compute dtype on the host (torch CPU casts) and return fp32."""
    if name == "float64":
        return np.asarray(x, dtype=np.float64)
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch_dtype(name)).float().numpy()


def cuda_tensor(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to("cuda:0")
    return ts.Tensor(t if dtype is None else t.to(dtype), device="cuda:0")


def test_golden_quant_fixture(golden):
    """The reference's own int8 round trip (two appends of a [2,2,3,16] chunk)."""
    case = golden("quant")
    raw = case["raw"]
    with ts.no_grad():
        cache = nn.KVCache(2, 2, 16, 5, device="cuda:0", quantized=True)
        x = cuda_tensor(raw)
        cache.append(ts.Tensor(x._data[:, :, :2]), ts.Tensor(x._data[:, :, :2]))
        cache.append(ts.Tensor(x._data[:, :, 2:]), ts.Tensor(x._data[:, :, 2:]))
        keys, values, kscale, vscale = cache.storage
        np.testing.assert_array_equal(keys.cpu().numpy(), case["int8"])
        np.testing.assert_array_equal(kscale.cpu().numpy(), case["scales"])
        np.testing.assert_array_equal(cache.get()[0].numpy(), case["deq"])
        assert cache.memory_bytes == int(case["memory_bytes"])
        np.testing.assert_allclose(cache.get()[0].numpy(), raw, atol=0.015)


@pytest.mark.parametrize("name", ["float32", "float16", "bfloat16", "float64"])
@pytest.mark.parametrize("src", ["float32", "same"])
def test_quantising_append_bit_exact(name, src):
    """Chunked appends with ragged channel counts (80 keys, 48 values) and a
    near-zero row (scale floor 1e-8)."""
    rng = np.random.default_rng(7)
    b, h, d, dv, cap = 2, 3, 80, 48, 24
    chunks = [5, 1, 7]
    total = sum(chunks)
    k = (rng.standard_normal((b, h, total, d)) * 3).astype(np.float32)
    v = rng.standard_normal((b, h, total, dv)).astype(np.float32)
    k[1, 2, 3] = 1e-12
    k[0, 0, 6] = 0.0
    host_dtype = np.float64 if name == "float64" else np.float32
    ref = oracle.KVCacheOracle(b, h, d, cap, dtype=host_dtype, quantized=True, value_dim=dv)
    tdt = torch_dtype(name)
    with ts.no_grad():
        cache = nn.KVCache(b, h, d, cap, device="cuda:0", dtype=name, quantized=True, value_dim=dv)
        start = 0
        for n in chunks:
            kc, vc = k[:, :, start : start + n], v[:, :, start : start + n]
            in_dtype = torch.float32 if src == "float32" else tdt
            cache.append(cuda_tensor(kc, in_dtype), cuda_tensor(vc, in_dtype))
            ref.append(host_round(kc, name).astype(host_dtype), host_round(vc, name).astype(host_dtype))
            start += n
        keys, values, ks, vs = cache.storage
        np.testing.assert_array_equal(keys.cpu().numpy(), ref.keys)
        np.testing.assert_array_equal(values.cpu().numpy(), ref.values)
        np.testing.assert_array_equal(ks.cpu().numpy(), ref.key_scales)
        np.testing.assert_array_equal(vs.cpu().numpy(), ref.value_scales)
        gk, gv = cache.get()
        rk, rv = ref.get()
        assert gk.dtype == tdt or str(gk.dtype).endswith(name)
        np.testing.assert_array_equal(to_np(gk._data), host_round(rk, name))
        np.testing.assert_array_equal(to_np(gv._data), host_round(rv, name))
        assert cache.memory_bytes == 2 * b * h * cap * 4 + b * h * cap * (d + dv)


def test_int8_ragged_append_and_reorder():
    rng = np.random.default_rng(11)
    b, h, d, cap = 3, 2, 64, 16
    first = rng.standard_normal((b, h, 4, d)).astype(np.float32)
    second = rng.standard_normal((b, h, 2, d)).astype(np.float32)
    lens = np.array([4, 1, 3])
    with ts.no_grad():
        cache = nn.KVCache(b, h, d, cap, device="cuda:0", quantized=True)
        cache.append(cuda_tensor(first), cuda_tensor(first))
        cache.set_lengths(lens)
        cache.append(cuda_tensor(second), cuda_tensor(second))
        expect_k = np.zeros((b, h, cap, d), np.int8)
        expect_s = np.ones((b, h, cap, 1), np.float32)
        for row in range(b):
            q1, s1 = oracle.quantize_int8(first[row])
            expect_k[row, :, :4], expect_s[row, :, :4] = q1, s1
            q2, s2 = oracle.quantize_int8(second[row])
            n = lens[row]
            expect_k[row, :, n : n + 2], expect_s[row, :, n : n + 2] = q2, s2
        keys, _, ks, _ = cache.storage
        np.testing.assert_array_equal(keys.cpu().numpy(), expect_k)
        np.testing.assert_array_equal(ks.cpu().numpy(), expect_s)
        np.testing.assert_array_equal(cache.lengths, lens + 2)
        cache.reorder([2, 0, 0])
        keys, values, ks, vs = cache.storage
        np.testing.assert_array_equal(keys.cpu().numpy(), expect_k[[2, 0, 0]])
        np.testing.assert_array_equal(values.cpu().numpy(), expect_k[[2, 0, 0]])
        np.testing.assert_array_equal(ks.cpu().numpy(), expect_s[[2, 0, 0]])
        np.testing.assert_array_equal(cache.lengths, (lens + 2)[[2, 0, 0]])


def _int8_problem(name, b, hq, hkv, d, lens, tq, seed):
    rng = np.random.default_rng(seed)
    cap = max(max(lens), 1) + 3
    kf = rng.standard_normal((b, hkv, cap, d)).astype(np.float32)
    vf = rng.standard_normal((b, hkv, cap, d)).astype(np.float32)
    k8, ks = oracle.quantize_int8(kf)
    v8, vs = oracle.quantize_int8(vf)
    q = host_round(rng.standard_normal((b, hq, tq, d)).astype(np.float32), name)
    # What the reference attends over: fp32 products rounded to the compute dtype.
    kd = host_round(k8.astype(np.float32) * ks, name)
    vd = host_round(v8.astype(np.float32) * vs, name)
    return q, k8, ks, v8, vs, kd, vd


def _expected(q, kd, vd, lens, tq):
    outs, lses = [], []
    for row, n in enumerate(lens):
        if n == 0:
            outs.append(np.zeros((1, q.shape[1], tq, vd.shape[3])))
            lses.append(np.full((1, q.shape[1], tq), -np.inf))
            continue
        o, l = oracle.decode_attention(q[row : row + 1].astype(np.float64), kd[row : row + 1].astype(np.float64),
                                       vd[row : row + 1].astype(np.float64), [n], enable_gqa=True)
        outs.append(o)
        lses.append(l)
    return np.concatenate(outs), np.concatenate(lses)


DECODE_CASES = [
    # (dtype, B, Hq, Hkv, D, per-row lengths, query tokens)
    ("float16", 2, 8, 8, 128, [700, 1500], 1),
    ("bfloat16", 2, 16, 2, 128, [4100, 257], 1),  # 8 query heads per KV head: four groups of 2
    ("float32", 3, 4, 2, 64, [33, 2, 900], 2),
    ("float16", 1, 6, 2, 256, [3000], 1),  # 3 rows per KV head: the second group has a dead slot
    ("bfloat16", 3, 4, 4, 64, [0, 50, 31], 1),  # an empty row: zero output, lse -inf
    ("float16", 2, 4, 1, 128, [9000, 8191], 1),
]


@pytest.mark.parametrize("case", DECODE_CASES, ids=lambda c: f"{c[0]}-B{c[1]}-H{c[2]}/{c[3]}-D{c[4]}-T{c[6]}")
def test_fused_int8_decode_matches_oracle(case):
    name, b, hq, hkv, d, lens, tq = case
    q, k8, ks, v8, vs, kd, vd = _int8_problem(name, b, hq, hkv, d, lens, tq, seed=sum(lens) + d)
    dt = torch_dtype(name)
    dev = "cuda:0"
    qg = torch.from_numpy(q).to(dev, dt)
    k8g, v8g = torch.from_numpy(k8).to(dev), torch.from_numpy(v8).to(dev)
    ksg, vsg = torch.from_numpy(ks).to(dev), torch.from_numpy(vs).to(dev)
    kv_len = max(lens)
    lens_g = torch.tensor(lens, dtype=torch.int32, device=dev)
    out, lse = engine.decode_int8(qg, k8g[:, :, :kv_len], v8g[:, :, :kv_len], ksg, vsg, kv_lens=lens_g,
                                  need_lse=True)
    torch.cuda.synchronize()
    engine.check_device_status(dev)
    ref_o, _ = _expected(q, kd, vd, lens, tq)
    assert_close(to_np(out), ref_o, name, "int8 decode output")
    # The kernel never rounds k8 * scale to the compute dtype, so its softmax
    # statistics follow the exactly dequantised cache to fp32 accuracy.
    kx = k8.astype(np.float64) * ks
    vx = v8.astype(np.float64) * vs
    exact_o, exact_l = _expected(q, kx, vx, lens, tq)
    assert_close(to_np(lse), exact_l, "float32", "int8 decode lse (exact dequantisation)")
    if name == "float32":
        assert_close(to_np(out), exact_o, name, "int8 decode output (exact dequantisation)")
    # Against the engine's own decode over the dequantised cache (same device, same dtype).
    kdg = torch.empty((b, hkv, kv_len, d), dtype=dt, device=dev)
    vdg = torch.empty_like(kdg)
    engine.kv_dequant_int8(k8g, ksg, kdg, kv_len)
    engine.kv_dequant_int8(v8g, vsg, vdg, kv_len)
    np.testing.assert_array_equal(to_np(kdg), kd[:, :, :kv_len])
    plain, _ = engine.decode(qg, kdg, vdg, kv_lens=lens_g)
    assert_close(to_np(out), to_np(plain), name, "int8 decode vs dequantised decode")


def test_int8_decode_uniform_length_causal_offset():
    """No kv_lens: every row sees causal_offset + t + 1 keys."""
    name, b, hq, hkv, d, n, tq = "bfloat16", 2, 4, 2, 128, 1000, 2
    q, k8, ks, v8, vs, kd, vd = _int8_problem(name, b, hq, hkv, d, [n] * b, tq, seed=5)
    dt, dev = torch_dtype(name), "cuda:0"
    out, _ = engine.decode_int8(torch.from_numpy(q).to(dev, dt), torch.from_numpy(k8[:, :, :n]).to(dev),
                                torch.from_numpy(v8[:, :, :n]).to(dev), torch.from_numpy(ks).to(dev),
                                torch.from_numpy(vs).to(dev), causal_offset=n - tq)
    ref_o, _ = _expected(q, kd, vd, [n] * b, tq)
    assert_close(to_np(out), ref_o, name, "int8 decode, uniform rows")


def test_int8_decode_rejects_unsupported_shape():
    dev = "cuda:0"
    q = torch.randn(1, 2, 1, 32, device=dev, dtype=torch.float16)
    k8 = torch.zeros(1, 2, 8, 32, dtype=torch.int8, device=dev)
    sc = torch.ones(1, 2, 8, dtype=torch.float32, device=dev)
    with pytest.raises(_lib.EngineError) as info:
        engine.decode_int8(q, k8, k8, sc, sc)
    assert info.value.status == _lib.ERR_UNSUPPORTED


@pytest.mark.parametrize("quantized", [False, True])
@pytest.mark.parametrize("tq,hq,d", [(1, 8, 128), (3, 4, 64), (16, 4, 128), (2, 2, 32)])
def test_cache_attend_matches_sdpa_over_get(quantized, tq, hq, d):
    """KVCache.attend == scaled_dot_product_attention over get() (ragged rows)."""
    rng = np.random.default_rng(tq * 100 + hq + d)
    b, hkv, cap = 2, 2, 600
    name = "float16"
    with ts.no_grad():
        cache = nn.KVCache(b, hkv, d, cap, device="cuda:0", dtype=name, quantized=quantized)
        cache.set_lengths([300, 120])
        # Fill the existing prefixes, then append the query tokens' own keys.
        keys, values, ks, vs = cache.storage
        pre = rng.standard_normal((b, hkv, 300, d)).astype(np.float32)
        if quantized:
            k8, s8 = oracle.quantize_int8(pre)
            keys[:, :, :300] = torch.from_numpy(k8).cuda()
            values[:, :, :300] = torch.from_numpy(k8).cuda()
            ks[:, :, :300] = torch.from_numpy(s8).cuda()
            vs[:, :, :300] = torch.from_numpy(s8).cuda()
        else:
            keys[:, :, :300] = torch.from_numpy(pre).cuda().half()
            values[:, :, :300] = torch.from_numpy(pre).cuda().half()
        new = rng.standard_normal((b, hkv, tq, d)).astype(np.float32)
        cache.append(cuda_tensor(new, torch.float16), cuda_tensor(new, torch.float16))
        query = cuda_tensor(rng.standard_normal((b, hq, tq, d)).astype(np.float32), torch.float16)
        got = cache.attend(query)
        kk, vv = cache.get()
        lens = cache.lengths
        ref = np.concatenate([
            oracle.decode_attention(to_np(query._data)[r : r + 1].astype(np.float64),
                                    to_np(kk._data)[r : r + 1].astype(np.float64),
                                    to_np(vv._data)[r : r + 1].astype(np.float64), [lens[r]], enable_gqa=True)[0]
            for r in range(b)
        ])
        assert_close(to_np(got._data), ref, name, f"attend quantized={quantized}")


def test_quantized_append_rotary_matches_rope_then_quantise():
    rng = np.random.default_rng(3)
    b, h, d, cap, n = 2, 2, 64, 32, 5
    x = rng.standard_normal((b, h, n, d)).astype(np.float32)
    with ts.no_grad():
        cache = nn.KVCache(b, h, d, cap, device="cuda:0", quantized=True)
        cache.append(cuda_tensor(x[:, :, :2]), cuda_tensor(x[:, :, :2]))
        cache.append_rotary(cuda_tensor(x[:, :, 2:]), cuda_tensor(x[:, :, 2:]))
        rotated = to_np(engine.rope(torch.from_numpy(x[:, :, 2:]).cuda(), offset=2))
        np.testing.assert_allclose(rotated, oracle.rope(x[:, :, 2:], 2), rtol=1e-5, atol=1e-5)
        q8, s8 = oracle.quantize_int8(rotated)
        keys, values, ks, _ = cache.storage
        np.testing.assert_array_equal(keys[:, :, 2:n].cpu().numpy(), q8)
        np.testing.assert_array_equal(ks[:, :, 2:n].cpu().numpy(), s8)
        np.testing.assert_array_equal(values[:, :, 2:n].cpu().numpy(), oracle.quantize_int8(x[:, :, 2:])[0])
