"""KVCache, tape and SDPA API parity with tensorsmith's behaviour (GPU).

Mirrors tests/test_transformer.py:247-285 and :305-337 of the reference, and
checks the engine against the committed golden outputs of the reference.
"""

import numpy as np
import pytest

import oracle
from helpers import assert_close, to_np

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import tensorsmith_b200 as ts  # noqa: E402
from tensorsmith_b200 import nn  # noqa: E402


def cuda_tensor(x, **kw):
    return ts.Tensor(np.asarray(x), device="cuda:0", **kw)


def test_cache_storage_reset_reorder_and_capacity():
    raw = np.random.default_rng(1).standard_normal((2, 2, 3, 16)).astype(np.float32)
    with ts.no_grad():
        cache = nn.KVCache(2, 2, 16, 5, device="cuda:0")
        x = cuda_tensor(raw)
        cache.append(ts.Tensor(x._data[:, :, :2]), ts.Tensor(x._data[:, :, :2]))
        cache.append(ts.Tensor(x._data[:, :, 2:]), ts.Tensor(x._data[:, :, 2:]))
        np.testing.assert_array_equal(cache.get()[0].numpy(), raw)
        cache.reorder([1, 1])
        np.testing.assert_array_equal(cache.get()[0].numpy(), raw[[1, 1]])
        with pytest.raises(ValueError):
            cache.append(x, x)
        assert cache.length == 3
        cache.truncate(2)
        assert cache.get()[0].shape[2] == 2
        cache.reset()
        assert cache.get()[0].shape[2] == 0
        cache.append(x, x)
        np.testing.assert_array_equal(cache.get()[0].numpy(), raw)
        assert cache.memory_bytes == 2 * 2 * 2 * 5 * 16 * 4


def test_cache_requires_inference():
    cache = nn.KVCache(1, 2, 4, 8, device="cuda:0")
    x = cuda_tensor(np.ones((1, 2, 2, 4), np.float32), requires_grad=True)
    with pytest.raises(RuntimeError):
        cache.append(x, x)
    with ts.no_grad():
        cache.append(x, x)
    assert cache.length == 2


def test_golden_cache_chunked_decode(golden):
    case = golden("cache")
    q, k, v = case["q"], case["k"], case["v"]
    b, h, _, d = q.shape
    outs, start = [], 0
    with ts.no_grad():
        cache = nn.KVCache(b, h, d, int(case["capacity"]), device="cuda:0")
        for n in case["chunks"]:
            offset = cache.length
            kk, vv = cache.append(cuda_tensor(k[:, :, start : start + n]), cuda_tensor(v[:, :, start : start + n]))
            o = nn.scaled_dot_product_attention(cuda_tensor(q[:, :, start : start + n]), kk, vv,
                                                is_causal=True, causal_offset=offset)
            outs.append(o.numpy())
            start += n
        np.testing.assert_allclose(np.concatenate(outs, axis=2), case["out"], rtol=1e-4, atol=2e-5)
        np.testing.assert_array_equal(cache.get()[0].numpy(), case["keys"])
        cache.reorder([1, 0])
        np.testing.assert_array_equal(cache.get()[0].numpy(), case["reordered_keys"])


def test_golden_ragged_decode_via_mask_and_lengths(golden):
    case = golden("ragged")
    q, k, v, lens = case["q"], case["k"], case["v"], case["lengths"]
    mask = oracle.key_valid_mask(lens, k.shape[2])
    with ts.no_grad():
        o_mask = nn.scaled_dot_product_attention(cuda_tensor(q), cuda_tensor(k), cuda_tensor(v),
                                                 cuda_tensor(mask), enable_gqa=True)
        kv_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
        o_lens = nn.scaled_dot_product_attention(cuda_tensor(q), cuda_tensor(k), cuda_tensor(v),
                                                 enable_gqa=True, is_causal=True, kv_lens=kv_lens)
    np.testing.assert_allclose(o_mask.numpy(), case["out"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(o_lens.numpy(), case["out"], rtol=1e-4, atol=2e-5)


def test_ragged_cache_append_positions():
    rng = np.random.default_rng(3)
    b, h, d, cap = 3, 2, 64, 40
    with ts.no_grad():
        cache = nn.KVCache(b, h, d, cap, device="cuda:0", dtype="float16")
        cache.set_lengths([5, 0, 17])
        host_k = np.zeros((b, h, cap, d), np.float16)
        lens = np.array([5, 0, 17])
        for step in range(3):
            kv = rng.standard_normal((b, h, 1, d)).astype(np.float16)
            cache.append(cuda_tensor(kv), cuda_tensor(kv))
            for row in range(b):
                host_k[row, :, lens[row]] = kv[row, :, 0]
            lens += 1
        torch.cuda.synchronize()
        np.testing.assert_array_equal(cache.lengths, lens)
        np.testing.assert_array_equal(cache.seq_lens.cpu().numpy(), lens)
        keys = cache.storage[0].float().cpu().numpy()
        for row in range(b):
            np.testing.assert_array_equal(keys[row, :, lens[row] - 3 : lens[row]],
                                          host_k[row, :, lens[row] - 3 : lens[row]].astype(np.float32))


@pytest.mark.parametrize("golden_name,kw", [
    ("vjp_offset", dict(is_causal=True, causal_offset=2)),
])
def test_golden_vjp_fp64(golden, golden_name, kw):
    case = golden(golden_name)
    tensors = [cuda_tensor(case[n], requires_grad=True) for n in ("q", "k", "v")]
    out = nn.scaled_dot_product_attention(*tensors, **kw)
    out.backward(cuda_tensor(case["dout"]))
    for name, got in zip(("out", "dq", "dk", "dv"), [out] + [t.grad for t in tensors]):
        np.testing.assert_allclose(got.numpy(), case[f"streaming_{name}"], rtol=1e-9, atol=1e-11)


@pytest.mark.parametrize("kind", ["bool", "float"])
def test_golden_masks(golden, kind):
    case = golden("masks")
    tensors = [cuda_tensor(case[n], requires_grad=True) for n in ("q", "k", "v")]
    out = nn.scaled_dot_product_attention(*tensors, cuda_tensor(case[f"{kind}_mask"]), is_causal=True)
    out.backward(cuda_tensor(case["dout"]))
    for name, got in zip(("out", "dq", "dk", "dv"), [out] + [t.grad for t in tensors]):
        np.testing.assert_allclose(got.numpy(), case[f"streaming_{kind}_{name}"], rtol=1e-4, atol=3e-5)


@pytest.mark.parametrize("tag", ["full", "causal"])
def test_golden_gqa_and_unmasked(golden, tag):
    for name, gqa in (("gqa", True), ("unmasked", False)):
        case = golden(name)
        tensors = [cuda_tensor(case[n], requires_grad=True) for n in ("q", "k", "v")]
        out = nn.scaled_dot_product_attention(*tensors, is_causal=tag == "causal", enable_gqa=gqa)
        out.backward(cuda_tensor(case["dout"]))
        for key, got in zip(("out", "dq", "dk", "dv"), [out] + [t.grad for t in tensors]):
            np.testing.assert_allclose(got.numpy(), case[f"{tag}_{key}"], rtol=2e-4, atol=4e-5)


def test_golden_c1_config(golden):
    case = golden("c1")
    rng = np.random.default_rng(0)
    raw = [rng.standard_normal((2, 4, 256, 64), dtype=np.float32) for _ in range(3)]
    up = rng.standard_normal((2, 4, 256, 64), dtype=np.float32)
    tensors = [cuda_tensor(a, requires_grad=True) for a in raw]
    out = nn.scaled_dot_product_attention(*tensors, is_causal=True)
    out.backward(cuda_tensor(up))
    step = int(case["rows_step"])
    for key, got in zip(("out", "dq", "dk", "dv"), [out] + [t.grad for t in tensors]):
        np.testing.assert_allclose(got.numpy()[:, :, ::step], case[key], rtol=1e-4, atol=2e-5, err_msg=key)


def test_golden_half_inputs(golden):
    case = golden("half")
    tensors = [cuda_tensor(case[n], requires_grad=True) for n in ("q", "k", "v")]
    out = nn.scaled_dot_product_attention(*tensors, is_causal=True)
    out.backward(cuda_tensor(case["dout"]))
    for key, got in zip(("out", "dq", "dk", "dv"), [out] + [t.grad for t in tensors]):
        assert_close(got.numpy(), case[f"streaming_{key}"].astype(np.float32), "float16", key, scaled=key != "out")


def test_no_grad_returns_plain_tensor_and_permute_vjp():
    rng = np.random.default_rng(4)
    x = [cuda_tensor(rng.standard_normal((1, 5, 2, 8)).astype(np.float32), requires_grad=True) for _ in range(3)]
    q, k, v = (t.permute(0, 2, 1, 3) for t in x)
    with ts.no_grad():
        plain = nn.scaled_dot_product_attention(q, k, v, is_causal=True)
    assert not plain.requires_grad
    out = nn.scaled_dot_product_attention(q, k, v, is_causal=True)
    assert out.requires_grad and out._op == "sdpa_native"
    out.backward(cuda_tensor(np.ones(out.shape, np.float32)))
    assert x[0].grad.shape == (1, 5, 2, 8)


def test_api_validation_messages():
    q = cuda_tensor(np.zeros((1, 4, 3, 8), np.float32))
    k = cuda_tensor(np.zeros((1, 2, 5, 8), np.float32))
    with pytest.raises(ValueError, match="grouped-query attention requires enable_gqa"):
        nn.scaled_dot_product_attention(q, k, k)
    with pytest.raises(ValueError, match="attention backend must be"):
        nn.scaled_dot_product_attention(q, k, k, enable_gqa=True, backend="flash")
    with pytest.raises(ValueError, match="invalid dropout probability"):
        nn.scaled_dot_product_attention(q, k, k, enable_gqa=True, causal_offset=-1)
