"""Pin the CPU oracle against outputs of the tensorsmith reference itself.

The fixtures under tests/golden/ were produced by tests/golden/make_golden.py,
which calls the reference's public API.  Every oracle function used as the
checker of the CUDA kernels is compared here first.
"""

import numpy as np
import pytest

import oracle


def _grads(case, prefix, fwd_kw, bwd_kw=None, mask=None):
    bwd_kw = fwd_kw if bwd_kw is None else bwd_kw
    out, lse = oracle.attention_forward(case["q"], case["k"], case["v"], mask, **fwd_kw)
    dq, dk, dv = oracle.attention_backward(case["q"], case["k"], case["v"], out, lse, case["dout"],
                                           mask, **bwd_kw)
    return out, dq, dk, dv


def _check(got, case, prefix, rtol, atol):
    for key, val in zip(("out", "dq", "dk", "dv"), got):
        np.testing.assert_allclose(val, case[f"{prefix}_{key}"], rtol=rtol, atol=atol, err_msg=f"{prefix} {key}")


def test_vjp_offset_fp64(golden):
    case = golden("vjp_offset")
    for algorithm in ("dense", "streaming"):
        kw = dict(is_causal=True, causal_offset=2)
        got = _grads(case, algorithm, dict(kw, algorithm=algorithm, block_size=2), dict(kw, block_size=2))
        _check(got, case, algorithm, 1e-12, 1e-12)
        dense_bwd = oracle.attention_backward_dense(case["q"], case["k"], case["v"], case["dout"], **kw)
        for key, val in zip(("dq", "dk", "dv"), dense_bwd):
            np.testing.assert_allclose(val, case[f"dense_{key}"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("kind", ["bool", "float"])
@pytest.mark.parametrize("algorithm", ["dense", "streaming"])
def test_masks_fully_masked_row(golden, kind, algorithm):
    case = golden("masks")
    mask = case[f"{kind}_mask"]
    got = _grads(case, None, dict(is_causal=True, algorithm=algorithm, block_size=2),
                 dict(is_causal=True, block_size=2), mask=mask)
    _check(got, case, f"{algorithm}_{kind}", 1e-5, 1e-6)
    assert np.all(got[0][:, :, 1] == 0) and np.all(got[1][:, :, 1] == 0)
    _, lse = oracle.attention_forward(case["q"], case["k"], case["v"], mask, is_causal=True)
    assert np.all(np.isneginf(lse[:, :, 1])) and np.all(np.isfinite(lse[:, :, [0, 2, 3]]))


@pytest.mark.parametrize("tag", ["full", "causal"])
def test_gqa(golden, tag):
    case = golden("gqa")
    kw = dict(is_causal=tag == "causal", enable_gqa=True, block_size=2)
    got = _grads(case, tag, kw)
    _check(got, case, tag, 1e-5, 1e-6)


@pytest.mark.parametrize("tag", ["full", "causal"])
def test_unmasked(golden, tag):
    case = golden("unmasked")
    got = _grads(case, tag, dict(is_causal=tag == "causal"))
    _check(got, case, tag, 1e-5, 1e-6)


def test_c1_config(golden):
    case = golden("c1")
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((2, 4, 256, 64), dtype=np.float32) for _ in range(3))
    dout = rng.standard_normal((2, 4, 256, 64), dtype=np.float32)
    out, lse = oracle.attention_forward(q, k, v, is_causal=True)
    dq, dk, dv = oracle.attention_backward(q, k, v, out, lse, dout, is_causal=True)
    step = int(case["rows_step"])
    for key, val in zip(("out", "dq", "dk", "dv"), (out, dq, dk, dv)):
        np.testing.assert_allclose(val[:, :, ::step], case[key], rtol=1e-4, atol=2e-5, err_msg=key)
    sums = np.array([float(np.sum(x, dtype=np.float64)) for x in (out, dq, dk, dv)])
    np.testing.assert_allclose(sums, case["checksums"], rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("algorithm", ["dense", "streaming"])
def test_half_inputs(golden, algorithm):
    case = golden("half")
    out, lse = oracle.attention_forward(case["q"], case["k"], case["v"], is_causal=True,
                                        algorithm=algorithm, block_size=16)
    dq, dk, dv = oracle.attention_backward(case["q"], case["k"], case["v"], out, lse, case["dout"],
                                           is_causal=True, block_size=16)
    for key, val in zip(("out", "dq", "dk", "dv"), (out, dq, dk, dv)):
        ref = case[f"{algorithm}_{key}"].astype(np.float32)
        np.testing.assert_allclose(val.astype(np.float16).astype(np.float32), ref, rtol=2e-3, atol=2e-3)


def test_cache_chunked_decode(golden):
    case = golden("cache")
    q, k, v = case["q"], case["k"], case["v"]
    b, h, _, d = q.shape
    cache = oracle.KVCacheOracle(b, h, d, int(case["capacity"]))
    outs, start = [], 0
    for n in case["chunks"]:
        offset = cache.length
        keys, values = cache.append(k[:, :, start : start + n], v[:, :, start : start + n])
        o, _ = oracle.attention_forward(q[:, :, start : start + n], keys, values, is_causal=True,
                                        causal_offset=offset)
        outs.append(o)
        start += n
    np.testing.assert_allclose(np.concatenate(outs, axis=2), case["out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(cache.get()[0], case["keys"])
    cache.reorder(np.array([1, 0]))
    np.testing.assert_array_equal(cache.get()[0], case["reordered_keys"])
    cache.truncate(4)
    assert cache.length == int(case["truncated_len"])
    with pytest.raises(ValueError):
        cache.append(k, v)


def test_ragged_decode(golden):
    case = golden("ragged")
    mask = oracle.key_valid_mask(case["lengths"], case["k"].shape[2])
    out, _ = oracle.attention_forward(case["q"], case["k"], case["v"], mask, enable_gqa=True)
    np.testing.assert_allclose(out, case["out"], rtol=1e-5, atol=1e-6)
    # the per-row-length decode formulation equals the masked one for one query token
    dec, _ = oracle.decode_attention(case["q"], case["k"], case["v"], case["lengths"], enable_gqa=True)
    np.testing.assert_allclose(dec, case["out"], rtol=1e-5, atol=1e-6)


def test_rope(golden):
    case = golden("rope")
    np.testing.assert_allclose(oracle.rope(case["x1"], offset=5, rotary_dim=4), case["y1"], rtol=1e-12)
    np.testing.assert_allclose(oracle.rope(case["x2"], offset=3), case["y2"], rtol=1e-6, atol=1e-7)


def test_quantized_cache(golden):
    case = golden("quant")
    raw = case["raw"]
    cache = oracle.KVCacheOracle(2, 2, 16, 5, quantized=True)
    cache.append(raw[:, :, :2], raw[:, :, :2])
    cache.append(raw[:, :, 2:], raw[:, :, 2:])
    np.testing.assert_array_equal(cache.keys[:, :, :3], case["int8"][:, :, :3])
    np.testing.assert_allclose(cache.get()[0], case["deq"], rtol=1e-6, atol=1e-7)


def test_causal_pairs_formula():
    assert oracle.causal_pairs(2, 4, 256, 256, 0) == 8 * 32896
    assert oracle.causal_pairs(1, 1, 3, 5, 2) == 3 + 4 + 5


@pytest.mark.parametrize("name", ["float32", "float64"])
def test_dropout_dense(golden, name):
    """The reference's dense dropout forward + VJP with the mask it drew."""
    case = golden("dropout")
    q, k, v, g = (case[f"{name}_{x}"] for x in ("q", "k", "v", "dout"))
    keep = case[f"{name}_keep"]
    kw = dict(is_causal=True, causal_offset=2, dropout_keep=keep, dropout_p=0.3)
    out, _ = oracle.attention_forward(q, k, v, algorithm="dense", **kw)
    dq, dk, dv = oracle.attention_backward_dense(q, k, v, g, **kw)
    tol = dict(rtol=1e-5, atol=1e-6) if name == "float32" else dict(rtol=1e-12, atol=1e-13)
    for got, ref in ((out, "out"), (dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(got, case[f"{name}_{ref}"], err_msg=ref, **tol)
    # Without the mask the outputs differ: the fixture really holds a dropped draw.
    plain, _ = oracle.attention_forward(q, k, v, algorithm="dense", is_causal=True, causal_offset=2)
    assert not np.allclose(plain, case[f"{name}_out"])
