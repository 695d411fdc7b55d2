"""Rotary embedding (nn/attention.py:255-296) and the fused RoPE + KV append,
through the C ABI, against the oracle and the reference's golden outputs."""

import numpy as np
import pytest

import oracle
from helpers import assert_close, rounded, to_cuda, to_np

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import tensorsmith_b200 as ts  # noqa: E402
from tensorsmith_b200 import engine, nn  # noqa: E402

# cos/sin of the same fp32 angle (CUDA sincosf vs NumPy) may differ by one fp32
# ulp, so fp64 inputs agree to ~1e-7, not to fp64 precision.
ROPE_TOL = {"float32": dict(rtol=2e-6, atol=2e-6), "float64": dict(rtol=3e-7, atol=3e-7)}


def _np_rope(x, name, offset, dim=None):
    """Oracle on the storage dtype itself (per-operation rounding like the reference)."""
    if name in ("float16", "bfloat16"):
        from helpers import np_dtype

        xs = x.astype(np_dtype(name))
        return oracle.rope(xs, offset=offset, rotary_dim=dim).astype(np.float64)
    return oracle.rope(x.astype(name), offset=offset, rotary_dim=dim)


@pytest.mark.parametrize("name", ["float32", "float64", "float16", "bfloat16"])
@pytest.mark.parametrize("offset,dim", [(0, None), (5, 32), (32768, None), (8191, 64)])
def test_rope_matches_oracle(name, offset, dim):
    rng = np.random.default_rng(3)
    x = rounded(rng.standard_normal((2, 3, 17, 64)), name)
    ref = _np_rope(x, name, offset, dim)
    got = to_np(engine.rope(to_cuda(x, name), offset=offset, rotary_dim=dim))
    if name in ROPE_TOL:
        np.testing.assert_allclose(got, ref, **ROPE_TOL[name])
    else:
        # one storage ulp: cos/sin of the same fp32 angle may round differently
        assert_close(got, ref, name, "rope")
    # the inverse rotation undoes the rotation (up to storage rounding)
    back = to_np(engine.rope(engine.rope(to_cuda(x, name), offset=offset, rotary_dim=dim), offset=offset,
                             rotary_dim=dim, inverse=True))
    assert_close(back, x, name if name not in ROPE_TOL else "bfloat16", "inverse", scaled=True)


def test_rope_golden_and_vjp(golden):
    case = golden("rope")
    x1 = ts.Tensor(case["x1"], device="cuda:0", requires_grad=True)
    y1 = nn.rotary_embedding(x1, offset=5, rotary_dim=4)
    np.testing.assert_allclose(y1.numpy(), case["y1"], rtol=3e-7, atol=3e-7)
    x2 = ts.Tensor(case["x2"], device="cuda:0")
    np.testing.assert_allclose(nn.rotary_embedding(x2, offset=3).numpy(), case["y2"], rtol=2e-6, atol=2e-6)
    # VJP of a rotation is the inverse rotation: <R x, g> == <x, R^T g>
    g = np.random.default_rng(1).standard_normal(case["x1"].shape)
    y1.backward(ts.Tensor(g, device="cuda:0"))
    lhs = float(np.sum(case["y1"] * g))
    rhs = float(np.sum(case["x1"] * x1.grad.numpy()))
    assert abs(lhs - rhs) < 1e-10


@pytest.mark.parametrize("ragged", [False, True])
def test_fused_rope_append_equals_rope_then_append(ragged):
    rng = np.random.default_rng(9)
    b, h, d, cap = 3, 4, 128, 64
    with ts.no_grad():
        fused = nn.KVCache(b, h, d, cap, device="cuda:0", dtype="bfloat16")
        plain = nn.KVCache(b, h, d, cap, device="cuda:0", dtype="bfloat16")
        if ragged:
            fused.set_lengths([3, 0, 10])
            plain_lens = np.array([3, 0, 10])
        for steps in (5, 1, 2):
            k = rounded(rng.standard_normal((b, h, steps, d)), "bfloat16")
            v = rounded(rng.standard_normal((b, h, steps, d)), "bfloat16")
            kt, vt = ts.Tensor(to_cuda(k, "bfloat16")), ts.Tensor(to_cuda(v, "bfloat16"))
            fused.append_rotary(kt, vt)
            if ragged:
                # reference formulation row by row: rotate at the row's own offset, then write
                for row in range(b):
                    n = int(plain_lens[row])
                    kr = engine.rope(kt._data[row : row + 1], offset=n)
                    plain._keys[row : row + 1, :, n : n + steps] = kr
                    plain._values[row : row + 1, :, n : n + steps] = vt._data[row : row + 1]
                plain_lens += steps
            else:
                plain.append(nn.rotary_embedding(kt, offset=plain.length), vt)
        torch.cuda.synchronize()
        engine.check_device_status()
        assert torch.equal(fused.storage[0], plain.storage[0])
        assert torch.equal(fused.storage[1], plain.storage[1])
