"""Backward parity: engine dQ/dK/dV (through the C ABI) vs the oracle's VJP
(LSE-recomputed blockwise VJP of nn/attention.py:220-247, GQA-reduced)."""

import numpy as np
import pytest

from helpers import assert_close, oracle_backward, rounded, to_cuda, to_np

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from tensorsmith_b200 import engine  # noqa: E402

SHAPES = [
    (1, 2, 2, 3, 5, 4, 3, True, 2),
    (1, 4, 2, 3, 5, 4, 4, False, 0),
    (1, 2, 2, 7, 7, 8, 8, True, 0),
    (2, 4, 4, 256, 256, 64, 64, True, 0),
    (1, 2, 1, 65, 127, 32, 48, True, 62),
    (1, 2, 2, 130, 130, 128, 128, True, 0),
]


def _case(shape, name, seed):
    b, hq, hkv, tq, tk, d, dv, causal, off = shape
    rng = np.random.default_rng(seed)
    q = rounded(rng.standard_normal((b, hq, tq, d)), name)
    k = rounded(rng.standard_normal((b, hkv, tk, d)), name)
    v = rounded(rng.standard_normal((b, hkv, tk, dv)), name)
    g = rounded(rng.standard_normal((b, hq, tq, dv)), name)
    return q, k, v, g


@pytest.mark.parametrize("name", ["float32", "float64", "float16", "bfloat16"])
@pytest.mark.parametrize("shape", SHAPES, ids=str)
def test_backward(shape, name):
    b, hq, hkv, tq, tk, d, dv, causal, off = shape
    q, k, v, g = _case(shape, name, 3)
    kw = dict(is_causal=causal, causal_offset=off, enable_gqa=hq != hkv)
    _, _, (rdq, rdk, rdv) = oracle_backward(q, k, v, g, **kw)
    tq_, tk_, tv_, tg = (to_cuda(x, name) for x in (q, k, v, g))
    out, lse = engine.forward(tq_, tk_, tv_, is_causal=causal, causal_offset=off)
    dq, dk, dv_ = engine.backward(tq_, tk_, tv_, out, lse, tg, is_causal=causal, causal_offset=off)
    torch.cuda.synchronize()
    engine.check_device_status()
    assert_close(to_np(dq), rdq, name, f"dq {shape}", scaled=True)
    assert_close(to_np(dk), rdk, name, f"dk {shape}", scaled=True)
    assert_close(to_np(dv_), rdv, name, f"dv {shape}", scaled=True)


@pytest.mark.parametrize("kind", ["bool", "float"])
def test_backward_masked_rows_have_zero_grad(kind):
    rng = np.random.default_rng(11)
    q, k, v, g = (rng.standard_normal((2, 2, 4, 4)).astype(np.float32) for _ in range(4))
    boolean = np.ones((4, 4), dtype=bool)
    boolean[1] = False
    boolean[3, 0] = False
    mask = boolean if kind == "bool" else np.where(boolean, 0, -np.inf).astype(np.float32)
    _, _, (rdq, rdk, rdv) = oracle_backward(q, k, v, g, mask=mask, is_causal=True)
    tm = torch.from_numpy(mask).cuda()
    tq_, tk_, tv_, tg = (to_cuda(x, "float32") for x in (q, k, v, g))
    out, lse = engine.forward(tq_, tk_, tv_, is_causal=True, mask=tm)
    dq, dk, dv_ = engine.backward(tq_, tk_, tv_, out, lse, tg, is_causal=True, mask=tm)
    assert_close(to_np(dq), rdq, "float32", "dq")
    assert_close(to_np(dk), rdk, "float32", "dk")
    assert_close(to_np(dv_), rdv, "float32", "dv")
    assert np.all(to_np(dq)[:, :, 1] == 0)


TC_SHAPES = [
    (1, 2, 2, 128, 128, 128, 128, True, 0),
    (1, 2, 2, 128, 128, 128, 128, False, 0),
    (2, 3, 3, 200, 200, 64, 64, True, 0),
    (1, 4, 2, 300, 333, 128, 128, True, 33),   # GQA + offset + ragged tiles
    (1, 2, 2, 100, 700, 64, 64, False, 0),
    (1, 8, 1, 257, 257, 128, 128, True, 0),    # rep 8
    (1, 2, 2, 1024, 1024, 128, 128, True, 0),
]


@pytest.mark.parametrize("name", ["bfloat16", "float16"])
@pytest.mark.parametrize("shape", TC_SHAPES, ids=str)
def test_backward_tcgen05(shape, name):
    b, hq, hkv, tq, tk, d, dv, causal, off = shape
    q, k, v, g = _case(shape, name, 5)
    kw = dict(is_causal=causal, causal_offset=off, enable_gqa=hq != hkv)
    _, _, (rdq, rdk, rdv) = oracle_backward(q, k, v, g, **kw)
    tq_, tk_, tv_, tg = (to_cuda(x, name) for x in (q, k, v, g))
    out, lse = engine.forward(tq_, tk_, tv_, is_causal=causal, causal_offset=off)
    assert engine.bwd_path(tq_, tk_, tv_, out, lse, tg, is_causal=causal, causal_offset=off) == "tcgen05"
    dq, dk, dv_ = engine.backward(tq_, tk_, tv_, out, lse, tg, is_causal=causal, causal_offset=off)
    torch.cuda.synchronize()
    engine.check_device_status()
    assert_close(to_np(dq), rdq, name, f"dq {shape}", scaled=True)
    assert_close(to_np(dk), rdk, name, f"dk {shape}", scaled=True)
    assert_close(to_np(dv_), rdv, name, f"dv {shape}", scaled=True)


def test_backward_tcgen05_kv_lens_and_btdh_views():
    rng = np.random.default_rng(13)
    b, t, h, d = 3, 200, 2, 128
    lens = np.array([200, 77, 130])
    base = [rounded(rng.standard_normal((b, t, h, d)), "bfloat16") for _ in range(4)]
    q, k, v, g = (to_cuda(x, "bfloat16").permute(0, 2, 1, 3) for x in base)
    kv_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out, lse = engine.forward(q, k, v, is_causal=True, kv_lens=kv_lens)
    assert engine.bwd_path(q, k, v, out, lse, g, is_causal=True, kv_lens=kv_lens) == "tcgen05"
    dq, dk, dv_ = engine.backward(q, k, v, out, lse, g, is_causal=True, kv_lens=kv_lens)
    torch.cuda.synchronize()
    for row in range(b):
        n = int(lens[row])
        qn, kn, vn, gn = (x[row : row + 1].transpose(0, 2, 1, 3) for x in base)
        # keys past the row's length are masked; queries sit at the end of the valid keys
        mask = np.arange(t)[None, None, None, :] < n
        _, _, (rdq, rdk, rdv) = oracle_backward(qn, kn, vn, gn, mask=mask, is_causal=True, causal_offset=n - t)
        assert_close(to_np(dq[row : row + 1]), rdq, "bfloat16", f"dq row {row}", scaled=True)
        assert_close(to_np(dk[row : row + 1]), rdk, "bfloat16", f"dk row {row}", scaled=True)
        assert_close(to_np(dv_[row : row + 1]), rdv, "bfloat16", f"dv row {row}", scaled=True)
