"""In-kernel attention dropout against the oracle (nn/attention.py:140-144, 212-216).

The engine draws its keep mask from a counter-based generator; the tests
materialise that mask (``engine.dropout_mask``, the same generator the kernels
call) and give it to the oracle's dense dropout forward / VJP, which is pinned
to the reference's own dropout fixture in test_oracle_golden.py.
"""

import numpy as np
import pytest

import oracle
from helpers import TOL, assert_close, rounded, to_cuda, to_np

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import tensorsmith_b200 as ts  # noqa: E402
from tensorsmith_b200 import engine, nn  # noqa: E402


def test_mask_statistics_and_determinism():
    b, h, tq, tk, p = 2, 3, 64, 300, 0.3
    m0 = engine.dropout_mask(b, h, tq, tk, (p, 1234, 0), "cuda:0").cpu().numpy()
    again = engine.dropout_mask(b, h, tq, tk, (p, 1234, 0), "cuda:0").cpu().numpy()
    m1 = engine.dropout_mask(b, h, tq, tk, (p, 1234, 1), "cuda:0").cpu().numpy()
    m2 = engine.dropout_mask(b, h, tq, tk, (p, 99, 0), "cuda:0").cpu().numpy()
    np.testing.assert_array_equal(m0, again)
    n = m0.size
    for m in (m0, m1, m2):
        assert set(np.unique(m)) <= {0, 1}
        # keep fraction within 5 standard deviations of 1 - p
        assert abs(m.mean() - (1 - p)) < 5 * np.sqrt(p * (1 - p) / n)
    assert (m0 != m1).mean() > 0.3 and (m0 != m2).mean() > 0.3
    # neighbouring keys, rows and heads are uncorrelated
    x = m0.astype(np.float64) - m0.mean()
    for a, c in ((x[..., 1:], x[..., :-1]), (x[:, :, 1:], x[:, :, :-1]), (x[:, 1:], x[:, :-1])):
        assert abs(np.mean(a * c)) / x.var() < 0.05
    assert engine.dropout_mask(1, 1, 4, 9, (0.0, 5, 0), "cuda:0").cpu().numpy().all()


CASES = [
    # (dtype, B, Hq, Hkv, Tq, Tk, D, Dv, causal, offset, mask)
    ("float32", 2, 4, 4, 37, 53, 64, 64, True, 16, None),
    ("float64", 1, 2, 2, 9, 13, 16, 8, True, 4, None),
    ("float16", 2, 4, 2, 70, 70, 128, 128, True, 0, None),
    ("bfloat16", 1, 4, 1, 33, 129, 64, 32, False, 0, "bool"),
    ("float32", 1, 2, 2, 16, 40, 32, 32, False, 0, "float"),
]


def _mask(kind, b, h, tq, tk, rng):
    if kind is None:
        return None, None
    allowed = rng.random((b, 1, tq, tk)) > 0.2
    allowed[:, :, 3] = False  # a fully masked row: zero output and gradients
    if kind == "bool":
        return allowed, torch.from_numpy(allowed).cuda()
    add = np.where(allowed, rng.normal(size=allowed.shape) * 0.5, -np.inf)
    return add, torch.from_numpy(add.astype(np.float32)).cuda()


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-H{c[2]}/{c[3]}-T{c[4]}x{c[5]}-{c[10]}")
@pytest.mark.parametrize("p", [0.1, 0.5])
def test_dropout_forward_backward_match_oracle(case, p):
    name, b, hq, hkv, tq, tk, d, dv, causal, offset, mask_kind = case
    rng = np.random.default_rng(tq * 1000 + tk + int(p * 10) + d)
    q, k, v = (rng.normal(size=s) for s in ((b, hq, tq, d), (b, hkv, tk, d), (b, hkv, tk, dv)))
    g = rng.normal(size=(b, hq, tq, dv))
    host_mask, dev_mask = _mask(mask_kind, b, hq, tq, tk, rng)
    qr, kr, vr, gr = (rounded(x, name) for x in (q, k, v, g))
    tq_, tk_, tv_, tg_ = (to_cuda(x, name) for x in (q, k, v, g))
    args = (p, 777, 41)
    kw = dict(is_causal=causal, causal_offset=offset, mask=dev_mask)
    out, lse = engine.forward(tq_, tk_, tv_, dropout=args, **kw)
    dq, dk, dvv = engine.backward(tq_, tk_, tv_, out, lse, tg_, dropout=args, **kw)
    torch.cuda.synchronize()
    keep = engine.dropout_mask(b, hq, tq, tk, args, "cuda:0").cpu().numpy().astype(bool)
    okw = dict(is_causal=causal, causal_offset=offset, enable_gqa=hq != hkv, dropout_keep=keep, dropout_p=p)
    ref_o, ref_l = oracle.attention_forward(qr, kr, vr, host_mask, algorithm="dense", **okw)
    assert_close(to_np(out), ref_o, name, "dropout out")
    assert_close(to_np(lse), ref_l, "float64" if name == "float64" else "float32", "dropout lse")
    # The backward's Delta uses the stored (dtype-rounded) output, as the engine does.
    rdq, rdk, rdv = oracle.attention_backward_dense(qr, kr, vr, gr, host_mask, **okw)
    for got, ref, what in ((dq, rdq, "dq"), (dk, rdk, "dk"), (dvv, rdv, "dv")):
        assert_close(to_np(got), ref, name, f"dropout {what}", scaled=True)


def test_dropout_zero_probability_equals_plain_forward():
    rng = np.random.default_rng(2)
    q, k, v = (to_cuda(rng.normal(size=(1, 2, 20, 32)), "float32") for _ in range(3))
    a, _ = engine.forward(q, k, v, is_causal=True, dropout=(0.0, 1, 0))
    bq, _ = engine.forward(q, k, v, is_causal=True)
    np.testing.assert_allclose(to_np(a), to_np(bq), **TOL["float32"])


def test_sdpa_dropout_api_and_tape():
    """nn.scaled_dot_product_attention(dropout_p=...) draws (seed, offset) per call,
    the VJP replays the same mask, and the reference's backend rule holds."""
    rng = np.random.default_rng(8)
    raw = [rng.normal(size=(1, 2, 6, 8)).astype(np.float32) for _ in range(3)]
    up = rng.normal(size=(1, 2, 6, 8)).astype(np.float32)
    tensors = [ts.Tensor(torch.from_numpy(a).cuda(), requires_grad=True) for a in raw]
    ts.seed(8)
    out = nn.scaled_dot_product_attention(*tensors, dropout_p=0.3, is_causal=True)
    out.backward(ts.Tensor(torch.from_numpy(up).cuda()))
    keep = engine.dropout_mask(1, 2, 6, 6, (0.3, 8, 0), "cuda:0").cpu().numpy().astype(bool)
    kw = dict(is_causal=True, dropout_keep=keep, dropout_p=0.3)
    raw64 = [a.astype(np.float64) for a in raw]
    ref_o, _ = oracle.attention_forward(*raw64, algorithm="dense", **kw)
    ref_g = oracle.attention_backward_dense(*raw64, up.astype(np.float64), **kw)
    assert_close(out.numpy(), ref_o, "float32", "sdpa dropout out")
    for t, r, what in zip(tensors, ref_g, ("dq", "dk", "dv")):
        assert_close(t.grad.numpy(), r, "float32", f"sdpa dropout {what}")
    second = nn.scaled_dot_product_attention(*tensors, dropout_p=0.3, is_causal=True)
    assert not np.allclose(second.numpy(), out.numpy())  # next call, next offset
    with ts.no_grad():
        plain = nn.scaled_dot_product_attention(*tensors, dropout_p=0.3, backend="dense")
    assert plain.shape == out.shape
    for backend in ("streaming", "native"):
        with pytest.raises(ValueError, match="dense backend"):
            nn.scaled_dot_product_attention(*tensors, dropout_p=0.1, backend=backend)


TC_CASES = [
    # (dtype, B, Hq, Hkv, Tq, Tk, D, causal, offset, p): shapes the tcgen05 kernels take,
    # several key tiles, lengths that are not multiples of the tile or of a key quad
    ("bfloat16", 1, 4, 2, 200, 331, 64, True, 131, 0.2),
    ("bfloat16", 2, 2, 2, 130, 130, 128, False, 0, 0.5),
    ("float16", 1, 2, 1, 257, 257, 128, True, 0, 0.1),
    # 148 pairs x 2 units: by default the persistent one-tile forward's kDrop instantiation
    ("bfloat16", 1, 148, 74, 300, 300, 64, True, 0, 0.2),
]


@pytest.mark.parametrize("kernel", ["default", "other"])
@pytest.mark.parametrize("case", TC_CASES, ids=lambda c: f"{c[0]}-D{c[6]}-T{c[4]}x{c[5]}-p{c[9]}")
def test_tcgen05_dropout_matches_oracle(case, kernel, monkeypatch):
    """The tensor-core forward and backward (kDrop instantiations) draw the same
    mask as the materialised one and match the oracle's dense dropout VJP.
    "default" runs the one-tile forward (persistent for the 148-pair case), the
    default with dropout; "other" selects the two-tile kernel's kDrop variant."""
    name, b, hq, hkv, tq, tk, d, causal, offset, p = case
    if kernel == "other":
        monkeypatch.setenv("TS_FWD_KERNEL", "pair")
    rng = np.random.default_rng(tq + tk + d)
    q, k, v = (rng.normal(size=s) for s in ((b, hq, tq, d), (b, hkv, tk, d), (b, hkv, tk, d)))
    g = rng.normal(size=(b, hq, tq, d))
    qr, kr, vr, gr = (rounded(x, name) for x in (q, k, v, g))
    tq_, tk_, tv_, tg_ = (to_cuda(x, name) for x in (q, k, v, g))
    args = (p, 4242, 7)
    kw = dict(is_causal=causal, causal_offset=offset)
    assert engine.fwd_path(tq_, tk_, tv_, **kw) == "tcgen05"
    out, lse = engine.forward(tq_, tk_, tv_, dropout=args, **kw)
    assert engine.bwd_path(tq_, tk_, tv_, out, lse, tg_, **kw) == "tcgen05"
    dq, dk, dvv = engine.backward(tq_, tk_, tv_, out, lse, tg_, dropout=args, **kw)
    torch.cuda.synchronize()
    keep = engine.dropout_mask(b, hq, tq, tk, args, "cuda:0").cpu().numpy().astype(bool)
    okw = dict(is_causal=causal, causal_offset=offset, enable_gqa=hq != hkv, dropout_keep=keep, dropout_p=p)
    ref_o, ref_l = oracle.attention_forward(qr, kr, vr, algorithm="dense", **okw)
    assert_close(to_np(out), ref_o, name, "tc dropout out")
    assert_close(to_np(lse), ref_l, "float32", "tc dropout lse")
    rdq, rdk, rdv = oracle.attention_backward_dense(qr, kr, vr, gr, None, **okw)
    for got, ref, what in ((dq, rdq, "dq"), (dk, rdk, "dk"), (dvv, rdv, "dv")):
        assert_close(to_np(got), ref, name, f"tc dropout {what}", scaled=True)
