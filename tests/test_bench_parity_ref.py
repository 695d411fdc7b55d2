"""The fp64 reference that bench.py uses for its parity object agrees with the oracle."""

import numpy as np
import torch

import bench
import oracle


def test_ref_rows_matches_oracle():
    rng = np.random.default_rng(3)
    q = rng.standard_normal((1, 1, 40, 16))
    k = rng.standard_normal((1, 1, 50, 16))
    v = rng.standard_normal((1, 1, 50, 8))
    ref_o, ref_l = oracle.attention_forward(q, k, v, is_causal=True, causal_offset=10, algorithm="dense")
    rows = np.array([0, 7, 39])
    o, l = bench.ref_rows(torch.from_numpy(q[0, 0][rows]), torch.from_numpy(k[0, 0]), torch.from_numpy(v[0, 0]),
                          rows + 11, 0.25)
    ref_o, ref_l = oracle.attention_forward(q, k, v, is_causal=True, causal_offset=10, scale=0.25, algorithm="dense")
    np.testing.assert_allclose(o.numpy(), ref_o[0, 0][rows], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(l.numpy(), ref_l[0, 0][rows], rtol=1e-12, atol=1e-12)


def test_ref_slice_backward_matches_oracle():
    rng = np.random.default_rng(4)
    q, k, v, g = (rng.standard_normal((1, 1, 33, 16)) for _ in range(4))
    o, l, dq, dk, dv = bench.ref_slice_backward(*(torch.from_numpy(x[0, 0]) for x in (q, k, v, g)), 0.25)
    ref_o, ref_l = oracle.attention_forward(q, k, v, is_causal=True, scale=0.25, algorithm="dense")
    rdq, rdk, rdv = oracle.attention_backward(q, k, v, ref_o, ref_l, g, is_causal=True, scale=0.25)
    for got, ref in ((o, ref_o), (l, ref_l), (dq, rdq), (dk, rdk), (dv, rdv)):
        np.testing.assert_allclose(got.numpy(), ref[0, 0], rtol=1e-10, atol=1e-12)


def test_ref_slice_backward_with_dropout_matches_oracle():
    rng = np.random.default_rng(5)
    q, k, v, g = (rng.standard_normal((1, 1, 29, 16)) for _ in range(4))
    keep = rng.random((1, 1, 29, 29)) >= 0.3
    o, l, dq, dk, dv = bench.ref_slice_backward(*(torch.from_numpy(x[0, 0]) for x in (q, k, v, g)), 0.25,
                                                torch.from_numpy(keep[0, 0]), 0.3)
    kw = dict(is_causal=True, scale=0.25, dropout_keep=keep, dropout_p=0.3)
    ref_o, ref_l = oracle.attention_forward(q, k, v, algorithm="dense", **kw)
    rdq, rdk, rdv = oracle.attention_backward_dense(q, k, v, g, None, **kw)
    for got, ref in ((o, ref_o), (l, ref_l), (dq, rdq), (dk, rdk), (dv, rdv)):
        np.testing.assert_allclose(got.numpy(), ref[0, 0], rtol=1e-10, atol=1e-12)
