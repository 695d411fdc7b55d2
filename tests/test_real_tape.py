"""The engine's attention node on tensorsmith's own tape (CPU, no GPU).

``tensorsmith_b200.interop.attention_node`` builds the node with the Tensor
class of its inputs.  Here those are tensorsmith's real Tensors (NumPy arrays
on the cpu device), so the reference's ``Tensor._from_op`` records the node
and its ``_run_backward`` sweeps it: contributions summed over branches and
cast to each tensor's dtype (src/tensorsmith/tensor.py:662-724).  The
attention arithmetic is injected (the oracle on the host, standing in for the
CUDA kernels, which need a GPU); what is checked is the hook-up: DLPack
hand-over of raw arrays, the node's parents and op name, gradient dtypes,
branch sums and the no-grad path.

tensorsmith is imported from ``TENSORSMITH_SRC`` or from a ``reference/src``
checkout beside this repository; the test is skipped when neither exists (the
GPU boxes have no copy of the reference).

The second half checks the same contract on the torch-backed tape mirror
(``tensorsmith_b200.tensor``), whose sweep is the engine's own.
"""

import importlib
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from tensorsmith_b200 import interop
from tensorsmith_b200.tensor import Tensor as MirrorTensor

ROOT = Path(__file__).resolve().parent.parent


def _tensorsmith():
    candidates = [os.environ.get("TENSORSMITH_SRC"), str(ROOT.parent / "reference" / "src")]
    for path in candidates:
        if path and (Path(path) / "tensorsmith" / "__init__.py").exists():
            if path not in sys.path:
                sys.path.insert(0, path)
            try:
                return importlib.import_module("tensorsmith")
            except ImportError:
                return None
    return None


class OracleCompute:
    """The engine's compute interface (forward / decode / backward on torch tensors), evaluated by the
    oracle in fp64 on the host."""

    calls: list = []

    @staticmethod
    def _kw(q, k, kw):
        return dict(is_causal=kw.get("is_causal", False), scale=kw.get("scale"),
                    causal_offset=kw.get("causal_offset", 0), enable_gqa=q.shape[1] != k.shape[1])

    @classmethod
    def forward(cls, q, k, v, *, need_lse=True, **kw):
        cls.calls.append("forward")
        o, l = oracle.attention_forward(*(x.numpy().astype(np.float64) for x in (q, k, v)), algorithm="dense",
                                        **cls._kw(q, k, kw))
        return torch.from_numpy(o).to(q.dtype), (torch.from_numpy(l) if need_lse else None)

    @classmethod
    def decode(cls, q, k, v, **kw):
        cls.calls.append("decode")
        return cls.forward(q, k, v, need_lse=False, **kw)

    @classmethod
    def backward(cls, q, k, v, out, lse, dout, **kw):
        cls.calls.append("backward")
        arrays = (x.numpy().astype(np.float64) for x in (q, k, v, out, lse, dout))
        grads = oracle.attention_backward(*arrays, **cls._kw(q, k, kw))
        return tuple(torch.from_numpy(g).to(t.dtype) for g, t in zip(grads, (q, k, v)))


def _arrays(seed, shapes, dtype):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal(s).astype(dtype) for s in shapes]


def test_node_on_tensorsmith_tape_sums_branches_and_keeps_dtypes():
    ts = _tensorsmith()
    if ts is None:
        pytest.skip("tensorsmith is not importable here")
    q_np, k_np, v_np, k2_np, v2_np = _arrays(1, [(1, 4, 5, 8), (1, 2, 7, 8), (1, 2, 7, 8), (1, 2, 3, 8),
                                                 (1, 2, 3, 8)], np.float32)
    g1, g2 = _arrays(2, [(1, 4, 5, 8), (1, 4, 5, 8)], np.float32)
    q = ts.tensor(q_np, requires_grad=True)
    k = ts.tensor(k_np, requires_grad=True)
    v = ts.tensor(v_np, requires_grad=True)
    k2, v2 = ts.tensor(k2_np), ts.tensor(v2_np)  # constants: the node returns None-consuming parents
    OracleCompute.calls = []
    out1 = interop.attention_node(q, k, v, is_causal=True, causal_offset=2, compute=OracleCompute)
    out2 = interop.attention_node(q, k2, v2, compute=OracleCompute)
    assert type(out1) is type(q) and out1._op == "sdpa_native" and out1._parents == (q, k, v)
    assert isinstance(out1._data, np.ndarray) and out1.dtype == q.dtype
    # q reaches the loss along two branches; the tape must sum them.
    loss = (out1 * ts.tensor(g1)).sum() + (out2 * ts.tensor(g2)).sum()
    loss.backward()
    assert OracleCompute.calls.count("backward") == 2
    kw1 = dict(is_causal=True, causal_offset=2, enable_gqa=True)
    o1, l1 = oracle.attention_forward(q_np, k_np, v_np, algorithm="dense", **kw1)
    dq1, dk1, dv1 = oracle.attention_backward(q_np, k_np, v_np, o1, l1, g1, **kw1)
    o2, l2 = oracle.attention_forward(q_np, k2_np, v2_np, algorithm="dense", enable_gqa=True)
    dq2, _, _ = oracle.attention_backward(q_np, k2_np, v2_np, o2, l2, g2, enable_gqa=True)
    np.testing.assert_allclose(out1.numpy(), o1, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(q.grad.numpy(), dq1 + dq2, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(k.grad.numpy(), dk1, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(v.grad.numpy(), dv1, rtol=1e-5, atol=1e-5)
    for t in (q, k, v):
        assert t.grad.dtype == t.dtype
    assert k2.grad is None


def test_node_on_tensorsmith_tape_half_inputs_and_no_grad():
    ts = _tensorsmith()
    if ts is None:
        pytest.skip("tensorsmith is not importable here")
    q_np, k_np, v_np = _arrays(3, [(2, 2, 4, 8)] * 3, np.float16)
    (g,) = _arrays(4, [(2, 2, 4, 8)], np.float32)
    q, k, v = (ts.tensor(a, requires_grad=True) for a in (q_np, k_np, v_np))
    out = interop.attention_node(q, k, v, is_causal=True, compute=OracleCompute)
    assert out.dtype == q.dtype
    # A float32 upstream reaches the float16 node: the tape casts it (tensor.py:689-690).
    (out.astype("float32") * ts.tensor(g)).sum().backward()
    for t in (q, k, v):
        assert t.grad is not None and t.grad.dtype == t.dtype
    q64, k64, v64 = (a.astype(np.float64) for a in (q_np, k_np, v_np))
    o, l = oracle.attention_forward(q64, k64, v64, is_causal=True, algorithm="dense")
    g16 = g.astype(np.float16).astype(np.float64)
    dq, dk, dv = oracle.attention_backward(q64, k64, v64, o, l, g16, is_causal=True)
    for got, ref in ((q.grad, dq), (k.grad, dk), (v.grad, dv)):
        np.testing.assert_allclose(got.numpy().astype(np.float64), ref, rtol=2e-2, atol=2e-2)
    with ts.no_grad():
        plain = interop.attention_node(q, k, v, is_causal=True, recording=False, compute=OracleCompute,
                                       decode_rows=8)
    assert not plain.requires_grad and plain._parents == () and type(plain) is type(q)


def test_mirror_tape_contract():
    # The mirror's own sweep: branch sums, dtype casts, one VJP call per node, graph release.
    calls = []
    x = MirrorTensor(torch.arange(6, dtype=torch.float32).reshape(2, 3), requires_grad=True)
    h = MirrorTensor(torch.ones(2, 3, dtype=torch.float16), requires_grad=True)

    def node(parents, fn, op):
        def backward(g):
            calls.append(op)
            return fn(g)
        return MirrorTensor._from_op(parents[0]._data.clone(), parents, backward, op)

    a = node((x,), lambda g: (g * 2,), "a")
    b = node((x,), lambda g: (g * 3,), "b")
    c = node((a, b, h), lambda g: (g, g, g.double()), "c")  # a float64 contribution for the half leaf
    c.backward(torch.ones(2, 3))
    assert sorted(calls) == ["a", "b", "c"]
    torch.testing.assert_close(x._grad, torch.full((2, 3), 5.0))
    assert h._grad.dtype == torch.float16 and torch.equal(h._grad, torch.ones(2, 3, dtype=torch.float16))
    assert c._graph_freed and c._parents == ()
    with pytest.raises(RuntimeError):
        c.backward(torch.ones(2, 3))
    # retain_graph keeps it for a second pass, whose gradients accumulate
    d = node((x,), lambda g: (g,), "d")
    d.backward(torch.ones(2, 3), retain_graph=True)
    d.backward(torch.ones(2, 3))
    torch.testing.assert_close(x._grad, torch.full((2, 3), 7.0))
