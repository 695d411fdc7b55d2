"""Record the engine's attention as one node on a tensorsmith-style tape.

tensorsmith records reverse-mode nodes with ``Tensor._from_op(data, parents,
backward, op)`` (src/tensorsmith/tensor.py:121-135).  A node's ``backward``
receives the upstream gradient as a raw array and returns one raw array (or
None) per parent (:709-717); the tape casts each contribution to the parent's
dtype and sums contributions that reach a tensor along several branches
(:689-690, :714-717).  ``attention_node`` builds that node for any Tensor class
with this interface: tensorsmith's own (raw arrays are CuPy arrays on cuda,
NumPy arrays on cpu) or the torch-backed mirror in ``tensorsmith_b200.tensor``.

Raw arrays reach the engine through DLPack (``torch.from_dlpack``), without a
copy, and results go back into the caller's array type through its
namespace's ``from_dlpack`` (``cupy.from_dlpack``, ``numpy.from_dlpack``).
``compute`` supplies the attention arithmetic; the default is the engine
(``tensorsmith_b200.engine``: its C ABI and CUDA kernels).
"""

from __future__ import annotations

import torch

from . import engine


def to_torch(raw) -> torch.Tensor:
    """A torch view of a raw array (zero-copy DLPack import; torch tensors pass through)."""
    if raw is None or isinstance(raw, torch.Tensor):
        return raw
    return torch.from_dlpack(raw)


def from_torch(t: torch.Tensor, like):
    """``t`` as an array of the same kind as ``like`` (zero-copy DLPack export)."""
    if t is None or isinstance(like, torch.Tensor):
        return t
    namespace = like.__array_namespace__() if hasattr(like, "__array_namespace__") else None
    if namespace is None or not hasattr(namespace, "from_dlpack"):
        raise TypeError(f"cannot hand engine results back as {type(like).__name__} (no DLPack import)")
    return namespace.from_dlpack(t)


def attention_node(query, key, value, *, mask=None, is_causal=False, scale=None, causal_offset=0,
                   kv_lens=None, dropout=None, op="sdpa_native", recording=True, compute=engine,
                   decode_rows=None):
    """Attention output of ``query``/``key``/``value`` (Tensors of one tape implementation) as a
    Tensor of the same class: one ``_from_op`` node whose backward returns ``(dq, dk, dv)`` in the
    parents' array type and dtypes, or a plain Tensor when nothing is recorded.

    ``dropout = (p, seed, offset)`` (the forward's draw, replayed by the backward).
    ``decode_rows`` (query rows per KV head) lets a short, unmasked, unrecorded call take the
    split-K decode path."""
    cls = type(query)
    raw_q = query._data
    q, k, v = to_torch(raw_q), to_torch(key._data), to_torch(value._data)
    m = to_torch(mask)
    kwargs = dict(is_causal=is_causal, scale=scale, causal_offset=causal_offset, kv_lens=to_torch(kv_lens), mask=m)
    if dropout is not None:
        kwargs["dropout"] = dropout
    if not recording:
        if dropout is None and m is None and decode_rows is not None and decode_rows <= engine.DECODE_MAX_ROWS:
            out, _ = compute.decode(q, k, v, **kwargs)
        else:
            out, _ = compute.forward(q, k, v, need_lse=False, **kwargs)
        return cls(from_torch(out, raw_q), device=query.device)
    out, lse = compute.forward(q, k, v, need_lse=True, **kwargs)

    def backward(upstream):
        dq, dk, dv = compute.backward(q, k, v, out, lse, to_torch(upstream), **kwargs)
        return from_torch(dq, raw_q), from_torch(dk, key._data), from_torch(dv, value._data)

    return cls._from_op(from_torch(out, raw_q), (query, key, value), backward, op)
