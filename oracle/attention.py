"""CPU oracle for tensorsmith's attention path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The B200 engine (``tensorsmith_b200``) never calls into it and has
no CPU fallback.

It restates, in NumPy, the algorithm of tensorsmith 0.3.0's attention path
(paths relative to the tensorsmith project root):

* ``scaled_dot_product_attention``  -- src/tensorsmith/nn/attention.py:16-252
    - validation and backend choice   :36-87
    - compute dtype (half -> fp32)    :63
    - GQA key/value expansion         :93-100
    - ``scores`` (scale, masks, causal offset)  :102-113
    - dense forward                   :132-145
    - streaming online-softmax forward with saved LSE  :175-198
    - dense and blockwise VJP         :200-244
    - attention dropout (dense only)  :140-144, 212-216
    - GQA gradient reduction          :245-247
* ``rotary_embedding``               -- src/tensorsmith/nn/attention.py:255-296
* ``KVCache``                        -- src/tensorsmith/nn/cache.py:12-142

Parity pin: ``tests/golden/make_golden.py`` runs the reference itself on seeded
inputs and stores its outputs under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks every function here against those fixtures.
"""

from __future__ import annotations

import math

import numpy as np

NEG_INF = -np.inf


def compute_dtype(dtype) -> np.dtype:
    """Half-precision inputs are computed in fp32 (nn/attention.py:63)."""
    dtype = np.dtype(dtype)
    if dtype == np.float16 or dtype.name == "bfloat16":
        return np.dtype(np.float32)
    return dtype


def _expand_groups(x: np.ndarray, q_heads: int) -> np.ndarray:
    """Repeat each KV head for its query-head group (nn/attention.py:93-100)."""
    kv_heads = x.shape[1]
    if kv_heads == q_heads:
        return x
    rep = q_heads // kv_heads
    return np.repeat(x, rep, axis=1)


def _allowed(qlen: int, klen: int, q0: int, k0: int, causal: bool, offset: int):
    """Causal rule ``i + offset >= j`` for absolute query i / key j (nn/attention.py:108-112)."""
    if not causal:
        return None
    qi = np.arange(q0, q0 + qlen)[:, None]
    kj = np.arange(k0, k0 + klen)[None, :]
    return qi + offset >= kj


def _scores(qb, kb, q0, k0, scale, mask, causal, offset):
    """``scores()`` of nn/attention.py:102-113: scale*Q K^T, masks, causal rule."""
    s = np.matmul(qb, np.swapaxes(kb, -1, -2)) * scale
    nq, nk = qb.shape[2], kb.shape[2]
    if mask is not None:
        part = mask[:, :, q0 : q0 + nq, k0 : k0 + nk]
        if part.dtype == np.bool_:
            s = np.where(part, s, NEG_INF)
        else:
            s = s + part
    allowed = _allowed(nq, nk, q0, k0, causal, offset)
    if allowed is not None:
        s = np.where(allowed, s, NEG_INF)
    return s


def _prepare(q, k, v, mask, scale, enable_gqa):
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("attention expects [batch, heads, sequence, channels]")
    b, hq, tq, d = q.shape
    hkv, tk = k.shape[1], k.shape[2]
    if hq != hkv and (not enable_gqa or hq % hkv):
        raise ValueError("grouped-query attention requires enable_gqa and divisible heads")
    cdt = compute_dtype(q.dtype)
    qc, kc, vc = (x.astype(cdt) for x in (q, k, v))
    kc, vc = _expand_groups(kc, hq), _expand_groups(vc, hq)
    multiplier = 1.0 / math.sqrt(d) if scale is None else scale
    full_mask = None
    if mask is not None:
        mask = np.asarray(mask)
        if mask.dtype != np.bool_:
            mask = mask.astype(cdt)
        full_mask = np.broadcast_to(mask, (b, hq, tq, tk))
    return qc, kc, vc, multiplier, full_mask, cdt


def attention_forward(
    q,
    k,
    v,
    mask=None,
    *,
    is_causal=False,
    scale=None,
    causal_offset=0,
    enable_gqa=False,
    algorithm="streaming",
    block_size=64,
    dropout_keep=None,
    dropout_p=0.0,
):
    """Forward of ``scaled_dot_product_attention`` (nn/attention.py:16-198).

    ``dropout_keep`` (bool ``[B,Hq,Tq,Tk]``) with ``dropout_p`` applies the
    reference's dense dropout (nn/attention.py:140-144): ``P * keep / (1 - p)``
    before ``P V``; the LSE is unaffected.

    Returns ``(out, lse)`` in the compute dtype: out ``[B,Hq,Tq,Dv]`` and the
    natural-log normaliser ``lse`` ``[B,Hq,Tq]`` (``-inf`` for fully masked
    rows, whose output is zero).  ``algorithm`` selects the dense
    (nn/attention.py:132-145) or the streaming online-softmax
    (nn/attention.py:175-198) formulation; both are exact.
    """
    qc, kc, vc, scale, mask, cdt = _prepare(q, k, v, mask, scale, enable_gqa)
    tq, tk = qc.shape[2], kc.shape[2]
    if algorithm == "dense":
        s = _scores(qc, kc, 0, 0, scale, mask, is_causal, causal_offset)
        m = np.max(s, axis=-1, keepdims=True)
        m = np.where(np.isfinite(m), m, 0).astype(cdt)
        e = np.exp(s - m)
        total = np.sum(e, axis=-1, keepdims=True)
        p = e / np.where(total > 0, total, 1)
        if dropout_keep is not None and dropout_p:
            p = p * (np.asarray(dropout_keep).astype(cdt) / (1 - dropout_p))
        out = np.matmul(p, vc)
        lse = np.where(total > 0, m + np.log(np.where(total > 0, total, 1)), NEG_INF)
        return out.astype(cdt), lse[..., 0].astype(cdt)
    if dropout_keep is not None and dropout_p:
        raise ValueError("attention dropout currently requires the dense backend")
    if algorithm != "streaming":
        raise ValueError("algorithm must be dense or streaming")
    outs, lses = [], []
    for q0 in range(0, tq, block_size):
        qb = qc[:, :, q0 : q0 + block_size]
        shape = qb.shape[:3] + (1,)
        m = np.full(shape, NEG_INF, dtype=cdt)
        total = np.zeros(shape, dtype=cdt)
        acc = np.zeros(qb.shape[:3] + (vc.shape[-1],), dtype=cdt)
        for k0 in range(0, tk, block_size):
            s = _scores(qb, kc[:, :, k0 : k0 + block_size], q0, k0, scale, mask, is_causal, causal_offset)
            m_next = np.maximum(m, np.max(s, axis=-1, keepdims=True))
            m_safe = np.where(np.isfinite(m_next), m_next, 0).astype(cdt)
            corr = np.exp(m - m_safe)
            p = np.exp(s - m_safe)
            acc = acc * corr + np.matmul(p, vc[:, :, k0 : k0 + block_size])
            total = total * corr + np.sum(p, axis=-1, keepdims=True)
            m = m_next
        safe_total = np.where(total > 0, total, 1)
        outs.append(acc / safe_total)
        lses.append(np.where(total > 0, m + np.log(safe_total), NEG_INF))
    out = np.concatenate(outs, axis=2).astype(cdt)
    lse = np.concatenate(lses, axis=2)[..., 0].astype(cdt)
    return out, lse


def attention_backward(
    q,
    k,
    v,
    out,
    lse,
    dout,
    mask=None,
    *,
    is_causal=False,
    scale=None,
    causal_offset=0,
    enable_gqa=False,
    block_size=64,
):
    """Blockwise VJP of nn/attention.py:220-247 (LSE-recomputed probabilities).

    ``out``/``lse`` are the compute-dtype forward results.  Returns
    ``(dq, dk, dv)`` in the compute dtype with KV-group reduction applied.
    """
    qc, kc, vc, scale, mask, cdt = _prepare(q, k, v, mask, scale, enable_gqa)
    b, hq, tq, d = qc.shape
    tk = kc.shape[2]
    g = np.asarray(dout).astype(cdt)
    out = np.asarray(out).astype(cdt)
    lse = np.asarray(lse).astype(cdt)[..., None]
    dq_blocks = []
    dk = np.zeros_like(kc)
    dv = np.zeros_like(vc)
    for q0 in range(0, tq, block_size):
        qb = qc[:, :, q0 : q0 + block_size]
        gb = g[:, :, q0 : q0 + block_size]
        lb = lse[:, :, q0 : q0 + block_size]
        lb = np.where(np.isfinite(lb), lb, 0)
        delta = np.sum(gb * out[:, :, q0 : q0 + block_size], axis=-1, keepdims=True)
        dqb = np.zeros_like(qb)
        for k0 in range(0, tk, block_size):
            kb, vb = kc[:, :, k0 : k0 + block_size], vc[:, :, k0 : k0 + block_size]
            s = _scores(qb, kb, q0, k0, scale, mask, is_causal, causal_offset)
            p = np.exp(s - lb)
            ds = p * (np.matmul(gb, np.swapaxes(vb, -1, -2)) - delta) * scale
            dqb = dqb + np.matmul(ds, kb)
            dk[:, :, k0 : k0 + kb.shape[2]] += np.matmul(np.swapaxes(ds, -1, -2), qb)
            dv[:, :, k0 : k0 + kb.shape[2]] += np.matmul(np.swapaxes(p, -1, -2), gb)
        dq_blocks.append(dqb)
    dq = np.concatenate(dq_blocks, axis=2)
    hkv = k.shape[1]
    if hkv != hq:
        rep = hq // hkv
        dk = dk.reshape(b, hkv, rep, tk, d).sum(axis=2)
        dv = dv.reshape(b, hkv, rep, tk, vc.shape[-1]).sum(axis=2)
    return dq.astype(cdt), dk.astype(cdt), dv.astype(cdt)


def attention_backward_dense(
    q, k, v, dout, mask=None, *, is_causal=False, scale=None, causal_offset=0, enable_gqa=False,
    dropout_keep=None, dropout_p=0.0,
):
    """Dense VJP of nn/attention.py:200-219 (probabilities materialised), with the
    forward's dropout mask when given (:212-216)."""
    qc, kc, vc, scale, mask, cdt = _prepare(q, k, v, mask, scale, enable_gqa)
    b, hq, tq, d = qc.shape
    tk = kc.shape[2]
    g = np.asarray(dout).astype(cdt)
    s = _scores(qc, kc, 0, 0, scale, mask, is_causal, causal_offset)
    m = np.max(s, axis=-1, keepdims=True)
    e = np.exp(s - np.where(np.isfinite(m), m, 0))
    total = np.sum(e, axis=-1, keepdims=True)
    p = e / np.where(total > 0, total, 1)
    drop = None
    if dropout_keep is not None and dropout_p:
        drop = np.asarray(dropout_keep).astype(cdt) / (1 - dropout_p)
    dv = np.matmul(np.swapaxes(p if drop is None else p * drop, -1, -2), g)
    dp = np.matmul(g, np.swapaxes(vc, -1, -2))
    if drop is not None:
        dp = dp * drop
    ds = p * (dp - np.sum(dp * p, axis=-1, keepdims=True)) * scale
    dq = np.matmul(ds, kc)
    dk = np.matmul(np.swapaxes(ds, -1, -2), qc)
    hkv = k.shape[1]
    if hkv != hq:
        rep = hq // hkv
        dk = dk.reshape(b, hkv, rep, tk, d).sum(axis=2)
        dv = dv.reshape(b, hkv, rep, tk, vc.shape[-1]).sum(axis=2)
    return dq.astype(cdt), dk.astype(cdt), dv.astype(cdt)


def key_valid_mask(lengths, klen: int) -> np.ndarray:
    """Boolean key-valid mask ``[B,1,1,K]`` (True = allowed) for ragged rows.

    tensorsmith has one cache length per batch (nn/cache.py:45); ragged
    batches are expressed with this mask form (docs/transformers.md:52-55).
    """
    lengths = np.asarray(lengths)
    return (np.arange(klen)[None, :] < lengths[:, None])[:, None, None, :]


def rope(x: np.ndarray, offset: int = 0, base: float = 10000.0, rotary_dim=None) -> np.ndarray:
    """Interleaved-pair rotary embedding of nn/attention.py:255-285."""
    dim = x.shape[-1] if rotary_dim is None else rotary_dim
    steps = x.shape[-2]
    freqs = base ** (-np.arange(0, dim, 2).astype(np.float32) / dim)
    angles = np.arange(offset, offset + steps).astype(np.float32)[:, None] * freqs[None, :]
    cos = np.repeat(np.cos(angles), 2, axis=-1).reshape(steps, dim).astype(x.dtype)
    sin = np.repeat(np.sin(angles), 2, axis=-1).reshape(steps, dim).astype(x.dtype)
    part = x[..., :dim]
    rotated = np.stack((-part[..., 1::2], part[..., 0::2]), axis=-1).reshape(part.shape)
    result = part * cos + rotated * sin
    if dim < x.shape[-1]:
        result = np.concatenate((result, x[..., dim:]), axis=-1)
    return result


def quantize_int8(x: np.ndarray):
    """Per-token/head symmetric int8 of nn/cache.py:70-75."""
    raw = x.astype(np.float32)
    scale = np.maximum(np.max(np.abs(raw), axis=-1, keepdims=True) / 127, 1e-8)
    return np.round(raw / scale).astype(np.int8), scale.astype(np.float32)


class KVCacheOracle:
    """Preallocated ``[B,H,cap,D]`` cache with the semantics of nn/cache.py:12-142.

    ``append`` validates, then writes ``[length:length+steps]`` (:54-86);
    ``get`` returns the prefix (:88-99); ``reset``/``truncate``/``reorder``
    follow :101-123.  Storage is kept in ``dtype`` (or int8 + fp32 scales).
    """

    def __init__(self, batch_size, num_heads, head_dim, max_seq_len, *, dtype=np.float32,
                 quantized=False, value_dim=None):
        if min(batch_size, num_heads, head_dim, max_seq_len) <= 0:
            raise ValueError("cache dimensions and capacity must be positive")
        self.batch_size, self.num_heads, self.head_dim = batch_size, num_heads, head_dim
        self.value_dim = head_dim if value_dim is None else value_dim
        self.max_seq_len = max_seq_len
        self.dtype = np.dtype(dtype)
        self.quantized = quantized
        self.length = 0
        store = np.int8 if quantized else self.dtype
        shape = (batch_size, num_heads, max_seq_len)
        self.keys = np.zeros(shape + (head_dim,), dtype=store)
        self.values = np.zeros(shape + (self.value_dim,), dtype=store)
        self.key_scales = np.ones(shape + (1,), np.float32) if quantized else None
        self.value_scales = np.ones(shape + (1,), np.float32) if quantized else None

    def append(self, key: np.ndarray, value: np.ndarray):
        prefix = (self.batch_size, self.num_heads)
        if key.ndim != 4 or key.shape[:2] != prefix or key.shape[-1] != self.head_dim:
            raise ValueError("key shape does not match cache configuration")
        if value.shape != key.shape[:3] + (self.value_dim,):
            raise ValueError("value shape does not match cache configuration")
        stop = self.length + key.shape[2]
        if key.shape[2] == 0 or stop > self.max_seq_len:
            raise ValueError(f"cache capacity {self.max_seq_len} exceeded or empty append")
        sl = slice(self.length, stop)
        keys, values = key.astype(self.dtype), value.astype(self.dtype)
        if self.quantized:
            keys, ks = quantize_int8(keys)
            values, vs = quantize_int8(values)
            self.key_scales[:, :, sl] = ks
            self.value_scales[:, :, sl] = vs
        self.keys[:, :, sl] = keys
        self.values[:, :, sl] = values
        self.length = stop
        return self.get()

    def get(self):
        keys = self.keys[:, :, : self.length]
        values = self.values[:, :, : self.length]
        if self.quantized:
            keys = (keys.astype(np.float32) * self.key_scales[:, :, : self.length]).astype(self.dtype)
            values = (values.astype(np.float32) * self.value_scales[:, :, : self.length]).astype(
                self.dtype
            )
        return keys, values

    def reset(self):
        self.length = 0

    def truncate(self, length: int):
        if not 0 <= length <= self.length:
            raise ValueError("truncate length must be between zero and the current length")
        self.length = length

    def reorder(self, indices):
        host = np.asarray(indices)
        if host.shape != (self.batch_size,) or host.dtype.kind not in "iu":
            raise ValueError("beam indices must be one integer per cache batch row")
        if (host < 0).any() or (host >= self.batch_size).any():
            raise ValueError("beam index out of range")
        self.keys, self.values = self.keys[host], self.values[host]
        if self.quantized:
            self.key_scales, self.value_scales = self.key_scales[host], self.value_scales[host]


def decode_attention(q, keys, values, lengths, *, causal_offset=None, scale=None, enable_gqa=False):
    """Cached decode: ``q`` ``[B,Hq,Tq,D]`` against a padded cache prefix.

    ``lengths[b]`` is the number of valid keys of row b (a key-valid mask,
    docs/transformers.md:52-55); queries sit at absolute positions
    ``lengths[b] - Tq + i`` so the causal rule of nn/attention.py:108-112 uses
    that per-row offset.  Returns ``(out, lse)`` in the compute dtype.
    """
    b, hq, tq, _ = q.shape
    lengths = np.asarray(lengths)
    outs, lses = [], []
    for row in range(b):
        n = int(lengths[row])
        off = n - tq if causal_offset is None else causal_offset
        o, l = attention_forward(
            q[row : row + 1], keys[row : row + 1, :, :n], values[row : row + 1, :, :n],
            is_causal=True, causal_offset=off, scale=scale, enable_gqa=enable_gqa,
            algorithm="dense",
        )
        outs.append(o)
        lses.append(l)
    return np.concatenate(outs, axis=0), np.concatenate(lses, axis=0)


def causal_pairs(batch: int, heads: int, qlen: int, klen: int, offset: int) -> int:
    """Number of allowed (query, key) pairs: B*H*sum_i min(K, i+1+offset)."""
    i = np.arange(qlen, dtype=np.int64)
    return int(batch * heads * np.minimum(klen, np.maximum(0, i + 1 + offset)).sum())
