"""Array-level entry points of the B200 attention engine.

These functions take CUDA device arrays (torch tensors are used as the device
allocator and stream source; any strided 4-D view is accepted), fill the C-ABI
parameter structs of include/ts_attn.h and launch on the current stream.  They
allocate outputs and workspaces on the caller's side of the ABI, exactly as the
C contract requires, and never compute anything on the host.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

_DTYPE_CODES = {
    torch.float32: _lib.F32,
    torch.float16: _lib.F16,
    torch.bfloat16: _lib.BF16,
    torch.float64: _lib.F64,
}

# Largest (query heads per KV head) x (query tokens) the split-K decode kernel takes.
DECODE_MAX_ROWS = 8


def lse_dtype(dtype: torch.dtype) -> torch.dtype:
    """LSE is fp32 (softmax statistics of half/fp32 inputs), fp64 for fp64 inputs."""
    return torch.float64 if dtype == torch.float64 else torch.float32


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise TypeError(f"the B200 attention engine does not support dtype {dtype}") from None


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("the B200 attention engine needs CUDA device tensors")


def view4(t: torch.Tensor) -> _lib.View4:
    if t.dim() != 4:
        raise ValueError("expected a [batch, heads, sequence, channels] view")
    return _lib.View4(t.data_ptr(), (ctypes.c_int64 * 4)(*t.stride()))


def _stream_handle(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def default_scale(head_dim: int) -> float:
    """1/sqrt(D), the reference default (nn/attention.py:60)."""
    return 1.0 / math.sqrt(head_dim)


def _mask_args(mask, shape, dtype):
    """Broadcast a bool / float mask to [B, H, Tq, Tk] strides (0 on broadcast axes).

    Additive masks are passed in the accumulation type (fp64 for fp64 inputs, else fp32)."""
    if mask is None:
        return _lib.MASK_NONE, None, (0, 0, 0, 0), None
    if mask.dtype == torch.bool:
        kind = _lib.MASK_BOOL
        keep = mask
    elif mask.is_floating_point():
        kind = _lib.MASK_ADD_F32
        acc = lse_dtype(dtype)
        keep = mask if mask.dtype == acc else mask.to(acc)
    else:
        raise TypeError("attention masks must be boolean or floating point")
    try:
        expanded = keep.expand(*shape)
    except RuntimeError as error:
        raise ValueError("attention mask is not broadcastable to [B,H,Q,K]") from error
    return kind, expanded.data_ptr(), tuple(expanded.stride()), keep


def make_params(q, k, v, o, lse, *, is_causal=False, scale=None, causal_offset=0, kv_lens=None,
                mask=None):
    """Fill ts_attn_params; returns (params, keepalive) -- keep the tuple alive until launch."""
    b, hq, tq, d = q.shape
    hkv, tk, dv = k.shape[1], k.shape[2], v.shape[3]
    p = _lib.AttnParams()
    p.q, p.k, p.v, p.o = view4(q), view4(k), view4(v), view4(o)
    p.lse = lse.data_ptr() if lse is not None else None
    if lse is not None:
        p.lse_stride = (ctypes.c_int64 * 3)(*lse.stride())
    p.dtype = dtype_code(q.dtype)
    p.batch, p.q_heads, p.kv_heads = b, hq, hkv
    p.q_len, p.kv_len, p.head_dim, p.value_dim = tq, tk, d, dv
    p.scale = default_scale(d) if scale is None else float(scale)
    p.is_causal = 1 if is_causal else 0
    p.causal_offset = int(causal_offset)
    lens = None
    if kv_lens is not None:
        lens = kv_lens if kv_lens.dtype == torch.int32 else kv_lens.to(torch.int32)
        p.kv_lens = lens.data_ptr()
    kind, ptr, strides, keep = _mask_args(mask, (b, hq, tq, tk), q.dtype)
    p.mask_kind = kind
    p.mask = ptr
    p.mask_stride = (ctypes.c_int64 * 4)(*strides)
    return p, (lens, keep)


def _check_inputs(q, k, v):
    _require_cuda(q, k, v)
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError("attention inputs must have the same floating-point dtype")
    dtype_code(q.dtype)


def fwd_path(q, k, v, *, decode=False, is_causal=False, scale=None, causal_offset=0, kv_lens=None,
             mask=None) -> str:
    """Name of the kernel family the engine selects for this problem."""
    o = torch.empty((q.shape[0], q.shape[1], q.shape[2], v.shape[3]), dtype=q.dtype, device=q.device)
    p, keep = make_params(q, k, v, o, None, is_causal=is_causal, scale=scale,
                          causal_offset=causal_offset, kv_lens=kv_lens, mask=mask)
    code = _lib.lib().ts_attn_fwd_path(ctypes.byref(p), 1 if decode else 0)
    if code < 0:
        _lib.check(code, "ts_attn_fwd_path")
    return _lib.PATH_NAMES[code]


def _dropout_struct(dropout) -> _lib.Dropout:
    p, seed, offset = dropout
    if not 0.0 <= float(p) < 1.0:
        raise ValueError("dropout probability must be in [0, 1)")
    return _lib.Dropout(float(p), int(seed) & (2**64 - 1), int(offset) & (2**64 - 1))


def forward(q, k, v, *, is_causal=False, scale=None, causal_offset=0, kv_lens=None, mask=None,
            need_lse=True, out=None, lse=None, dropout=None):
    """Attention forward: returns ``(out [B,Hq,Tq,Dv], lse [B,Hq,Tq] or None)``.

    ``lse`` is fp32 (fp64 for fp64 inputs), natural-log units, -inf on fully masked rows.
    ``dropout = (p, seed, offset)`` applies attention dropout (ts_attn_fwd_dropout); pass
    the same tuple to ``backward``."""
    _check_inputs(q, k, v)
    b, hq, tq, _ = q.shape
    if out is None:
        out = torch.empty((b, hq, tq, v.shape[3]), dtype=q.dtype, device=q.device)
    if need_lse and lse is None:
        lse = torch.empty((b, hq, tq), dtype=lse_dtype(q.dtype), device=q.device)
    p, keep = make_params(q, k, v, out, lse if need_lse else None, is_causal=is_causal, scale=scale,
                          causal_offset=causal_offset, kv_lens=kv_lens, mask=mask)
    if dropout is not None:
        d = _dropout_struct(dropout)
        _lib.check(_lib.lib().ts_attn_fwd_dropout(ctypes.byref(p), ctypes.byref(d), _stream_handle(q.device)),
                   "ts_attn_fwd_dropout")
    else:
        _lib.check(_lib.lib().ts_attn_fwd(ctypes.byref(p), _stream_handle(q.device)), "ts_attn_fwd")
    del keep
    return out, (lse if need_lse else None)


def decode_workspace_bytes(q, k, v, **kw) -> int:
    o = torch.empty((q.shape[0], q.shape[1], q.shape[2], v.shape[3]), dtype=q.dtype, device=q.device)
    p, keep = make_params(q, k, v, o, None, **kw)
    return int(_lib.lib().ts_attn_decode_workspace_size(ctypes.byref(p)))


def decode(q, k, v, *, is_causal=True, scale=None, causal_offset=0, kv_lens=None, mask=None,
           need_lse=False, out=None, lse=None, workspace=None):
    """Split-K decode for a few query tokens against a long KV cache."""
    _check_inputs(q, k, v)
    b, hq, tq, _ = q.shape
    if out is None:
        out = torch.empty((b, hq, tq, v.shape[3]), dtype=q.dtype, device=q.device)
    if need_lse and lse is None:
        lse = torch.empty((b, hq, tq), dtype=lse_dtype(q.dtype), device=q.device)
    p, keep = make_params(q, k, v, out, lse if need_lse else None, is_causal=is_causal, scale=scale,
                          causal_offset=causal_offset, kv_lens=kv_lens, mask=mask)
    handle = _lib.lib()
    need = int(handle.ts_attn_decode_workspace_size(ctypes.byref(p)))
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_ptr = workspace.data_ptr() if (need and workspace is not None) else None
    ws_bytes = workspace.numel() * workspace.element_size() if (need and workspace is not None) else 0
    _lib.check(handle.ts_attn_decode(ctypes.byref(p), ws_ptr, ws_bytes, _stream_handle(q.device)),
               "ts_attn_decode")
    del keep
    return out, (lse if need_lse else None)


def decode_noalloc(q, k, v, *, is_causal=True, scale=None, causal_offset=0, kv_lens=None,
                   need_lse=False, out=None, lse=None):
    """Decode through ts_attn_decode_noalloc: no workspace, no device allocation by the engine.

    For callers that cannot allocate device memory at decode time (all HBM
    already handed to KV-cache pages, or no cudaMalloc allowed between decode
    steps).  The split partials go to the library's fixed 8 MiB per-device
    scratch; calls that overlap on one device race on it.  Pass ``out`` (and
    ``lse`` when ``need_lse``) preallocated to keep the call allocation-free."""
    _check_inputs(q, k, v)
    b, hq, tq, _ = q.shape
    if out is None:
        out = torch.empty((b, hq, tq, v.shape[3]), dtype=q.dtype, device=q.device)
    if need_lse and lse is None:
        lse = torch.empty((b, hq, tq), dtype=lse_dtype(q.dtype), device=q.device)
    p, keep = make_params(q, k, v, out, lse if need_lse else None, is_causal=is_causal, scale=scale,
                          causal_offset=causal_offset, kv_lens=kv_lens)
    status = _lib.lib().ts_attn_decode_noalloc(ctypes.byref(p), _stream_handle(q.device))
    if status == _lib.ERR_WORKSPACE:
        raise _lib.EngineError(status, "ts_attn_decode_noalloc: problem needs more than the fixed "
                               f"{_lib.NOALLOC_SCRATCH_BYTES >> 20} MiB decode scratch")
    _lib.check(status, "ts_attn_decode_noalloc")
    del keep
    return out, (lse if need_lse else None)


def _bwd_params(q, k, v, out, lse, dout, dq, dk, dv, **kw):
    fp, keep = make_params(q, k, v, out, lse, **kw)
    bp = _lib.AttnBwdParams()
    bp.fwd = fp
    bp.dout, bp.dq, bp.dk, bp.dv = view4(dout), view4(dq), view4(dk), view4(dv)
    return bp, keep


def bwd_path(q, k, v, out, lse, dout, **kw) -> str:
    """Name of the kernel family ts_attn_bwd selects for this problem."""
    bp, keep = _bwd_params(q, k, v, out, lse, dout, torch.empty_like(q), torch.empty_like(k),
                           torch.empty_like(v), **kw)
    code = _lib.lib().ts_attn_bwd_path(ctypes.byref(bp))
    if code < 0:
        _lib.check(code, "ts_attn_bwd_path")
    return _lib.PATH_NAMES[code]


def backward(q, k, v, out, lse, dout, *, is_causal=False, scale=None, causal_offset=0, kv_lens=None,
             mask=None, dq=None, dk=None, dv=None, dropout=None):
    """dQ, dK, dV of attention from the forward output and its LSE (``dropout`` as given
    to the forward)."""
    _check_inputs(q, k, v)
    _require_cuda(out, lse, dout)
    dq = torch.empty_like(q) if dq is None else dq
    dk = torch.empty_like(k) if dk is None else dk
    dv = torch.empty_like(v) if dv is None else dv
    if dout.dtype != q.dtype:
        dout = dout.to(q.dtype)
    bp, keep = _bwd_params(q, k, v, out, lse, dout, dq, dk, dv, is_causal=is_causal, scale=scale,
                           causal_offset=causal_offset, kv_lens=kv_lens, mask=mask)
    handle = _lib.lib()
    if dropout is not None:
        d = _dropout_struct(dropout)
        need = int(handle.ts_attn_bwd_dropout_workspace_size(ctypes.byref(bp)))
        ws = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
        _lib.check(handle.ts_attn_bwd_dropout(ctypes.byref(bp), ctypes.byref(d), ws.data_ptr(), ws.numel(),
                                              _stream_handle(q.device)), "ts_attn_bwd_dropout")
        del keep
        return dq, dk, dv
    need = int(handle.ts_attn_bwd_workspace_size(ctypes.byref(bp)))
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    _lib.check(handle.ts_attn_bwd(ctypes.byref(bp), ws.data_ptr(), ws.numel(), _stream_handle(q.device)),
               "ts_attn_bwd")
    del keep
    return dq, dk, dv


def dropout_mask(batch, heads, q_len, kv_len, dropout, device) -> torch.Tensor:
    """The uint8 keep mask [B, Hq, Tq, Tk] that ``dropout = (p, seed, offset)`` applies."""
    d = _dropout_struct(dropout)
    mask = torch.empty((batch, heads, q_len, kv_len), dtype=torch.uint8, device=device)
    _lib.check(_lib.lib().ts_attn_dropout_mask(ctypes.byref(d), batch, heads, q_len, kv_len, mask.data_ptr(),
                                               _stream_handle(mask.device)), "ts_attn_dropout_mask")
    return mask


class _DropoutGenerator:
    """(seed, offset) source for attention dropout: ``seed()`` resets it, every draw
    takes the next offset (the counter that keeps calls' masks independent)."""

    def __init__(self):
        self.seed_value = int(torch.initial_seed()) & (2**64 - 1)
        self.offset = 0

    def seed(self, value: int) -> None:
        self.seed_value = int(value) & (2**64 - 1)
        self.offset = 0

    def draw(self, p: float) -> tuple:
        args = (float(p), self.seed_value, self.offset)
        self.offset += 1
        return args


DROPOUT_GENERATOR = _DropoutGenerator()


def seed(value: int) -> None:
    """Seed the attention-dropout generator (tensorsmith's ``ts.seed``, device.py:226-232)."""
    DROPOUT_GENERATOR.seed(value)


def kv_append(key, value, key_cache, value_cache, *, position=0, positions=None, positions_out=None):
    """Write a [B,H,steps,C] chunk into [B,H,cap,C] caches at ``position`` (or per-row ``positions``)."""
    _require_cuda(key, value, key_cache, value_cache)
    p = _lib.KvAppendParams()
    p.key, p.value = view4(key), view4(value)
    p.key_cache, p.value_cache = view4(key_cache), view4(value_cache)
    p.src_dtype = dtype_code(key.dtype)
    p.cache_dtype = dtype_code(key_cache.dtype)
    if value.dtype != key.dtype or value_cache.dtype != key_cache.dtype:
        raise TypeError("key/value and their caches must share a dtype each")
    p.batch, p.heads, p.steps = key.shape[0], key.shape[1], key.shape[2]
    p.head_dim, p.value_dim, p.capacity = key.shape[3], value.shape[3], key_cache.shape[2]
    p.position = int(position)
    p.positions = positions.data_ptr() if positions is not None else None
    p.positions_out = positions_out.data_ptr() if positions_out is not None else None
    _lib.check(_lib.lib().ts_kv_append(ctypes.byref(p), _stream_handle(key.device)), "ts_kv_append")


def _storage_code(dtype: torch.dtype) -> int:
    return _lib.I8 if dtype == torch.int8 else dtype_code(dtype)


def kv_reorder(src, dst, index, length):
    """dst[b, :, :length] = src[index[b], :, :length] (beam reorder; int8 storage too)."""
    _require_cuda(src, dst, index)
    idx = index if index.dtype == torch.int32 else index.to(torch.int32)
    _lib.check(
        _lib.lib().ts_kv_reorder(view4(src), view4(dst), _storage_code(src.dtype), src.shape[0],
                                 src.shape[1], int(length), src.shape[3], idx.data_ptr(),
                                 _stream_handle(src.device)),
        "ts_kv_reorder",
    )


def _check_int8_cache(cache, scales):
    if cache.dtype != torch.int8 or cache.dim() != 4:
        raise TypeError("int8 cache storage must be an int8 [B, H, capacity, C] tensor")
    if scales.dtype != torch.float32 or not scales.is_contiguous() or scales.numel() != cache.shape[0] * cache.shape[1] * cache.shape[2]:
        raise ValueError("int8 cache scales must be contiguous fp32 [B, H, capacity(, 1)]")


def kv_append_int8(key, value, key_cache, value_cache, key_scales, value_scales, *, compute_dtype,
                   position=0, positions=None, positions_out=None):
    """Quantising append (nn/cache.py:70-82): rows rounded to ``compute_dtype``, then
    symmetric int8 with one fp32 scale per (row, head, token) written to the scale arrays."""
    _require_cuda(key, value, key_cache, value_cache, key_scales, value_scales)
    _check_int8_cache(key_cache, key_scales)
    _check_int8_cache(value_cache, value_scales)
    if value.dtype != key.dtype:
        raise TypeError("key/value must share a dtype")
    p = _lib.KvAppendParams()
    p.key, p.value = view4(key), view4(value)
    p.key_cache, p.value_cache = view4(key_cache), view4(value_cache)
    p.src_dtype = dtype_code(key.dtype)
    p.cache_dtype = dtype_code(compute_dtype)
    p.batch, p.heads, p.steps = key.shape[0], key.shape[1], key.shape[2]
    p.head_dim, p.value_dim, p.capacity = key.shape[3], value.shape[3], key_cache.shape[2]
    p.position = int(position)
    p.positions = positions.data_ptr() if positions is not None else None
    p.positions_out = positions_out.data_ptr() if positions_out is not None else None
    _lib.check(_lib.lib().ts_kv_append_int8(ctypes.byref(p), key_scales.data_ptr(), value_scales.data_ptr(),
                                            _stream_handle(key.device)), "ts_kv_append_int8")


def kv_dequant_int8(src, scales, out, length):
    """out[:, :, :length] = dtype(float(src) * scale) for an int8 cache (nn/cache.py:91-99)."""
    _require_cuda(src, scales, out)
    _check_int8_cache(src, scales)
    _lib.check(
        _lib.lib().ts_kv_dequant_int8(view4(src), scales.data_ptr(), src.shape[2], view4(out),
                                      dtype_code(out.dtype), src.shape[0], src.shape[1], int(length),
                                      src.shape[3], _stream_handle(src.device)),
        "ts_kv_dequant_int8",
    )


def _int8_params(q, k8, v8, out, lse, kw):
    _require_cuda(q, k8, v8)
    if k8.dtype != torch.int8 or v8.dtype != torch.int8:
        raise TypeError("int8 decode expects int8 key/value storage")
    dtype_code(q.dtype)
    return make_params(q, k8, v8, out, lse, **kw)


def decode_int8_workspace_bytes(q, k8, v8, **kw) -> int:
    o = torch.empty((q.shape[0], q.shape[1], q.shape[2], v8.shape[3]), dtype=q.dtype, device=q.device)
    p, keep = _int8_params(q, k8, v8, o, None, kw)
    return int(_lib.lib().ts_attn_decode_int8_workspace_size(ctypes.byref(p)))


def decode_int8(q, k8, v8, key_scales, value_scales, *, is_causal=True, scale=None, causal_offset=0,
                kv_lens=None, need_lse=False, out=None, lse=None, workspace=None):
    """Split-K decode reading an int8 cache directly (dequantisation fused into the scores
    and the P.V sum).  ``k8``/``v8`` are the first ``kv_len`` positions of the int8 storage;
    ``key_scales``/``value_scales`` the full contiguous [B, H, capacity] scale arrays."""
    _require_cuda(key_scales, value_scales)
    b, hq, tq, _ = q.shape
    if out is None:
        out = torch.empty((b, hq, tq, v8.shape[3]), dtype=q.dtype, device=q.device)
    if need_lse and lse is None:
        lse = torch.empty((b, hq, tq), dtype=lse_dtype(q.dtype), device=q.device)
    kw = dict(is_causal=is_causal, scale=scale, causal_offset=causal_offset, kv_lens=kv_lens)
    p, keep = _int8_params(q, k8, v8, out, lse if need_lse else None, kw)
    cap = key_scales.numel() // (k8.shape[0] * k8.shape[1])
    if (key_scales.dtype != torch.float32 or value_scales.dtype != torch.float32 or not key_scales.is_contiguous()
            or not value_scales.is_contiguous() or value_scales.numel() != key_scales.numel()):
        raise ValueError("int8 cache scales must be contiguous fp32 [B, H, capacity(, 1)]")
    handle = _lib.lib()
    need = int(handle.ts_attn_decode_int8_workspace_size(ctypes.byref(p)))
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_ptr = workspace.data_ptr() if (need and workspace is not None) else None
    ws_bytes = workspace.numel() * workspace.element_size() if (need and workspace is not None) else 0
    _lib.check(handle.ts_attn_decode_int8(ctypes.byref(p), key_scales.data_ptr(), value_scales.data_ptr(), cap,
                                          ws_ptr, ws_bytes, _stream_handle(q.device)), "ts_attn_decode_int8")
    del keep
    return out, (lse if need_lse else None)


_INV_FREQ: dict = {}


def rope_inv_freq(rotary_dim: int, base: float, device) -> torch.Tensor:
    """inv_freq[i] = base^(-2i/rotary_dim) in fp32, evaluated as the reference
    does it (float32 exponent array, nn/attention.py:274), cached per device."""
    import numpy as np

    key = (int(rotary_dim), float(base), str(device))
    if key not in _INV_FREQ:
        host = base ** (-np.arange(0, rotary_dim, 2).astype(np.float32) / rotary_dim)
        _INV_FREQ[key] = torch.from_numpy(np.ascontiguousarray(host.astype(np.float32))).to(device)
    return _INV_FREQ[key]


def rope(x, *, offset=0, base=10000.0, rotary_dim=None, positions=None, inverse=False, out=None):
    """Interleaved-pair rotary embedding of a [B, H, T, C] view at positions offset + t
    (or positions[b] + t); ``inverse`` applies the inverse rotation (the VJP)."""
    _require_cuda(x)
    dim = x.shape[3] if rotary_dim is None else int(rotary_dim)
    out = torch.empty_like(x) if out is None else out
    inv = rope_inv_freq(dim, base, x.device)
    pos = None
    if positions is not None:
        pos = positions if positions.dtype == torch.int32 else positions.to(torch.int32)
    _lib.check(
        _lib.lib().ts_rope(view4(x), view4(out), dtype_code(x.dtype), x.shape[0], x.shape[1], x.shape[2],
                           x.shape[3], dim, int(offset), pos.data_ptr() if pos is not None else None,
                           inv.data_ptr(), 1 if inverse else 0, _stream_handle(x.device)),
        "ts_rope",
    )
    return out


def kv_append_rope(key, value, key_cache, value_cache, *, position=0, positions=None, positions_out=None,
                   base=10000.0, rotary_dim=None):
    """kv_append with the keys rotated at their cache positions in the same pass."""
    _require_cuda(key, value, key_cache, value_cache)
    dim = key.shape[3] if rotary_dim is None else int(rotary_dim)
    p = _lib.KvAppendParams()
    p.key, p.value = view4(key), view4(value)
    p.key_cache, p.value_cache = view4(key_cache), view4(value_cache)
    p.src_dtype = dtype_code(key.dtype)
    p.cache_dtype = dtype_code(key_cache.dtype)
    if value.dtype != key.dtype or value_cache.dtype != key_cache.dtype:
        raise TypeError("key/value and their caches must share a dtype each")
    p.batch, p.heads, p.steps = key.shape[0], key.shape[1], key.shape[2]
    p.head_dim, p.value_dim, p.capacity = key.shape[3], value.shape[3], key_cache.shape[2]
    p.position = int(position)
    p.positions = positions.data_ptr() if positions is not None else None
    p.positions_out = positions_out.data_ptr() if positions_out is not None else None
    inv = rope_inv_freq(dim, base, key.device)
    _lib.check(_lib.lib().ts_kv_append_rope(ctypes.byref(p), inv.data_ptr(), dim, _stream_handle(key.device)),
               "ts_kv_append_rope")


def device_status(device=None) -> tuple[int, int]:
    """(status, site) of the device fault word; clears it.  Synchronises the stream."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    info = ctypes.c_uint32(0)
    with torch.cuda.device(device):
        status = _lib.lib().ts_attn_device_status(_stream_handle(device), ctypes.byref(info))
    return status, info.value


def check_device_status(device=None) -> None:
    status, site = device_status(device)
    if status != _lib.OK:
        raise _lib.EngineError(status, f"device fault site 0x{site:x}")
