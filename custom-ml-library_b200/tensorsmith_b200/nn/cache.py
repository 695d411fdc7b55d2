"""``KVCache`` with tensorsmith's API, stored in HBM and written by the engine.

Constructor arguments, ``append``/``get``/``reset``/``truncate``/``reorder``/
``storage``/``memory_bytes``/``length`` and their validation follow
src/tensorsmith/nn/cache.py:12-142.  Storage is ``[B, H, capacity, D]`` per
tensor (the reference layout), zero-initialised, so a decode kernel may read a
whole 128-key tile past a row's valid length without meeting non-finite
values.

``quantized=True`` stores symmetric int8 rows with one fp32 scale per token
and head (nn/cache.py:47-52, 70-82); ``get`` returns dequantised copies as the
reference does, and ``attend`` decodes straight from the int8 rows.

Engine extension for ragged batches (the reference expresses them with a
key-valid mask over a padded cache, docs/transformers.md:52-55): after
``set_lengths(lengths)`` every row has its own valid length; ``append``
then writes each row at its own position and ``seq_lens`` is the device
int32 vector to pass as ``kv_lens`` to ``scaled_dot_product_attention``.
"""

from __future__ import annotations

import numpy as np
import torch

from .. import engine
from ..tensor import Tensor, as_device, is_grad_enabled

_DTYPES = {
    "float32": torch.float32,
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
    "float64": torch.float64,
}


def _torch_dtype(dtype) -> torch.dtype:
    if isinstance(dtype, torch.dtype):
        return dtype
    name = str(dtype).replace("torch.", "")
    if name in _DTYPES:
        return _DTYPES[name]
    try:
        return _DTYPES[np.dtype(dtype).name]
    except (TypeError, KeyError):
        raise TypeError("cache compute dtype must be floating point") from None


class KVCache:
    """Preallocated [B,H,capacity,D] keys/values for autoregressive inference."""

    def __init__(self, batch_size: int, num_heads: int, head_dim: int, max_seq_len: int, *,
                 device="cuda", dtype="float32", quantized: bool = False, value_dim=None):
        if min(batch_size, num_heads, head_dim, max_seq_len) <= 0:
            raise ValueError("cache dimensions and capacity must be positive")
        self.batch_size, self.num_heads, self.head_dim = batch_size, num_heads, head_dim
        self.value_dim = head_dim if value_dim is None else value_dim
        if self.value_dim <= 0:
            raise ValueError("value_dim must be positive")
        self.max_seq_len = max_seq_len
        self.device = as_device(device)
        if self.device.type != "cuda":
            raise ValueError("the B200 KV cache lives on a cuda device")
        self.dtype = _torch_dtype(dtype)
        if not self.dtype.is_floating_point:
            raise TypeError("cache compute dtype must be floating point")
        self.quantized = bool(quantized)
        self.length = 0
        dev = torch.device("cuda", self.device.index)
        shape = (batch_size, num_heads, max_seq_len)
        store = torch.int8 if self.quantized else self.dtype
        self._keys = torch.zeros(shape + (head_dim,), dtype=store, device=dev)
        self._values = torch.zeros(shape + (self.value_dim,), dtype=store, device=dev)
        self._key_scales = torch.ones(shape + (1,), dtype=torch.float32, device=dev) if self.quantized else None
        self._value_scales = torch.ones(shape + (1,), dtype=torch.float32, device=dev) if self.quantized else None
        self._host_lens: np.ndarray | None = None
        self._lens: torch.Tensor | None = None
        self._lens_next: torch.Tensor | None = None

    # -- reference API -----------------------------------------------------
    def append(self, key: Tensor, value: Tensor) -> tuple[Tensor, Tensor]:
        """Append a chunk after validating all shapes and capacity."""
        if key.device != self.device or value.device != self.device:
            raise ValueError("cache and key/value tensors must be on the same device")
        if is_grad_enabled() and (key.requires_grad or value.requires_grad):
            raise RuntimeError("KVCache is inference-only; use no_grad() for differentiable inputs")
        prefix = (self.batch_size, self.num_heads)
        if key.ndim != 4 or key.shape[:2] != prefix or key.shape[-1] != self.head_dim:
            raise ValueError("key shape does not match cache configuration")
        if value.shape != key.shape[:3] + (self.value_dim,):
            raise ValueError("value shape does not match cache configuration")
        steps = key.shape[2]
        top = self.length if self._host_lens is None else int(self._host_lens.max())
        stop = top + steps
        if steps == 0 or stop > self.max_seq_len:
            raise ValueError(f"cache capacity {self.max_seq_len} exceeded or empty append")
        self._write(key._data, value._data, steps)
        return self.get()

    def _write(self, key, value, steps: int) -> None:
        """One append kernel: plain copy/cast, or quantising for int8 storage."""
        where = {"position": self.length} if self._host_lens is None else {
            "positions": self._lens, "positions_out": self._lens_next}
        if self.quantized:
            engine.kv_append_int8(key, value, self._keys, self._values, self._key_scales, self._value_scales,
                                  compute_dtype=self.dtype, **where)
        else:
            engine.kv_append(key, value, self._keys, self._values, **where)
        self._advance(steps)

    def _advance(self, steps: int) -> None:
        if self._host_lens is None:
            self.length += steps
        else:
            self._lens, self._lens_next = self._lens_next, self._lens
            self._host_lens = self._host_lens + steps
            self.length = int(self._host_lens.max())

    def append_rotary(self, key: Tensor, value: Tensor, *, base: float = 10000.0,
                      rotary_dim: int | None = None) -> tuple[Tensor, Tensor]:
        """``append(rotary_embedding(key, self.length), value)`` in one kernel.

        The attention module rotates keys at their cache positions and then
        appends them (nn/transformer.py:139-142, nn/cache.py:54-86); this
        writes the rotated keys straight into the cache (per-row positions
        when the cache has ragged lengths)."""
        dim = self.head_dim if rotary_dim is None else rotary_dim
        if dim <= 0 or dim % 2 or dim > self.head_dim or base <= 0 or not np.isfinite(base):
            raise ValueError("RoPE requires a positive even rotary dimension and valid positions/base")
        if key.device != self.device or value.device != self.device:
            raise ValueError("cache and key/value tensors must be on the same device")
        if is_grad_enabled() and (key.requires_grad or value.requires_grad):
            raise RuntimeError("KVCache is inference-only; use no_grad() for differentiable inputs")
        prefix = (self.batch_size, self.num_heads)
        if key.ndim != 4 or key.shape[:2] != prefix or key.shape[-1] != self.head_dim:
            raise ValueError("key shape does not match cache configuration")
        if value.shape != key.shape[:3] + (self.value_dim,):
            raise ValueError("value shape does not match cache configuration")
        steps = key.shape[2]
        top = self.length if self._host_lens is None else int(self._host_lens.max())
        if steps == 0 or top + steps > self.max_seq_len:
            raise ValueError(f"cache capacity {self.max_seq_len} exceeded or empty append")
        if self.quantized:
            # Rotate, then quantise (the scale of a row depends on its rotated values).
            rotated = engine.rope(key._data, offset=self.length if self._host_lens is None else 0, base=base,
                                  rotary_dim=dim, positions=self._lens)
            self._write(rotated, value._data, steps)
            return self.get()
        where = {"position": self.length} if self._host_lens is None else {
            "positions": self._lens, "positions_out": self._lens_next}
        engine.kv_append_rope(key._data, value._data, self._keys, self._values, base=base, rotary_dim=dim, **where)
        self._advance(steps)
        return self.get()

    def get(self) -> tuple[Tensor, Tensor]:
        keys = self._keys[:, :, : self.length]
        values = self._values[:, :, : self.length]
        if self.quantized:
            # Dequantised copies of the active prefix (nn/cache.py:91-99).
            b, h, n = self.batch_size, self.num_heads, self.length
            keys = torch.empty((b, h, n, self.head_dim), dtype=self.dtype, device=self._keys.device)
            values = torch.empty((b, h, n, self.value_dim), dtype=self.dtype, device=self._keys.device)
            engine.kv_dequant_int8(self._keys, self._key_scales, keys, n)
            engine.kv_dequant_int8(self._values, self._value_scales, values, n)
        return Tensor(keys, device=self.device), Tensor(values, device=self.device)

    def attend(self, query: Tensor, *, scale: float | None = None, causal_offset: int | None = None) -> Tensor:
        """Causal attention of ``query`` [B, Hq, Tq, D] (the newest Tq cached tokens)
        over the cache, without materialising dequantised keys (engine extension).

        Equals ``scaled_dot_product_attention(query, *self.get(), is_causal=True,
        causal_offset=length - Tq, enable_gqa=True)`` (nn/transformer.py:143-154),
        per-row lengths included.  An int8 cache runs the fused-dequant decode
        kernel; shapes outside it dequantise and run the prefill kernels."""
        if query.ndim != 4 or query.shape[0] != self.batch_size or query.shape[-1] != self.head_dim:
            raise ValueError("query shape does not match cache configuration")
        if query.shape[1] % self.num_heads or query.device != self.device:
            raise ValueError("query heads must be a multiple of the cache heads, on the cache device")
        if query.dtype != self.dtype:
            raise TypeError("query dtype must be the cache compute dtype")
        n, tq = self.length, query.shape[2]
        if n == 0 or tq > n:
            raise ValueError("the cache must already hold the query tokens")
        offset = n - tq if causal_offset is None else int(causal_offset)
        kw = dict(is_causal=True, scale=scale, causal_offset=offset, kv_lens=self._lens)
        q = query._data
        if self.quantized:
            try:
                out, _ = engine.decode_int8(q, self._keys[:, :, :n], self._values[:, :, :n], self._key_scales,
                                            self._value_scales, **kw)
                return Tensor(out, device=self.device)
            except engine._lib.EngineError as error:
                if error.status != engine._lib.ERR_UNSUPPORTED:
                    raise
            keys, values = (t._data for t in self.get())
        else:
            keys, values = self._keys[:, :, :n], self._values[:, :, :n]
        if (query.shape[1] // self.num_heads) * tq <= engine.DECODE_MAX_ROWS:
            out, _ = engine.decode(q, keys, values, **kw)
        else:
            out, _ = engine.forward(q, keys, values, need_lse=False, **kw)
        return Tensor(out, device=self.device)

    def reset(self) -> None:
        """Reuse the allocation; future appends overwrite old entries."""
        self.length = 0
        if self._host_lens is not None:
            self.set_lengths(np.zeros(self.batch_size, dtype=np.int64))

    def truncate(self, length: int) -> None:
        if not 0 <= length <= self.length:
            raise ValueError("truncate length must be between zero and the current length")
        self.length = length
        if self._host_lens is not None:
            self.set_lengths(np.minimum(self._host_lens, length))

    def reorder(self, indices) -> None:
        """Reorder or duplicate batch rows for fixed-width beam search (device gather)."""
        raw = indices._data if isinstance(indices, Tensor) else indices
        host = raw.detach().cpu().numpy() if isinstance(raw, torch.Tensor) else np.asarray(raw)
        if host.shape != (self.batch_size,) or host.dtype.kind not in "iu":
            raise ValueError("beam indices must be one integer per cache batch row")
        if (host < 0).any() or (host >= self.batch_size).any():
            raise ValueError("beam index out of range")
        dev = self._keys.device
        order = torch.as_tensor(host.astype(np.int32), device=dev)
        keys, values = torch.empty_like(self._keys), torch.empty_like(self._values)
        engine.kv_reorder(self._keys, keys, order, self.max_seq_len)
        engine.kv_reorder(self._values, values, order, self.max_seq_len)
        self._keys, self._values = keys, values
        if self.quantized:
            ks, vs = torch.empty_like(self._key_scales), torch.empty_like(self._value_scales)
            engine.kv_reorder(self._key_scales, ks, order, self.max_seq_len)
            engine.kv_reorder(self._value_scales, vs, order, self.max_seq_len)
            self._key_scales, self._value_scales = ks, vs
        if self._host_lens is not None:
            self.set_lengths(self._host_lens[host])

    @property
    def storage(self) -> tuple:
        """Raw persistent arrays (keys, values, key scales, value scales)."""
        return self._keys, self._values, self._key_scales, self._value_scales

    @property
    def memory_bytes(self) -> int:
        """Allocated persistent payload (int8 rows plus fp32 scales when quantized)."""
        arrays = [self._keys, self._values]
        if self.quantized:
            arrays += [self._key_scales, self._value_scales]
        return sum(t.numel() * t.element_size() for t in arrays)

    def __len__(self):
        return self.length

    def __repr__(self):
        return (f"KVCache(length={self.length}, capacity={self.max_seq_len}, "
                f"quantized={self.quantized}, device='{self.device}')")

    # -- ragged rows (engine extension) ------------------------------------
    def set_lengths(self, lengths) -> None:
        """Give every batch row its own valid length (keys beyond it are ignored)."""
        host = np.asarray(lengths, dtype=np.int64).reshape(-1)
        if host.shape != (self.batch_size,) or (host < 0).any() or (host > self.max_seq_len).any():
            raise ValueError("lengths must be one value in [0, capacity] per cache batch row")
        dev = self._keys.device
        self._host_lens = host.copy()
        self._lens = torch.as_tensor(host.astype(np.int32), device=dev)
        self._lens_next = torch.empty_like(self._lens)
        self.length = int(host.max()) if host.size else 0

    @property
    def lengths(self) -> np.ndarray:
        """Per-row valid lengths (host copy)."""
        if self._host_lens is None:
            return np.full(self.batch_size, self.length, dtype=np.int64)
        return self._host_lens.copy()

    @property
    def seq_lens(self) -> torch.Tensor | None:
        """Device int32 [B] per-row lengths, or None when every row has ``length`` keys."""
        return self._lens
