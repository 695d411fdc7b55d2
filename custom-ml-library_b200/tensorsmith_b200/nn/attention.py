"""``scaled_dot_product_attention`` on the B200 engine, with tensorsmith's API.

Signature, argument meaning, validation order, exception types and messages
follow tensorsmith's src/tensorsmith/nn/attention.py:16-87; the compute behind
it is the engine (tcgen05 prefill, CUDA-core generic path, split-K decode) and
the VJP is the engine's recomputing backward, recorded as one tape node like
nn/attention.py:250-252 (``tensorsmith_b200.interop.attention_node``, which
works with tensorsmith's own Tensor class as well as the torch-backed mirror).  Every ``backend`` string routes to the engine on
CUDA (all of them are exact attention); there is no host fallback.
"""

from __future__ import annotations

import math

from .. import engine, interop
from ..tensor import Tensor, is_grad_enabled

BACKENDS = {"auto", "dense", "streaming", "native"}


def scaled_dot_product_attention(
    query: Tensor,
    key: Tensor,
    value: Tensor,
    attn_mask: Tensor | None = None,
    dropout_p: float = 0.0,
    is_causal: bool = False,
    *,
    scale: float | None = None,
    causal_offset: int = 0,
    backend: str = "auto",
    block_size: int = 64,
    enable_gqa: bool = False,
    kv_lens=None,
) -> Tensor:
    """Attention for [batch, heads, sequence, channels] tensors.

    Boolean masks use True=allowed; floating masks are added to scores. Fully
    masked rows return zero with zero gradients. ``causal_offset`` is the
    absolute position of the first query in a cached key sequence.

    Engine extension: ``kv_lens`` (int32 [B] on the device) gives each batch
    row its own number of valid keys, with its queries at the end of them;
    it is what ``KVCache`` passes for ragged rows.
    """
    if any(t.ndim != 4 for t in (query, key, value)):
        raise ValueError("attention expects [batch, heads, sequence, channels]")
    if query.device != key.device or query.device != value.device:
        raise ValueError("attention tensors must be on the same device")
    if query.dtype != key.dtype or query.dtype != value.dtype or "float" not in str(query.dtype):
        raise TypeError("attention inputs must have the same floating-point dtype")
    if query.shape[0] != key.shape[0] or key.shape[:3] != value.shape[:3]:
        raise ValueError("attention batch/head dimensions and key/value lengths must agree")
    repetitions = query.shape[1] // key.shape[1] if key.shape[1] else 0
    if query.shape[1] != key.shape[1] and (
        not enable_gqa or not repetitions or query.shape[1] % key.shape[1]
    ):
        raise ValueError(
            "grouped-query attention requires enable_gqa and query heads divisible by KV heads"
        )
    if query.shape[-1] != key.shape[-1] or min(*query.shape, *key.shape, *value.shape) <= 0:
        raise ValueError("query/key head dimensions must match and sequences must be nonempty")
    if not 0 <= dropout_p < 1 or block_size <= 0 or causal_offset < 0:
        raise ValueError("invalid dropout probability, block size, or causal offset")
    if backend not in BACKENDS:
        raise ValueError("attention backend must be auto, dense, streaming, or native")
    if query.device.type != "cuda":
        raise ValueError("the B200 attention engine runs on cuda tensors")
    b, h, qlen, dim = query.shape
    multiplier = 1 / math.sqrt(dim) if scale is None else scale
    if not math.isfinite(multiplier):
        raise ValueError("attention scale must be finite")
    mask = None
    if attn_mask is not None:
        if not any(name in str(attn_mask.dtype) for name in ("bool", "float")):
            raise TypeError("attention masks must be boolean or floating point")
        if attn_mask.requires_grad or attn_mask.device != query.device:
            raise ValueError("attention masks must be non-differentiable and on the input device")
        mask = attn_mask._data
        try:
            mask.expand(b, h, qlen, key.shape[2])
        except RuntimeError as error:
            raise ValueError("attention mask is not broadcastable to [B,H,Q,K]") from error
    # Backend names select nothing on CUDA (every one is exact attention on the engine),
    # but dropout keeps the reference's rule: dense only (nn/attention.py:76-83).
    selected = ("dense" if dropout_p else "native") if backend == "auto" else backend
    if selected in {"native", "streaming"} and dropout_p:
        raise ValueError("attention dropout currently requires the dense backend")

    recording = is_grad_enabled() and any(t.requires_grad for t in (query, key, value))
    dropout = engine.DROPOUT_GENERATOR.draw(dropout_p) if dropout_p else None  # one draw per call
    return interop.attention_node(query, key, value, mask=mask, is_causal=is_causal, scale=multiplier,
                                  causal_offset=causal_offset, kv_lens=kv_lens, dropout=dropout,
                                  op="sdpa_" + selected, recording=recording, decode_rows=repetitions * qlen)


def rotary_embedding(input: Tensor, offset: int = 0, base: float = 10000.0, rotary_dim: int | None = None) -> Tensor:
    """Interleaved-pair RoPE for [..., sequence, channels], with inverse-rotation VJP.

    Signature, validation and semantics of nn/attention.py:255-296; computed by
    the engine's rope kernel (per-operation rounding in the input dtype)."""
    if input.ndim < 2:
        raise ValueError("RoPE requires at least sequence and channel dimensions")
    dim = input.shape[-1] if rotary_dim is None else rotary_dim
    if (
        dim <= 0
        or dim % 2
        or dim > input.shape[-1]
        or offset < 0
        or base <= 0
        or not math.isfinite(base)
    ):
        raise ValueError("RoPE requires a positive even rotary dimension and valid positions/base")
    if input.device.type != "cuda":
        raise ValueError("the B200 attention engine runs on cuda tensors")
    raw = input._data
    shape = raw.shape
    x4 = raw.reshape((-1,) + tuple(shape[-2:]))[None] if raw.dim() != 4 else raw
    out = engine.rope(x4, offset=offset, base=base, rotary_dim=dim).reshape(shape)

    def backward(g):
        g4 = g.reshape((-1,) + tuple(shape[-2:]))[None] if g.dim() != 4 else g
        return (engine.rope(g4.contiguous() if not g4.is_contiguous() else g4, offset=offset, base=base,
                            rotary_dim=dim, inverse=True).reshape(shape),)

    return Tensor._from_op(out, (input,), backward, "rope")
