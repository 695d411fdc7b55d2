"""tensorsmith's decoder-only transformer with its attention path on the engine.

Mirrors src/tensorsmith/nn/transformer.py: ``MultiHeadAttention`` (:49-155),
``TransformerDecoderBlock`` (:158-194), ``TransformerConfig`` (:197-223),
``TransformerLM`` with cached ``forward`` / ``new_cache`` / ``generate``
(:226-402) and ``sample_logits`` (:405-439) -- same constructor arguments,
validation, error types and messages, cache rollback and ``logits_to_keep``.

What runs where:
  * the attention path is the engine: RoPE (``ts_rope``), the fused
    RoPE + KV-cache append (``ts_kv_append_rope``, ``KVCache.append_rotary``),
    and attention through ``nn.scaled_dot_product_attention`` (tcgen05 prefill,
    split-K decode, generic kernels) with ``causal_offset`` = the cache length;
  * projections, RMSNorm, SwiGLU, embeddings and the loss are plain torch ops
    on the device (tensorsmith's own GEMMs and elementwise ops are outside the
    attention path).

Tensors at this module's boundary are torch tensors (token ids int64
[B, T]; logits fp32 [B, T, V]).  Training works through torch autograd: RoPE
and attention are ``torch.autograd.Function`` nodes whose backward is the
engine's inverse rotation and recomputing attention backward.  Parameters are
fp32; ``torch.autocast`` gives the fp16 mixed precision of tensorsmith's
``amp.autocast`` (the projections hand fp16 q/k/v to the engine).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from .. import engine
from ..tensor import Tensor, is_grad_enabled, no_grad
from .attention import BACKENDS, scaled_dot_product_attention
from .cache import KVCache


def _grad_mode() -> bool:
    """Recording is on when both tensorsmith's grad mode (the mirror's) and torch's are on."""
    return is_grad_enabled() and torch.is_grad_enabled()


class _RopeFn(torch.autograd.Function):
    """Interleaved-pair RoPE (nn/attention.py:255-296) on the engine; VJP = inverse rotation."""

    @staticmethod
    def forward(ctx, x, offset):
        ctx.offset = offset
        return engine.rope(x, offset=offset)

    @staticmethod
    def backward(ctx, g):
        return engine.rope(g.contiguous(), offset=ctx.offset, inverse=True), None


class _AttentionFn(torch.autograd.Function):
    """Attention forward / recomputing backward on the engine (nn/attention.py:132-252)."""

    @staticmethod
    def forward(ctx, q, k, v, is_causal, causal_offset, scale, dropout):
        out, lse = engine.forward(q, k, v, is_causal=is_causal, causal_offset=causal_offset, scale=scale,
                                  need_lse=True, dropout=dropout)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.kw = dict(is_causal=is_causal, causal_offset=causal_offset, scale=scale, dropout=dropout)
        return out

    @staticmethod
    def backward(ctx, g):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = engine.backward(q, k, v, out, lse, g.contiguous(), **ctx.kw)
        return dq, dk, dv, None, None, None, None


def _param(shape, bound=None, *, std=None, device=None, ones=False):
    if ones:
        data = np.ones(shape, np.float32)
    elif std is not None:
        data = np.random.normal(0, std, shape).astype(np.float32)
    else:
        data = np.random.uniform(-bound, bound, shape).astype(np.float32)
    return torch.tensor(data, device=device, requires_grad=True)


class _Module:
    """Parameter container with tensorsmith's state-dict naming and train/eval modes."""

    training = True

    def _children(self):
        for name, value in vars(self).items():
            if isinstance(value, _Module):
                yield name, value
            elif isinstance(value, list):
                for i, item in enumerate(value):
                    if isinstance(item, _Module):
                        yield f"{name}.{i}", item

    def modules(self):
        yield self
        for _, child in self._children():
            yield from child.modules()

    def named_parameters(self, prefix=""):
        seen = set()
        for name, value in vars(self).items():
            if isinstance(value, torch.Tensor) and value.requires_grad and id(value) not in seen:
                seen.add(id(value))
                yield (f"{prefix}{name}", value)
        for name, child in self._children():
            for full, value in child.named_parameters(f"{prefix}{name}."):
                if id(value) not in seen:
                    seen.add(id(value))
                    yield full, value

    def parameters(self):
        return [p for _, p in self.named_parameters()]

    def state_dict(self):
        return {name: p.detach().cpu().numpy() for name, p in self.named_parameters()}

    def load_state_dict(self, state):
        params = dict(self.named_parameters())
        missing = set(params) - set(state)
        unexpected = set(state) - set(params)
        if missing or unexpected:
            raise KeyError(f"state dict mismatch: missing {sorted(missing)}, unexpected {sorted(unexpected)}")
        with torch.no_grad():
            for name, value in state.items():
                target = params[name]
                src = torch.as_tensor(np.asarray(value))
                if tuple(src.shape) != tuple(target.shape):
                    raise ValueError(f"shape mismatch for {name}: {tuple(src.shape)} vs {tuple(target.shape)}")
                target.copy_(src.to(target.dtype))

    def train(self, mode: bool = True):
        for module in self.modules():
            module.training = mode
        return self

    def eval(self):
        return self.train(False)

    def __call__(self, *args, **kwargs):
        return self.forward(*args, **kwargs)


class Linear(_Module):
    """x @ W^T (+ b), W [out, in] ~ U(-1/sqrt(in), 1/sqrt(in)) as nn/layers.py:20-31."""

    def __init__(self, in_features, out_features, bias=True, device=None):
        bound = 1 / math.sqrt(in_features)
        self.weight = _param((out_features, in_features), bound, device=device)
        self.bias = _param((out_features,), bound, device=device) if bias else None

    def forward(self, x):
        return F.linear(x, self.weight, self.bias)


class RMSNorm(_Module):
    """x * rsqrt(mean(x^2) + eps) * weight, computed in fp32 (nn/primitives.py:66-139)."""

    def __init__(self, dim, eps=1e-6, device=None):
        if dim <= 0:
            raise ValueError("normalization dimension must be positive")
        self.eps = eps
        self.weight = _param((dim,), ones=True, device=device)

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight
        return y.to(x.dtype)


class SwiGLU(_Module):
    def __init__(self, dim, hidden_dim, dropout=0.0, device=None):
        self.gate = Linear(dim, hidden_dim, bias=False, device=device)
        self.up = Linear(dim, hidden_dim, bias=False, device=device)
        self.down = Linear(hidden_dim, dim, bias=False, device=device)
        self.dropout = dropout

    def forward(self, x):
        h = self.down(F.silu(self.gate(x)) * self.up(x))
        return F.dropout(h, self.dropout, self.training) if self.dropout else h


def _mirror(t: torch.Tensor) -> Tensor:
    return Tensor(t, device=t.device)


class MultiHeadAttention(_Module):
    """Self attention with grouped-query heads and rotary positions (nn/transformer.py:49-155)."""

    def __init__(self, embed_dim, num_heads, *, num_kv_heads=None, dropout=0.0, bias=False, rotary=True,
                 backend="auto", device=None):
        kv_heads = num_heads if num_kv_heads is None else num_kv_heads
        if min(embed_dim, num_heads, kv_heads) <= 0 or embed_dim % num_heads or num_heads % kv_heads:
            raise ValueError("embed_dim must divide into heads and query heads must divide into KV groups")
        self.embed_dim, self.num_heads, self.num_kv_heads = embed_dim, num_heads, kv_heads
        self.head_dim = embed_dim // num_heads
        if rotary and self.head_dim % 2:
            raise ValueError("rotary attention requires an even head dimension")
        if not 0 <= dropout < 1 or backend not in BACKENDS:
            raise ValueError("invalid attention dropout/backend")
        self.rotary, self.backend, self.dropout_p = rotary, backend, dropout
        self.q_proj = Linear(embed_dim, embed_dim, bias=bias, device=device)
        self.k_proj = Linear(embed_dim, kv_heads * self.head_dim, bias=bias, device=device)
        self.v_proj = Linear(embed_dim, kv_heads * self.head_dim, bias=bias, device=device)
        self.out_proj = Linear(embed_dim, embed_dim, bias=bias, device=device)

    def forward(self, input, context=None, *, attn_mask=None, is_causal=True, cache: KVCache | None = None):
        if input.ndim != 3 or input.shape[-1] != self.embed_dim:
            raise ValueError("attention input must be [batch, sequence, embed_dim]")
        source = input if context is None else context
        if source.ndim != 3 or source.shape[0] != input.shape[0] or source.shape[-1] != self.embed_dim:
            raise ValueError("attention context must be [batch, sequence, embed_dim]")
        recording = _grad_mode()
        if cache is not None and (self.training or recording or context is not None):
            raise RuntimeError(
                "cached self-attention requires eval() and no_grad(); cross-attention caching is not supported"
            )
        batch, steps, _ = input.shape
        offset = 0 if cache is None else cache.length
        if attn_mask is not None:
            expected = (batch, self.num_heads, steps, offset + source.shape[1])
            try:
                if np.broadcast_shapes(tuple(attn_mask.shape), expected) != expected:
                    raise ValueError("mask expands attention dimensions")
                if attn_mask.dtype != torch.bool and not attn_mask.is_floating_point():
                    raise TypeError("attention masks must be boolean or floating point")
            except ValueError as error:
                raise ValueError("attention mask is not broadcastable to [B,H,Q,K]") from error
        # [B, T, H, D] projections viewed as [B, H, T, D] (strided, no copy; the kernels take strides)
        q = self.q_proj(input).reshape(batch, steps, self.num_heads, self.head_dim).permute(0, 2, 1, 3)
        k = self.k_proj(source).reshape(batch, source.shape[1], self.num_kv_heads, self.head_dim).permute(0, 2, 1, 3)
        v = self.v_proj(source).reshape(batch, source.shape[1], self.num_kv_heads, self.head_dim).permute(0, 2, 1, 3)
        gqa = self.num_kv_heads != self.num_heads
        dropout = self.dropout_p if self.training else 0.0
        if recording and attn_mask is None:
            # Training: autograd nodes over the engine's RoPE and attention kernels.
            if self.rotary:
                q = _RopeFn.apply(q, offset)
                k = _RopeFn.apply(k, offset if context is None else 0)
            draw = engine.DROPOUT_GENERATOR.draw(dropout) if dropout else None
            attended = _AttentionFn.apply(q, k, v, is_causal, offset, 1 / math.sqrt(self.head_dim), draw)
        else:
            if recording:
                raise NotImplementedError("training with an explicit attention mask is not routed to the engine")
            q_t = _mirror(engine.rope(q, offset=offset) if self.rotary else q)
            if cache is not None:
                # RoPE of the keys at their cache positions fused into the append (nn/transformer.py:139-142).
                if self.rotary:
                    k_t, v_t = cache.append_rotary(_mirror(k), _mirror(v))
                else:
                    k_t, v_t = cache.append(_mirror(k), _mirror(v))
            else:
                k_t = _mirror(engine.rope(k, offset=offset if context is None else 0) if self.rotary else k)
                v_t = _mirror(v)
            mask = None if attn_mask is None else _mirror(attn_mask)
            attended = scaled_dot_product_attention(q_t, k_t, v_t, mask, dropout, is_causal, causal_offset=offset,
                                                    backend=self.backend, enable_gqa=gqa)._data
        return self.out_proj(attended.permute(0, 2, 1, 3).reshape(batch, steps, self.embed_dim))


class TransformerDecoderBlock(_Module):
    """Pre-RMSNorm block: GQA/RoPE attention and a SwiGLU MLP (nn/transformer.py:158-194)."""

    def __init__(self, dim, num_heads, hidden_dim=None, *, num_kv_heads=None, dropout=0.0,
                 attention_backend="auto", device=None):
        self.attention_norm = RMSNorm(dim, device=device)
        self.attention = MultiHeadAttention(dim, num_heads, num_kv_heads=num_kv_heads, dropout=dropout,
                                            backend=attention_backend, device=device)
        self.residual_dropout = dropout
        self.ffn_norm = RMSNorm(dim, device=device)
        self.ffn = SwiGLU(dim, hidden_dim or 4 * dim, dropout, device)

    def forward(self, input, *, cache=None, attn_mask=None):
        a = self.attention(self.attention_norm(input), cache=cache, attn_mask=attn_mask)
        if self.residual_dropout and self.training:
            a = F.dropout(a, self.residual_dropout, True)
        hidden = input + a
        return hidden + self.ffn(self.ffn_norm(hidden))


@dataclass(frozen=True)
class TransformerConfig:
    vocab_size: int
    dim: int = 128
    num_heads: int = 4
    num_layers: int = 4
    hidden_dim: int | None = None
    num_kv_heads: int | None = None
    max_seq_len: int = 1024
    dropout: float = 0.0
    tie_weights: bool = True
    attention_backend: str = "auto"

    def __post_init__(self):
        if min(self.vocab_size, self.dim, self.num_heads, self.num_layers, self.max_seq_len) <= 0:
            raise ValueError("transformer dimensions must be positive")
        if self.hidden_dim is not None and self.hidden_dim <= 0:
            raise ValueError("hidden_dim must be positive")
        kv = self.num_heads if self.num_kv_heads is None else self.num_kv_heads
        if kv <= 0 or self.dim % self.num_heads or self.num_heads % kv or (self.dim // self.num_heads) % 2:
            raise ValueError("invalid attention head configuration")
        if not 0 <= self.dropout < 1:
            raise ValueError("dropout must be in [0, 1)")
        if self.attention_backend not in BACKENDS:
            raise ValueError("invalid attention backend")


def _as_tokens(tokens, device) -> torch.Tensor:
    if isinstance(tokens, Tensor):
        tokens = tokens._data
    t = torch.as_tensor(np.asarray(tokens) if not isinstance(tokens, torch.Tensor) else tokens)
    return t.to(device)


class TransformerLM(_Module):
    """Decoder-only language model with [B, T, V] logits and cached generation (nn/transformer.py:226-402)."""

    def __init__(self, config: TransformerConfig, device="cuda"):
        self.config = config
        self.device = torch.device(device)
        self._device_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.device = torch.device("cuda", self._device_index)
        self.token_embedding_weight = _param((config.vocab_size, config.dim), std=0.02, device=device)
        self.blocks = [
            TransformerDecoderBlock(config.dim, config.num_heads, config.hidden_dim, num_kv_heads=config.num_kv_heads,
                                    dropout=config.dropout, attention_backend=config.attention_backend,
                                    device=device)
            for _ in range(config.num_layers)
        ]
        self.final_norm = RMSNorm(config.dim, device=device)
        self.output_weight = (self.token_embedding_weight if config.tie_weights
                              else _param((config.vocab_size, config.dim), std=0.02, device=device))

    # tensorsmith's parameter names ("token_embedding.weight", "blocks.0.attention.q_proj.weight", ...)
    def named_parameters(self, prefix=""):
        for name, value in super().named_parameters(prefix):
            yield name.replace("token_embedding_weight", "token_embedding.weight"), value

    def forward(self, tokens, *, caches: list[KVCache] | None = None, attn_mask=None, logits_to_keep: int = 0):
        tokens = _as_tokens(tokens, self.device)
        if tokens.ndim != 2 or tokens.dtype not in (torch.int32, torch.int64) or tokens.shape[1] == 0:
            raise ValueError("tokens must be a nonempty integer [batch, time] tensor")
        if not isinstance(logits_to_keep, int) or not 0 <= logits_to_keep <= tokens.shape[1]:
            raise ValueError("logits_to_keep must be between zero (all) and the input length")
        offset = 0
        if caches is not None:
            if len(caches) != len(self.blocks) or len({cache.length for cache in caches}) != 1:
                raise ValueError("provide one cache per block, all at the same sequence position")
            if self.training or _grad_mode():
                raise RuntimeError("cached decoding requires eval() and no_grad()")
            offset = caches[0].length
            for block, cache in zip(self.blocks, caches):
                if cache.batch_size != tokens.shape[0] or cache.device.index != self._device_index:
                    raise ValueError("cache batch/device does not match tokens")
                if offset + tokens.shape[1] > cache.max_seq_len:
                    raise ValueError("cache capacity exceeded")
                attention = block.attention
                if (cache.num_heads != attention.num_kv_heads or cache.head_dim != attention.head_dim
                        or cache.value_dim != attention.head_dim or cache.dtype != self.token_embedding_weight.dtype):
                    raise ValueError("cache head configuration/dtype does not match model")
        if offset + tokens.shape[1] > self.config.max_seq_len:
            raise ValueError("model context length exceeded")
        hidden = F.embedding(tokens.long(), self.token_embedding_weight)
        if self.config.dropout and self.training:
            hidden = F.dropout(hidden, self.config.dropout, True)
        try:
            for i, block in enumerate(self.blocks):
                hidden = block(hidden, cache=None if caches is None else caches[i], attn_mask=attn_mask)
            if logits_to_keep:
                hidden = hidden[:, -logits_to_keep:, :]
            return F.linear(self.final_norm(hidden), self.output_weight).float()
        except Exception:
            if caches is not None:
                # Roll every cache back to where this call started (nn/transformer.py:308-312).
                for cache in caches:
                    cache.truncate(offset)
            raise

    def loss(self, tokens, targets, *, ignore_index=-100, label_smoothing=0.0):
        logits = self(tokens)
        targets = _as_tokens(targets, self.device).long()
        return F.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.reshape(-1), ignore_index=ignore_index,
                               label_smoothing=label_smoothing)

    def new_cache(self, batch_size: int, max_seq_len: int | None = None, *, quantized=False) -> list[KVCache]:
        capacity = self.config.max_seq_len if max_seq_len is None else max_seq_len
        if capacity <= 0 or capacity > self.config.max_seq_len:
            raise ValueError("cache capacity must fit the model context")
        return [
            KVCache(batch_size, block.attention.num_kv_heads, block.attention.head_dim, capacity,
                    device=f"cuda:{self._device_index}", dtype=self.token_embedding_weight.dtype, quantized=quantized)
            for block in self.blocks
        ]

    def generate(self, prompt, max_new_tokens: int, *, temperature=1.0, top_k: int | None = None, top_p: float = 1.0,
                 eos_token_id: int | None = None, use_cache: bool = True, quantized_cache: bool = False,
                 generator: torch.Generator | None = None) -> torch.Tensor:
        """Batched greedy / top-k / nucleus sampling; returns prompt plus generated tokens."""
        prompt = _as_tokens(prompt, self.device)
        if prompt.ndim != 2 or prompt.shape[1] == 0 or max_new_tokens < 0 or prompt.dtype not in (torch.int32,
                                                                                                   torch.int64):
            raise ValueError("invalid prompt or generation length")
        if prompt.shape[1] + max_new_tokens > self.config.max_seq_len:
            raise ValueError("generation exceeds the configured context length")
        if temperature < 0 or not np.isfinite(temperature) or not 0 < top_p <= 1:
            raise ValueError("temperature must be finite/nonnegative and top_p in (0,1]")
        if top_k is not None and not 1 <= top_k <= self.config.vocab_size:
            raise ValueError("top_k must be within the vocabulary")
        if eos_token_id is not None and not 0 <= eos_token_id < self.config.vocab_size:
            raise ValueError("eos_token_id out of range")
        modes = [(module, module.training) for module in self.modules()]
        try:
            self.eval()
            with no_grad(), torch.no_grad():
                caches = (self.new_cache(prompt.shape[0], prompt.shape[1] + max_new_tokens, quantized=quantized_cache)
                          if use_cache and max_new_tokens else None)
                result, current = prompt.long(), prompt.long()
                finished = torch.zeros(prompt.shape[0], dtype=torch.bool, device=self.device)
                for _ in range(max_new_tokens):
                    logits = self(current, caches=caches, logits_to_keep=1)[:, -1, :]
                    next_token = sample_logits(logits, temperature, top_k, top_p, generator=generator)
                    if eos_token_id is not None:
                        next_token = torch.where(finished, torch.full_like(next_token, eos_token_id), next_token)
                        finished = finished | (next_token == eos_token_id)
                    result = torch.cat((result, next_token[:, None]), dim=1)
                    if eos_token_id is not None and bool(finished.all()):
                        break
                    current = next_token[:, None] if caches is not None else result
        finally:
            for module, mode in modes:
                module.training = mode
        return result


def sample_logits(logits, temperature: float = 1.0, top_k: int | None = None, top_p: float = 1.0, *,
                  generator: torch.Generator | None = None) -> torch.Tensor:
    """Device-resident sampling from [batch, vocabulary] logits (nn/transformer.py:405-439)."""
    if logits.ndim != 2 or temperature < 0 or not np.isfinite(temperature) or not 0 < top_p <= 1:
        raise ValueError("invalid sampling configuration")
    vocab = logits.shape[-1]
    if top_k is not None and not 1 <= top_k <= vocab:
        raise ValueError("top_k must be within the vocabulary")
    if temperature == 0:
        return logits.argmax(dim=-1)
    scores = logits.float() / temperature
    if top_k is not None:
        candidate_scores, candidates = scores.topk(top_k, dim=-1)  # sorted, descending
        order, sorted_scores = candidates, candidate_scores
    else:
        sorted_scores, order = scores.sort(dim=-1, descending=True)
    probabilities = torch.softmax(sorted_scores, dim=-1)
    if top_p < 1:
        keep = probabilities.cumsum(-1) - probabilities < top_p
        probabilities = torch.where(keep, probabilities, torch.zeros_like(probabilities))
        probabilities = probabilities / probabilities.sum(-1, keepdim=True)
    uniform = torch.rand((logits.shape[0], 1), device=logits.device, generator=generator)
    cumulative = probabilities.cumsum(-1)
    cumulative = cumulative / cumulative[:, -1:]
    chosen = (cumulative < uniform).sum(-1).clamp(max=order.shape[-1] - 1)
    return order.gather(1, chosen[:, None])[:, 0]
