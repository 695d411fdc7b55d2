"""tensorsmith ``nn`` attention surface served by the B200 engine."""

from .attention import rotary_embedding, scaled_dot_product_attention  # noqa: F401
from .cache import KVCache  # noqa: F401
from .transformer import (  # noqa: F401
    MultiHeadAttention,
    RMSNorm,
    SwiGLU,
    TransformerConfig,
    TransformerDecoderBlock,
    TransformerLM,
    sample_logits,
)
