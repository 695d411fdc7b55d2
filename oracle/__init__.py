"""CPU oracle for the attention path.  TEST INFRASTRUCTURE ONLY.

Imported only by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / reference arm, and only as the checker.  The shipped engine
never imports this package.
"""

from .attention import (  # noqa: F401
    KVCacheOracle,
    attention_backward,
    attention_backward_dense,
    attention_forward,
    causal_pairs,
    compute_dtype,
    decode_attention,
    key_valid_mask,
    quantize_int8,
    rope,
)
