"""B200-native attention engine for tensorsmith.

Drop-in for tensorsmith's attention path: ``nn.scaled_dot_product_attention``
(forward + VJP), ``nn.KVCache`` and the cached decode it feeds.  Compute runs in
hand-written sm_100a kernels behind the C ABI of include/ts_attn.h
(``libts_attn.so``); this package fills the ABI structs and records the tape
node.  There is no CPU fallback.
"""

from . import engine, nn  # noqa: F401
from .engine import seed  # noqa: F401
from .tensor import Tensor, enable_grad, is_grad_enabled, no_grad, tensor  # noqa: F401

__version__ = "0.1.0"
