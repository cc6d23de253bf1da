"""B200-native (sm_100a) int8 KV cache for Qwen3-style GQA decoding.

Hot paths, as hand-written CUDA behind a C ABI (``include/halftone_b200.h``):
fused symmetric-int8 quantize-on-write (K per channel, V per token) and
split-KV int8 decode attention.  ``integration`` holds the drop-in surface of
the reference: ``QuantizedKVCache`` (an HF ``DynamicCache``) and the patched
Qwen3 ``eager_attention_forward``.
"""
from . import kernels
from ._lib import HalftoneError

__all__ = ["kernels", "HalftoneError"]
__version__ = "0.1.0"
