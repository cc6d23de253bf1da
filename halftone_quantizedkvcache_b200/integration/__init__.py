"""The reference's drop-in surface (its empty src/integration/quantized_attention.py)."""
from .quantized_attention import (Q_DIMS, QuantizedKVCache, install, installed, is_installed,
                                  quantized_attention_forward, uninstall)

__all__ = ["Q_DIMS", "QuantizedKVCache", "install", "installed", "is_installed",
           "quantized_attention_forward", "uninstall"]
