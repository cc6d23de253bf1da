"""Oracle (test infrastructure): symmetric int8 quantize-on-write in numpy.

Restates the reference quantizer bit for bit on CPU:

* ``quantize_int8`` follows reference/page_attention_int8_pytorch.py:23-30
  (``amax = |x|.amax(dims).clamp(1e-8)``, ``scale = amax / 127``,
  ``q = clamp(round(x / scale), -127, 127).int8``).  Every step is a float32
  IEEE operation: the divisions are true divisions (not reciprocal
  multiplies) and ``np.rint`` rounds half to even like ``torch.round``.
* ``QuantizedKVCacheOracle`` follows the storage rule of
  ``QuantizedKVCache.update`` (tests/qwen_kvcache_full.py:38-66): K is
  quantized per channel (reduce over the new tokens, dim 2), V per token
  (reduce over D, dim 3); scales are stored as float16; on an append the K
  codes are computed with the *new* call's per-channel scale but the stored
  K scale is the first call's (line 54); ``update`` returns the dequantized
  cache ``(codes.float() * scale_fp16.float()).to(dtype)`` (lines 64-65).

Arrays are numpy; bf16 values are carried as float32 arrays whose values are
bf16-representable, with ``round_to_bf16`` doing the float32 -> bf16
round-to-nearest-even that ``tensor.to(torch.bfloat16)`` does.
"""
from __future__ import annotations

import numpy as np

QMAX = 127.0
AMAX_FLOOR = np.float32(1e-8)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 (round to nearest, ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.float32(np.nan)
    return out


def cast(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` ("f32", "bf16", "f16"), as float32."""
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return round_to_bf16(x)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)
    raise ValueError(dtype)


def pack(x: np.ndarray, dtype: str) -> np.ndarray:
    """Compact storage of ``dtype`` values held in float32: bf16 as uint16 bit
    patterns, f16 as float16, f32 unchanged (used by the golden fixtures)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == "bf16":
        return (x.view(np.uint32) >> 16).astype(np.uint16)
    if dtype == "f16":
        return x.astype(np.float16)
    return x


def unpack(a: np.ndarray, dtype: str) -> np.ndarray:
    """Inverse of ``pack``: float32 array of ``dtype`` values."""
    if dtype == "bf16":
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def quantize_int8(x: np.ndarray, reduce_dims) -> tuple[np.ndarray, np.ndarray]:
    """reference/page_attention_int8_pytorch.py:23-30 -> (int8 codes, float32 scale)."""
    x = np.asarray(x, dtype=np.float32)
    amax = np.abs(x).max(axis=tuple(reduce_dims), keepdims=True) if x.size else np.zeros(
        [1 if i in tuple(reduce_dims) else n for i, n in enumerate(x.shape)], np.float32)
    amax = np.maximum(amax, AMAX_FLOOR).astype(np.float32)
    scale = (amax / np.float32(QMAX)).astype(np.float32)
    q = np.clip(np.rint(x / scale), -QMAX, QMAX).astype(np.int8)
    return q, scale


def dequantize_int8(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """reference/page_attention_int8_pytorch.py:33-34."""
    return q.astype(np.float32) * np.asarray(scale, dtype=np.float32)


def quant_k_perchannel(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """K per channel on ``[B, H, S, D]``: reduce over S (dim 2) -> scale ``[B, H, 1, D]``.

    Same math as tests/qwen_kvcache_full.py:41-43 and the K half of
    src/kernels/quant_kv_triton.py:16-50 (which rounds half away from zero;
    the oracle, like torch, rounds half to even).
    """
    return quantize_int8(x, (2,))


def quant_v_pertoken(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """V per token on ``[B, H, S, D]``: reduce over D (dim 3) -> scale ``[B, H, S, 1]``.

    tests/qwen_kvcache_full.py:45-47; src/kernels/quant_kv_triton.py:55-87.
    """
    return quantize_int8(x, (3,))


def quant_k_static(x: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """Codes of ``x [B, H, S, D]`` for a given per-channel scale (broadcast as
    ``[.., H, 1, D]``): the code step of ``quantize_int8``
    (reference/page_attention_int8_pytorch.py:23-30) - IEEE float32 division,
    round half to even, clamp to +-127 - with the scale supplied (static
    quantization, the reference roadmap item README.md:140)."""
    xf = np.asarray(x, np.float32)
    s = np.asarray(scale, np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        q = np.clip(np.rint(xf / s), -127, 127)
    return np.nan_to_num(q, nan=0.0).astype(np.int8)


def to_f16(scale: np.ndarray) -> np.ndarray:
    """``scale.to(torch.float16)`` (round to nearest even; overflow -> inf)."""
    with np.errstate(over="ignore"):
        return np.asarray(scale, dtype=np.float32).astype(np.float16)


class QuantizedKVCacheOracle:
    """numpy restatement of ``QuantizedKVCache`` (tests/qwen_kvcache_full.py:27-89)."""

    def __init__(self):
        self._k_i8: dict[int, np.ndarray] = {}
        self._v_i8: dict[int, np.ndarray] = {}
        self._k_sc: dict[int, np.ndarray] = {}   # float16 [B, H, 1, D]
        self._v_sc: dict[int, np.ndarray] = {}   # float16 [B, H, S, 1]
        self._lens: dict[int, int] = {}

    def update(self, key_states, value_states, layer_idx, dtype="bf16"):
        """tests/qwen_kvcache_full.py:38-66. Inputs are float32 arrays holding
        ``dtype`` values; returns the dequantized cache rounded to ``dtype``."""
        k_int8, k_scale = quantize_int8(key_states, (2,))
        v_int8, v_scale = quantize_int8(value_states, (3,))
        if layer_idx in self._k_i8:
            self._k_i8[layer_idx] = np.concatenate([self._k_i8[layer_idx], k_int8], axis=2)
            self._v_i8[layer_idx] = np.concatenate([self._v_i8[layer_idx], v_int8], axis=2)
            self._v_sc[layer_idx] = np.concatenate([self._v_sc[layer_idx], to_f16(v_scale)], axis=2)
            # the stored K scale keeps the first call's value (line 54)
        else:
            self._k_i8[layer_idx] = k_int8
            self._v_i8[layer_idx] = v_int8
            self._k_sc[layer_idx] = to_f16(k_scale)
            self._v_sc[layer_idx] = to_f16(v_scale)
        self._lens[layer_idx] = self._k_i8[layer_idx].shape[2]
        return self.dequantized(layer_idx, dtype)

    def dequantized(self, layer_idx, dtype="bf16"):
        """tests/qwen_kvcache_full.py:64-65."""
        with np.errstate(invalid="ignore", over="ignore"):
            k = self._k_i8[layer_idx].astype(np.float32) * self._k_sc[layer_idx].astype(np.float32)
            v = self._v_i8[layer_idx].astype(np.float32) * self._v_sc[layer_idx].astype(np.float32)
        return cast(k, dtype), cast(v, dtype)

    def get_seq_length(self, layer_idx=0):
        return self._lens.get(layer_idx, 0)

    def __len__(self):
        return len(self._k_i8)

    def storage_bytes(self):
        """tests/qwen_kvcache_full.py:75-82: int8 codes 1 B, fp16 scales 2 B."""
        b = sum(t.size for d in (self._k_i8, self._v_i8) for t in d.values())
        b += sum(t.size * 2 for d in (self._k_sc, self._v_sc) for t in d.values())
        return b

    def fp16_equiv_bytes(self):
        """tests/qwen_kvcache_full.py:84-89."""
        return sum(t.size * 2 for d in (self._k_i8, self._v_i8) for t in d.values())
