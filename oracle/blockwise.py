"""Oracle (test infrastructure): the block-wise per-channel K layout, in numpy.

The reference lists block-wise per-channel K as a roadmap item (README.md:141)
and has no implementation of it, so there is no reference output to pin this
layout to directly.  The oracle states the layout from the reference's own
quantizer: each block of ``block`` consecutive tokens is quantized per channel by
``quantize_int8`` (reference/page_attention_int8_pytorch.py:23-30, restated bit
for bit and pinned to the reference's golden vectors in ``oracle.quant``), with
the amax taken over the block's tokens, the last block over the tokens it holds.
A single block covering the whole sequence is therefore exactly the
reference's per-channel K of one write (tests/qwen_kvcache_full.py:41-47); that
identity is what ties this layout to the pinned rule.  V stays per token.

* ``quant_k_blockwise(x, block)`` -> (codes ``[B,H,S,D]`` int8, scales
  ``[B,H,ceil(S/block),D]`` float32).
* ``decode_blockwise`` dequantizes K with its block scales and V with its token
  scales and runs the reference attention (``page_attention_reference``,
  reference/page_attention_reference.py:31-54) in float64.
"""
from __future__ import annotations

import numpy as np

from .attention import page_attention_reference
from .quant import quantize_int8


def quant_k_blockwise(x: np.ndarray, block: int):
    """Per (block of ``block`` tokens, channel) symmetric int8 of ``x [B,H,S,D]``."""
    x = np.asarray(x, np.float32)
    B, H, S, D = x.shape
    nblk = -(-S // block)
    codes = np.empty((B, H, S, D), np.int8)
    scales = np.empty((B, H, nblk, D), np.float32)
    for i in range(nblk):
        lo, hi = i * block, min(S, (i + 1) * block)
        q, s = quantize_int8(x[:, :, lo:hi], (2,))
        codes[:, :, lo:hi] = q
        scales[:, :, i] = s[:, :, 0]
    return codes, scales


def dequant_k_blockwise(codes: np.ndarray, scales: np.ndarray, block: int) -> np.ndarray:
    """codes ``[B,H,S,D]`` * the scale of each token's block, float32."""
    S = codes.shape[2]
    per_token = np.repeat(np.asarray(scales, np.float32), block, axis=2)[:, :, :S]
    return codes.astype(np.float32) * per_token


def decode_blockwise(q, k_codes, k_scales, v_codes, v_scales, block, sm_scale=None):
    """q ``[B,Hq,D]`` over block-wise K and per-token V (``v_scales [B,H,S]``), float64."""
    k = dequant_k_blockwise(k_codes, k_scales, block)
    S = v_codes.shape[2]
    v = v_codes.astype(np.float32) * np.asarray(v_scales, np.float32).reshape(
        v_codes.shape[0], v_codes.shape[1], S, 1)
    out = page_attention_reference(np.asarray(q, np.float32)[:, :, None, :], k, v, None,
                                   sm_scale, "f64")
    return out[:, :, 0, :]
