"""Oracle (test infrastructure): seeded synthetic inputs for every workload.

No public dataset is involved. The distributions follow the reference's
offline study of Qwen3-0.6B K/V (channel outliers in K, symmetric V;
src/analysis_kvcache/analyze_distribution.py:49-68, data/distribution_report.txt)
as fixed by the workload definitions: K ~ N(0, 1) with 4 random channels per
head scaled x20, V ~ N(0, 1), q ~ N(0, 1).

Generators are numpy ``default_rng(seed)`` so the same bits are produced on
every host; values are rounded to the requested element type (bf16 by
default) and returned as float32.
"""
from __future__ import annotations

import numpy as np

from .quant import cast, quant_k_perchannel, quant_v_pertoken

OUTLIER_CHANNELS = 4
OUTLIER_GAIN = 20.0


def outlier_k(rng, B, H, S, D, dtype="bf16"):
    """K ``[B, H, S, D]`` ~ N(0, 1) with 4 random channels per (b, h) scaled x20."""
    k = rng.standard_normal((B, H, S, D), dtype=np.float32)
    for b in range(B):
        for h in range(H):
            ch = rng.permutation(D)[:OUTLIER_CHANNELS]
            k[b, h, :, ch] *= np.float32(OUTLIER_GAIN)
    return cast(k, dtype)


def normal(rng, shape, dtype="bf16"):
    return cast(rng.standard_normal(shape, dtype=np.float32), dtype)


def decode_case(seed, B, Hq, Hkv, S, D, kv_dtype="bf16", q_dtype="bf16"):
    """One decode-attention case: q ``[B, Hq, D]`` plus the int8 cache the
    oracle quantizer makes from outlier K and normal V (fp32 scales)."""
    rng = np.random.default_rng(seed)
    k = outlier_k(rng, B, Hkv, S, D, kv_dtype)
    v = normal(rng, (B, Hkv, S, D), kv_dtype)
    q = normal(rng, (B, Hq, D), q_dtype)
    k_i8, k_sc = quant_k_perchannel(k)
    v_i8, v_sc = quant_v_pertoken(v)
    return dict(q=q, k=k, v=v, k_i8=k_i8, k_sc=k_sc, v_i8=v_i8, v_sc=v_sc)


def config0(seed=0):
    """CPU reference single layer: B=1, Hq=16, Hkv=8, D=128, S=512, float32."""
    rng = np.random.default_rng(seed)
    k = outlier_k(rng, 1, 8, 512, 128, "f32")
    v = normal(rng, (1, 8, 512, 128), "f32")
    q = normal(rng, (1, 16, 128), "f32")
    return q, k, v
