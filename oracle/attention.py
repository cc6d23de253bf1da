"""Oracle (test infrastructure): decode attention over an int8 KV cache, in numpy.

* ``page_attention_reference`` restates reference/page_attention_reference.py:23-54
  (``repeat_kv`` GQA, ``q @ K^T / sqrt(D)``, float32 softmax, ``@ V``).
* ``decode_int8`` is the int8 decode the reference kernel computes
  (src/kernels/int8_decode_attn_triton.py:15-63, checked there against
  ``_ref`` on dequantized K/V at :131-135,168-169): dequantize K per channel
  and V per token (reference/page_attention_int8_pytorch.py:33-34), then the
  attention above.
* ``quant_dequant`` restates the per-token q fake quantization of the HF patch
  (tests/qwen_kvcache_full.py:19-23,103).
* ``prefill_int8`` restates the patch's prefill branch (causal, several
  queries) over the dequantized cache that update() returns (:64-65,95-113).
* ``split_partials`` / ``lse_combine`` restate the flash-decoding split: each
  sequence chunk yields (m, l, o) with m the running max of the base-2 scaled
  scores, l = sum 2^(s - m), o = sum 2^(s - m) v; the combine rescales by
  2^(m_i - M).  The reference has no split (one program per q head,
  int8_decode_attn_triton.py:104); the combined result must equal the
  unsplit attention to float32 round-off.

Arrays: q ``[B, Hq, D]``, K/V ``[B, Hkv, S, D]``; ``acc`` picks float32 (the
reference's own precision) or float64 (a tighter checker).
"""
from __future__ import annotations

import math

import numpy as np

from .quant import cast, dequantize_int8, quantize_int8

LOG2E = 1.4426950408889634


def repeat_kv(x: np.ndarray, n_rep: int, axis: int = 1) -> np.ndarray:
    """reference/page_attention_reference.py:23-28: q head h reads kv head h // n_rep."""
    return x if n_rep == 1 else np.repeat(x, n_rep, axis=axis)


def page_attention_reference(q, k, v, n_rep=None, sm_scale=None, acc="f32"):
    """reference/page_attention_reference.py:31-54 with a batch axis.

    q ``[B, Hq, Sq, D]`` or ``[Hq, Sq, D]``; k, v ``[B, Hkv, S, D]`` or ``[Hkv, S, D]``.
    """
    dt = np.float64 if acc == "f64" else np.float32
    batched = q.ndim == 4
    if not batched:
        q, k, v = q[None], k[None], v[None]
    hq, hkv, d = q.shape[1], k.shape[1], q.shape[-1]
    if n_rep is None:
        assert hq % hkv == 0
        n_rep = hq // hkv
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(d)
    # grouped GQA without materialising repeat_kv: q head h = g * n_rep + r reads kv head g
    B, _, Sq, _ = q.shape
    qg = q.astype(dt).reshape(B, hkv, n_rep, Sq, d)
    scores = np.matmul(qg, np.swapaxes(k.astype(dt), -1, -2)[:, :, None]) * dt(sm_scale)
    scores = scores - scores.max(axis=-1, keepdims=True)
    p = np.exp(scores)
    p = p / p.sum(axis=-1, keepdims=True)
    out = np.matmul(p, v.astype(dt)[:, :, None]).reshape(B, hq, Sq, d)
    return out if batched else out[0]


def decode_int8(q, k_i8, k_sc, v_i8, v_sc, n_rep=None, sm_scale=None, acc="f32"):
    """Int8 decode attention: q ``[B, Hq, D]`` -> ``[B, Hq, D]``.

    k_sc ``[B, Hkv, 1, D]`` (or ``[B, Hkv, D]``), v_sc ``[B, Hkv, S, 1]`` (or ``[B, Hkv, S]``).
    """
    B, Hkv, S, D = k_i8.shape
    k_sc = np.asarray(k_sc, np.float32).reshape(B, Hkv, 1, D)
    v_sc = np.asarray(v_sc, np.float32).reshape(B, Hkv, S, 1)
    k = dequantize_int8(k_i8, k_sc)
    v = dequantize_int8(v_i8, v_sc)
    out = page_attention_reference(np.asarray(q, np.float32)[:, :, None, :], k, v, n_rep,
                                   sm_scale, acc)
    return out[:, :, 0, :]


def prefill_int8(q, k_i8, k_sc, v_i8, v_sc, n_rep=None, sm_scale=None, dtype="bf16",
                 q_quant=True, acc="f64"):
    """The prefill branch of the reference's patched attention over its cache
    (tests/qwen_kvcache_full.py:95-113 on the update() return value, :64-65).

    q ``[B, Hq, Sq, D]`` (values of ``dtype``); codes ``[B, Hkv, S, D]`` with
    ``S >= Sq``; k_sc ``[B, Hkv, 1, D]``, v_sc ``[B, Hkv, S, 1]``.  K and V are
    dequantized and rounded to ``dtype`` as update() returns them, q is
    per-token fake-quantized (line 103, ``q_quant``), the scores
    ``q K^T * sm_scale`` are masked causally (query i sees keys <= S - Sq + i)
    and the softmax and ``P V`` run in ``acc`` precision without the
    reference's intermediate bf16 roundings.  Returns ``[B, Sq, Hq, D]``.
    """
    dt = np.float64 if acc == "f64" else np.float32
    B, Hq, Sq, D = q.shape
    _, Hkv, S, _ = k_i8.shape
    n_rep = Hq // Hkv if n_rep is None else n_rep
    sm_scale = 1.0 / math.sqrt(D) if sm_scale is None else sm_scale
    k = cast(dequantize_int8(k_i8, np.asarray(k_sc, np.float32)), dtype).astype(dt)
    v = cast(dequantize_int8(v_i8, np.asarray(v_sc, np.float32)), dtype).astype(dt)
    qq = quant_dequant(q, (3,), dtype) if q_quant else np.asarray(q, np.float32)
    qg = qq.astype(dt).reshape(B, Hkv, n_rep, Sq, D)
    scores = np.matmul(qg, np.swapaxes(k, -1, -2)[:, :, None]) * dt(sm_scale)
    allowed = np.arange(S)[None, :] <= np.arange(Sq)[:, None] + (S - Sq)
    scores = np.where(allowed, scores, -np.inf)
    scores = scores - scores.max(axis=-1, keepdims=True)
    p = np.exp(scores)
    p = p / p.sum(axis=-1, keepdims=True)
    out = np.matmul(p, v[:, :, None]).reshape(B, Hq, Sq, D)
    return np.ascontiguousarray(out.transpose(0, 2, 1, 3))


def decode_dense(q, k, v, n_rep=None, sm_scale=None, acc="f32"):
    """Same attention on dense (bf16/fp16-valued) K/V: the twin kernel's check."""
    out = page_attention_reference(np.asarray(q, np.float32)[:, :, None, :],
                                   np.asarray(k, np.float32), np.asarray(v, np.float32),
                                   n_rep, sm_scale, acc)
    return out[:, :, 0, :]


def quant_dequant(x, reduce_dims, dtype="bf16"):
    """tests/qwen_kvcache_full.py:19-23: ``(round-clamp(x / scale) * scale).to(x.dtype)``."""
    q, scale = quantize_int8(x, reduce_dims)
    return cast(q.astype(np.float32) * scale, dtype)


def split_partials(q, k, v, bounds, n_rep, sm_scale):
    """Per-chunk flash-decoding partials over dense float K/V.

    q ``[B, Hq, D]``; ``bounds`` = list of (s0, s1) chunks.  Returns a list of
    (m ``[B, Hq]``, l ``[B, Hq]``, o ``[B, Hq, D]``) in float64, with scores in
    base 2 (``s * sm_scale * log2(e)``).
    """
    K = repeat_kv(np.asarray(k, np.float64), n_rep)
    V = repeat_kv(np.asarray(v, np.float64), n_rep)
    qq = np.asarray(q, np.float64)
    parts = []
    for s0, s1 in bounds:
        s = np.einsum("bhd,bhsd->bhs", qq, K[:, :, s0:s1]) * (sm_scale * LOG2E)
        m = s.max(axis=-1) if s1 > s0 else np.full(s.shape[:2], -np.inf)
        p = np.exp2(s - m[..., None]) if s1 > s0 else np.zeros_like(s)
        parts.append((m, p.sum(-1), np.einsum("bhs,bhsd->bhd", p, V[:, :, s0:s1])))
    return parts


def lse_combine(parts):
    """Combine (m, l, o) partials: M = max m_i, out = sum 2^(m_i-M) o_i / sum 2^(m_i-M) l_i."""
    M = np.max(np.stack([p[0] for p in parts]), axis=0)
    L = np.zeros_like(M)
    O = np.zeros_like(parts[0][2])
    for m, l, o in parts:
        w = np.where(np.isneginf(m), 0.0, np.exp2(m - M))
        L += w * l
        O += w[..., None] * o
    return O / L[..., None]
