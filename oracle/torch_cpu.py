"""Oracle (test infrastructure): the reference's CPU PyTorch decode path, in torch.

The timed CPU baseline of ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) runs the reference's own sequence of torch
operations on the host cores, restated here line by line:

* ``dequantize_int8``            reference/page_attention_int8_pytorch.py:33-34
* ``repeat_kv``                  reference/page_attention_reference.py:23-28
* ``page_attention_reference``   reference/page_attention_reference.py:31-54
  (``bmm(q, K^T) * 1/sqrt(D)``, softmax in float32 cast back to q's dtype, ``bmm``)

``decode_layer`` is one decode step of one layer over an int8 cache (K per
channel, V per token): dequantize both, then the attention above - the
reference's config-0 chain (quantize_int8 -> dequantize_int8 ->
page_attention_reference) from the dequantization on.  The quantize-on-write
side of the CPU baseline is ``oracle.hf_reference.OracleQuantizedKVCache``
(tests/qwen_kvcache_full.py:38-66), already torch.  Nothing in the product
imports this module.
"""
from __future__ import annotations

import torch


def dequantize_int8(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """reference/page_attention_int8_pytorch.py:33-34."""
    return q.float() * scale


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """reference/page_attention_reference.py:23-28: [H_kv, S, D] -> [H_kv * n_rep, S, D]."""
    return x if n_rep == 1 else x.repeat_interleave(n_rep, dim=0)


@torch.no_grad()
def page_attention_reference(q, k_cache, v_cache, n_rep=None):
    """reference/page_attention_reference.py:31-54: q [H_q, Sq, D], K/V [H_kv, S, D]."""
    H_q, _, D = q.shape
    if n_rep is None:
        n_rep = H_q // k_cache.shape[0]
    K = repeat_kv(k_cache, n_rep)
    V = repeat_kv(v_cache, n_rep)
    scores = torch.bmm(q, K.transpose(1, 2)) * (1.0 / (D ** 0.5))
    attn = torch.softmax(scores.float(), dim=-1).to(q.dtype)
    return torch.bmm(attn, V)


@torch.no_grad()
def decode_layer(q, k_i8, k_sc, v_i8, v_sc):
    """One layer's decode over one sequence's int8 cache, the reference's CPU ops:
    q [H_q, 1, D] float32; k_i8 / v_i8 [H_kv, S, D] int8; k_sc [H_kv, 1, D] and
    v_sc [H_kv, S, 1] float32 -> [H_q, 1, D]."""
    return page_attention_reference(q, dequantize_int8(k_i8, k_sc), dequantize_int8(v_i8, v_sc))
