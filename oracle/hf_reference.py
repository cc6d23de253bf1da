"""Oracle (test infrastructure): torch restatement of the reference's HF drop-in.

The whole-model check drives a random-init Qwen3 through HF transformers twice:
once with the product's ``QuantizedKVCache`` + patched attention (CUDA
kernels), once with the restatement below, and compares logits.

* ``OracleQuantizedKVCache`` restates ``QuantizedKVCache``
  (tests/qwen_kvcache_full.py:27-89): quantize on every ``update`` (K per
  channel over the new tokens, V per token), append codes and fp16 V scales,
  keep the first call's fp16 K scale, return the whole cache dequantized to
  the input dtype.
* ``oracle_attention_forward`` restates ``quantized_attention_forward``
  (tests/qwen_kvcache_full.py:92-113): per-token fake quantization of q
  (``Q_DIMS = (3,)``), GQA by ``repeat_interleave``, ``q K^T * scaling`` plus
  the mask, float32 softmax cast back to the model dtype, ``@ V``, output
  ``[B, Sq, Hq, D]``.

It is device-agnostic torch code, so the checker can run it on CPU (small
cases) or on the GPU (the full Qwen3-0.6B shape) as the reference itself ran.
The restatement is pinned to the real reference by
``tests/golden/hf_logits.npz`` (``tests/test_oracle_golden.py``).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from transformers.cache_utils import DynamicCache

Q_DIMS = (3,)


def sym_int8(x: torch.Tensor, dims):
    """Symmetric int8 of ``x`` reduced over ``dims``: float32 (codes, scale).

    ``amax / 127`` is an IEEE true division on every device.  On the CPU this
    is what the reference computes (bit-identical, pinned by the golden
    logits); on a GPU torch would turn a division by the Python scalar 127.0
    into a multiply by its reciprocal, so the divisor is a tensor here.
    """
    xf = x.float()
    amax = xf.abs().amax(dim=dims, keepdim=True).clamp(min=1e-8)
    scale = amax / torch.full((), 127.0, dtype=torch.float32, device=x.device)
    return torch.clamp(torch.round(xf / scale), -127, 127), scale


def fake_quant(x: torch.Tensor, dims) -> torch.Tensor:
    """tests/qwen_kvcache_full.py:19-23."""
    codes, scale = sym_int8(x, dims)
    return (codes * scale).to(x.dtype)


class OracleQuantizedKVCache(DynamicCache):
    """Restatement of tests/qwen_kvcache_full.py:27-89."""

    def __init__(self):
        super().__init__()
        self._k_i8, self._v_i8, self._k_sc, self._v_sc, self._lens = {}, {}, {}, {}, {}

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        k_codes, k_scale = sym_int8(key_states, 2)
        v_codes, v_scale = sym_int8(value_states, 3)
        k_codes, v_codes = k_codes.to(torch.int8), v_codes.to(torch.int8)
        if layer_idx not in self._k_i8:
            self._k_i8[layer_idx], self._v_i8[layer_idx] = k_codes, v_codes
            self._k_sc[layer_idx] = k_scale.to(torch.float16)
            self._v_sc[layer_idx] = v_scale.to(torch.float16)
        else:
            self._k_i8[layer_idx] = torch.cat([self._k_i8[layer_idx], k_codes], 2)
            self._v_i8[layer_idx] = torch.cat([self._v_i8[layer_idx], v_codes], 2)
            self._v_sc[layer_idx] = torch.cat(
                [self._v_sc[layer_idx], v_scale.to(torch.float16)], 2)
        self._lens[layer_idx] = self._k_i8[layer_idx].shape[2]
        k = self._k_i8[layer_idx].float() * self._k_sc[layer_idx].float()
        v = self._v_i8[layer_idx].float() * self._v_sc[layer_idx].float()
        return k.to(key_states.dtype), v.to(value_states.dtype)

    def get_seq_length(self, layer_idx=0, cache_position=None):
        return self._lens.get(layer_idx, 0)

    def __len__(self):
        return len(self._k_i8)


def oracle_attention_forward(module, query, key, value, attention_mask, scaling=None,
                             dropout=0.0, fp32_math=False, **kwargs):
    """Restatement of tests/qwen_kvcache_full.py:95-113.

    ``fp32_math=True`` evaluates the same attention in float32 (then casts
    back): the reference's sensitivity to its own bf16 arithmetic, used as
    the noise floor of whole-model comparisons.
    """
    if fp32_math:
        out, _ = oracle_attention_forward(
            module, query.float(), key.float(), value.float(),
            None if attention_mask is None else attention_mask.float(), scaling, dropout)
        return out.to(query.dtype), None
    if scaling is None:
        scaling = module.head_dim ** -0.5
    n_rep = module.num_key_value_groups
    q = fake_quant(query, Q_DIMS)
    if n_rep != 1:
        key = key.repeat_interleave(n_rep, dim=1)
        value = value.repeat_interleave(n_rep, dim=1)
    scores = torch.matmul(q, key.transpose(2, 3)) * scaling
    if attention_mask is not None:
        scores = scores + attention_mask[:, :, :, : key.shape[-2]]
    probs = F.softmax(scores, dim=-1, dtype=torch.float32).to(q.dtype)
    probs = F.dropout(probs, p=dropout, training=module.training)
    return torch.matmul(probs, value).transpose(1, 2).contiguous(), None


def oracle_attention_f32(module, query, key, value, attention_mask, scaling=None, dropout=0.0,
                         math_dtype=torch.float32, **kwargs):
    """The reference's attention (tests/qwen_kvcache_full.py:95-113) evaluated in
    float32 (or ``math_dtype``): q fake-quantized per token in the model dtype
    exactly as the reference does (:103), then - with ``key`` / ``value`` the
    float32 dequantized codes (``code * scale``, not rounded to the model
    dtype) - ``q K^T * scaling`` plus the mask, softmax, ``@ V``, all in
    ``math_dtype``, and the output cast to the model dtype.  In float32 this is
    the arithmetic of the int8 decode kernel (exact code products, float32
    softmax); in float64 it is the most exact evaluation of the reference's
    math, the yardstick both are measured against."""
    if scaling is None:
        scaling = module.head_dim ** -0.5
    n_rep = module.num_key_value_groups
    q = fake_quant(query, Q_DIMS).to(math_dtype)
    k, v = key.to(math_dtype), value.to(math_dtype)
    if n_rep != 1:
        k = k.repeat_interleave(n_rep, dim=1)
        v = v.repeat_interleave(n_rep, dim=1)
    scores = torch.matmul(q, k.transpose(2, 3)) * scaling
    if attention_mask is not None:
        scores = scores + attention_mask[:, :, :, : k.shape[-2]].to(math_dtype)
    probs = F.softmax(scores, dim=-1, dtype=math_dtype)
    return torch.matmul(probs, v).transpose(1, 2).contiguous().to(query.dtype), None


def oracle_attention_f64(*args, **kwargs):
    """``oracle_attention_f32`` with every product and the softmax in float64."""
    return oracle_attention_f32(*args, math_dtype=torch.float64, **kwargs)


def qwen3_config(num_layers=28, vocab=151936, hidden=1024, heads=16, kv_heads=8,
                 head_dim=128, intermediate=3072):
    """The Qwen3-0.6B architecture (random init; no weights are loaded)."""
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=intermediate,
                       num_hidden_layers=num_layers, num_attention_heads=heads,
                       num_key_value_heads=kv_heads, head_dim=head_dim, rope_theta=1e6,
                       max_position_embeddings=40960, rms_norm_eps=1e-6, tie_word_embeddings=True,
                       attention_bias=False, use_sliding_window=False)


class patched_attention:
    """Context manager: install ``fn`` as Qwen3's ``eager_attention_forward``
    (the reference assigns the module global, tests/qwen_kvcache_full.py:161,186)."""

    def __init__(self, fn):
        self.fn = fn

    def __enter__(self):
        import transformers.models.qwen3.modeling_qwen3 as m
        self._mod, self._orig = m, m.eager_attention_forward
        m.eager_attention_forward = self.fn
        return self

    def __exit__(self, *exc):
        self._mod.eager_attention_forward = self._orig
        return False
