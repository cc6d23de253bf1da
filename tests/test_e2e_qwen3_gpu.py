"""Whole-model check: random-init Qwen3 through HF transformers on the GPU.

Ours:   ``QuantizedKVCache`` + ``quantized_attention_forward`` (CUDA kernels).
Oracle: the torch restatement of the reference drop-in
        (``oracle.hf_reference``, tests/qwen_kvcache_full.py:19-113), which
        tests/test_oracle_golden.py pins to the reference's own logits.
Both see the same weights and the same teacher-forced token stream, so a
single argmax flip cannot make the two decodes diverge.  Tolerance: max-abs
1e-2 on bf16 logits (north star).
"""
import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200.integration import QuantizedKVCache, installed
from oracle.hf_reference import (OracleQuantizedKVCache, oracle_attention_forward,
                                 patched_attention, qwen3_config)

pytestmark = pytest.mark.gpu
TOL = 1e-2


def build(num_layers, vocab=151936, seed=0):
    from transformers import Qwen3ForCausalLM
    cfg = qwen3_config(num_layers=num_layers, vocab=vocab)
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    with torch.device("cuda"):
        model = Qwen3ForCausalLM(cfg)
    return model.to(torch.bfloat16).eval()


@torch.no_grad()
def run(model, ids, n_prefill, cache):
    logits = [model(ids[:, :n_prefill], past_key_values=cache, use_cache=True).logits[:, -1]]
    for t in range(n_prefill, ids.shape[1]):
        logits.append(model(ids[:, t:t + 1], past_key_values=cache, use_cache=True).logits[:, -1])
    return torch.stack(logits, 1).float()


def compare(num_layers, n_prefill, n_decode, batch=1):
    model = build(num_layers)
    gen = torch.Generator().manual_seed(1)
    ids = torch.randint(0, model.config.vocab_size, (batch, n_prefill + n_decode), generator=gen)
    ids = ids.cuda()
    with installed():
        cache = QuantizedKVCache()
        ours = run(model, ids, n_prefill, cache)
        assert cache.get_seq_length(0) == n_prefill + n_decode
    with patched_attention(oracle_attention_forward):
        ref = run(model, ids, n_prefill, OracleQuantizedKVCache())
    err = (ours - ref).abs()
    return err, ref


def test_small_model_logits():
    err, ref = compare(num_layers=2, n_prefill=64, n_decode=16, batch=2)
    assert float(err[:, 0].max()) < TOL   # prefill: same math, dequantized cache
    assert float(err.max()) < TOL, float(err.max())


def test_qwen3_06b_shape_prefill512_decode256():
    """Config 1: 28 layers, prefill 512 uniform token ids, 256 decode steps."""
    err, ref = compare(num_layers=28, n_prefill=512, n_decode=256)
    print(f"max|dlogit| {float(err.max()):.3e}  mean {float(err.mean()):.3e}  "
          f"|logit| max {float(ref.abs().max()):.3f}")
    assert float(err.max()) < TOL
