"""QuantizedKVCache on the GPU: the reference's update rule, bit for bit.

Golden: tests/golden/cache_golden.npz, written by the reference's own
QuantizedKVCache (tests/qwen_kvcache_full.py:27-89).  Longer sequences are
checked against the oracle restatement ``oracle.quant.QuantizedKVCacheOracle``.
"""
import hashlib

import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200.integration import QuantizedKVCache
from oracle import inputs as oin
from oracle import quant as oq

pytestmark = pytest.mark.gpu


def bf16(x):
    return torch.from_numpy(np.ascontiguousarray(x)).bfloat16().cuda()


def sha_bf16(t):
    return hashlib.sha256(oq.pack(t.float().cpu().numpy(), "bf16").tobytes()).hexdigest()


def test_golden_update_sequence(golden):
    g = golden("cache_golden.npz")
    cache = QuantizedKVCache(mode="dequant")
    for i in range(int(g["nsteps"])):
        k = bf16(oq.unpack(g[f"step{i}/k"], "bf16"))
        v = bf16(oq.unpack(g[f"step{i}/v"], "bf16"))
        for layer in (0, 3):
            ko, vo = cache.update(k, v, layer)
        assert ko.dtype == torch.bfloat16
        assert sha_bf16(ko) == str(g[f"step{i}/k_out_sha"]), f"step {i} dequantized K"
        assert sha_bf16(vo) == str(g[f"step{i}/v_out_sha"]), f"step {i} dequantized V"
    for layer in (0, 3):
        np.testing.assert_array_equal(cache._k_i8[layer].cpu().numpy(), g[f"layer{layer}/k_i8"])
        np.testing.assert_array_equal(cache._v_i8[layer].cpu().numpy(), g[f"layer{layer}/v_i8"])
        np.testing.assert_array_equal(cache._k_sc[layer].cpu().numpy(), g[f"layer{layer}/k_sc"])
        np.testing.assert_array_equal(cache._v_sc[layer].cpu().numpy(), g[f"layer{layer}/v_sc"])
    assert cache.storage_bytes() == int(g["storage_bytes"])
    assert cache.fp16_equiv_bytes() == int(g["fp16_equiv_bytes"])
    assert cache.get_seq_length(0) == int(g["seq_length"])
    assert len(cache) == int(g["len"])


@pytest.mark.parametrize("prefill,appends", [
    (200, [1] * 400),            # grows past the first capacity (456) one token at a time
    (31, [3, 64, 65, 100, 1]),   # fused append (<= 64) and the bulk-kernel path (> 64)
    (1, [1, 1]),
])
def test_against_oracle_cache(prefill, appends):
    rng = np.random.default_rng(prefill)
    B, H, D = 2, 8, 128
    ours = QuantizedKVCache(mode="fused")
    ref = oq.QuantizedKVCacheOracle()
    for n in [prefill] + appends:
        k = oin.outlier_k(rng, B, H, n, D)
        v = oin.normal(rng, (B, H, n, D))
        kt, vt = ours.update(bf16(k), bf16(v), 5)
        ref.update(k, v, 5)
        assert kt.dtype == torch.int8 and hasattr(kt, "_hq_store")
    np.testing.assert_array_equal(ours._k_i8[5].cpu().numpy(), ref._k_i8[5])
    np.testing.assert_array_equal(ours._v_i8[5].cpu().numpy(), ref._v_i8[5])
    np.testing.assert_array_equal(ours._k_sc[5].cpu().numpy(), ref._k_sc[5])
    np.testing.assert_array_equal(ours._v_sc[5].cpu().numpy(), ref._v_sc[5])
    assert ours.get_seq_length(5) == ref.get_seq_length(5)
    assert ours.storage_bytes() == ref.storage_bytes()


def test_hf_strided_inputs():
    """Qwen3 passes [B, H, S, D] views of [B, S, H, D] tensors."""
    rng = np.random.default_rng(9)
    k = oin.outlier_k(rng, 1, 40, 8, 128)   # stored [B, S, H, D]
    v = oin.normal(rng, (1, 40, 8, 128))
    ours = QuantizedKVCache(mode="fused")
    ours.update(bf16(k).transpose(1, 2), bf16(v).transpose(1, 2), 0)
    k2 = oin.outlier_k(rng, 1, 1, 8, 128)
    v2 = oin.normal(rng, (1, 1, 8, 128))
    ours.update(bf16(k2).transpose(1, 2), bf16(v2).transpose(1, 2), 0)
    ref = oq.QuantizedKVCacheOracle()
    ref.update(k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3), 0)
    ref.update(k2.transpose(0, 2, 1, 3), v2.transpose(0, 2, 1, 3), 0)
    for name in ("_k_i8", "_v_i8", "_k_sc", "_v_sc"):
        np.testing.assert_array_equal(getattr(ours, name)[0].cpu().numpy(), getattr(ref, name)[0])


def test_decode_with_full_width_padding_mask():
    """A decode mask with one column per cached token (padding: some columns at
    the dtype's minimum) is applied as the reference adds it
    (tests/qwen_kvcache_full.py:108-109): the step takes the reference's math
    over the dequantized cache, so it equals the oracle restatement exactly; a
    one-column mask (what HF builds for this cache) keeps the int8 kernel."""
    from halftone_quantizedkvcache_b200.integration import quantized_attention_forward
    from oracle.hf_reference import OracleQuantizedKVCache, oracle_attention_forward

    class Attn:
        num_key_value_groups, head_dim, training = 2, 128, False

    torch.manual_seed(3)
    B, Hq, Hkv, S, D = 2, 16, 8, 77, 128
    k = (torch.randn(B, Hkv, S, D) * 2).bfloat16().cuda()
    v = torch.randn(B, Hkv, S, D).bfloat16().cuda()
    kn = torch.randn(B, Hkv, 1, D).bfloat16().cuda()
    vn = torch.randn(B, Hkv, 1, D).bfloat16().cuda()
    q = torch.randn(B, Hq, 1, D).bfloat16().cuda()
    ours, ref = QuantizedKVCache(mode="fused"), OracleQuantizedKVCache()
    ours.update(k, v, 0)
    ref.update(k, v, 0)
    ko, vo = ours.update(kn, vn, 0)
    kr, vr = ref.update(kn, vn, 0)
    mask = torch.zeros(B, 1, 1, S + 1, dtype=torch.bfloat16, device="cuda")
    mask[0, :, :, :5] = torch.finfo(torch.bfloat16).min     # left padding of sequence 0
    mask[1, :, :, 40:44] = torch.finfo(torch.bfloat16).min
    a, _ = quantized_attention_forward(Attn(), q, ko, vo, mask, scaling=D ** -0.5)
    b, _ = oracle_attention_forward(Attn(), q, kr, vr, mask, scaling=D ** -0.5)
    assert torch.equal(a, b)
    # one column: the kernel path, within the decode tolerance of the unmasked oracle
    a1, _ = quantized_attention_forward(Attn(), q, ko, vo, mask[..., :1] * 0, scaling=D ** -0.5)
    b1, _ = oracle_attention_forward(Attn(), q, kr, vr, None, scaling=D ** -0.5)
    assert float((a1.float() - b1.float()).abs().max()) < 5e-2
