"""Pin the CPU oracle to the reference's own outputs (fixtures in tests/golden/).

The fixtures were produced by ``tests/golden/make_golden.py``, which runs the
reference's torch functions (reference/page_attention_int8_pytorch.py:23-34,
reference/page_attention_reference.py:31-54, tests/qwen_kvcache_full.py:27-113).
Codes and scales must match bit for bit; attention to float32 round-off.
"""
import hashlib

import numpy as np
import pytest

from oracle import attention as oa
from oracle import inputs as oin
from oracle import quant as oq


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _cases(npz):
    return sorted({k.split("/")[0] for k in npz.files if "/" in k})


def test_quant_edge_cases_bit_exact(golden):
    g = golden("quant_golden.npz")
    names = _cases(g)
    assert len(names) >= 9
    for name in names:
        dt = str(g[f"{name}/dtype"])
        x = oq.unpack(g[f"{name}/x"], dt)
        for tag, fn in (("k", oq.quant_k_perchannel), ("v", oq.quant_v_pertoken)):
            codes, scale = fn(x)
            np.testing.assert_array_equal(codes, g[f"{name}/{tag}_codes"], err_msg=f"{name} {tag}")
            np.testing.assert_array_equal(scale, g[f"{name}/{tag}_scale"], err_msg=f"{name} {tag}")
            np.testing.assert_array_equal(oq.to_f16(scale), g[f"{name}/{tag}_scale_f16"],
                                          err_msg=f"{name} {tag} f16")


def test_ties_round_half_even(golden):
    g = golden("quant_golden.npz")
    codes = g["ties/v_codes"][0, 0, 0, :127].astype(np.int32)
    ks = np.arange(-126, 127, 2)
    # k + 0.5 with k even rounds down to k (half to even), never away from zero
    np.testing.assert_array_equal(codes, ks)


def test_config0_full_size(golden):
    g = golden("config0_golden.npz")
    q, k, v = oin.config0(int(g["seed"]))
    k_i8, k_sc = oq.quantize_int8(k[0], (1,))
    v_i8, v_sc = oq.quantize_int8(v[0], (2,))
    assert _sha(k_i8) == str(g["k_codes_sha"])
    assert _sha(v_i8) == str(g["v_codes_sha"])
    np.testing.assert_array_equal(k_sc, g["k_scale"])
    np.testing.assert_array_equal(v_sc, g["v_scale"])
    out = oa.decode_int8(q, k_i8[None], k_sc[None], v_i8[None], v_sc[None])
    np.testing.assert_allclose(out[0], g["attn_out"], rtol=1e-4, atol=1e-5)


def test_decode_cases(golden):
    g = golden("decode_golden.npz")
    for name in _cases(g):
        dt = str(g[f"{name}/dtype"])
        q = oq.unpack(g[f"{name}/q"], dt)
        out = oa.decode_int8(q, g[f"{name}/k_i8"], g[f"{name}/k_sc"], g[f"{name}/v_i8"],
                             g[f"{name}/v_sc"])
        np.testing.assert_allclose(out, g[f"{name}/out"], rtol=1e-4, atol=1e-5, err_msg=name)


def test_cache_update_sequence(golden):
    g = golden("cache_golden.npz")
    cache = oq.QuantizedKVCacheOracle()
    for i in range(int(g["nsteps"])):
        k = oq.unpack(g[f"step{i}/k"], "bf16")
        v = oq.unpack(g[f"step{i}/v"], "bf16")
        for layer in (0, 3):
            ko, vo = cache.update(k, v, layer)
        assert _sha(oq.pack(ko, "bf16")) == str(g[f"step{i}/k_out_sha"]), i
        assert _sha(oq.pack(vo, "bf16")) == str(g[f"step{i}/v_out_sha"]), i
    for layer in (0, 3):
        for key in ("k_i8", "v_i8", "k_sc", "v_sc"):
            np.testing.assert_array_equal(getattr(cache, "_" + key)[layer], g[f"layer{layer}/{key}"])
    assert cache.storage_bytes() == int(g["storage_bytes"])
    assert cache.fp16_equiv_bytes() == int(g["fp16_equiv_bytes"])
    assert cache.get_seq_length(0) == int(g["seq_length"])
    assert len(cache) == int(g["len"])


def test_appended_k_codes_saturate(golden):
    """The reference keeps the prefill K scale but codes a 1-token append with
    its own per-channel scale, so every nonzero appended K code is +-127."""
    g = golden("cache_golden.npz")
    appended = g["layer0/k_i8"][:, :, 40:46, :]
    nz = appended[appended != 0]
    assert np.all(np.abs(nz.astype(np.int32)) == 127)


def test_split_combine_matches_unsplit():
    c = oin.decode_case(3, 2, 16, 8, 777, 128)
    k = oq.dequantize_int8(c["k_i8"], c["k_sc"])
    v = oq.dequantize_int8(c["v_i8"], c["v_sc"])
    sm = 1.0 / np.sqrt(128)
    bounds = [(0, 100), (100, 101), (101, 101), (101, 512), (512, 777)]
    got = oa.lse_combine(oa.split_partials(c["q"], k, v, bounds, 2, sm))
    ref = oa.decode_dense(c["q"], k, v, 2, sm, acc="f64")
    np.testing.assert_allclose(got, ref, rtol=1e-10, atol=1e-12)


def test_hf_restatement_matches_reference_logits(golden):
    torch = pytest.importorskip("torch")
    from transformers import Qwen3ForCausalLM

    from oracle.hf_reference import (OracleQuantizedKVCache, oracle_attention_forward,
                                     patched_attention, qwen3_config)
    g = golden("hf_logits.npz")
    cfg = qwen3_config(num_layers=2, vocab=1000, hidden=256, heads=4, kv_heads=2,
                       head_dim=128, intermediate=512)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
    ids = torch.from_numpy(g["ids"])
    n0 = int(g["prefill"])
    logits = []
    with patched_attention(oracle_attention_forward), torch.no_grad():
        cache = OracleQuantizedKVCache()
        o = model(ids[:, :n0], past_key_values=cache, use_cache=True)
        logits.append(o.logits[0, -1].float().numpy())
        for t in range(n0, ids.shape[1]):
            o = model(ids[:, t:t + 1], past_key_values=cache, use_cache=True)
            logits.append(o.logits[0, -1].float().numpy())
    np.testing.assert_array_equal(np.stack(logits), g["logits"])


def test_f32_comparator_is_the_pinned_restatement_in_float32():
    """``oracle_attention_f32`` (the whole-model comparator at the int8 kernel's
    precision) is the pinned restatement evaluated in float32: on float32
    inputs the two are the same operations, bit for bit (on a bf16 model it
    differs only in keeping the scores, softmax and products in float32)."""
    torch = pytest.importorskip("torch")
    from oracle.hf_reference import oracle_attention_f32, oracle_attention_forward

    class Attn:
        num_key_value_groups, head_dim, training = 2, 128, False

    g = torch.Generator().manual_seed(5)
    q = torch.randn((2, 8, 3, 128), generator=g)
    k = torch.randn((2, 4, 40, 128), generator=g) * 3
    v = torch.randn((2, 4, 40, 128), generator=g)
    mask = torch.zeros((2, 1, 3, 40))
    mask[0, :, :, :4] = -1e30
    a, _ = oracle_attention_f32(Attn(), q, k, v, mask)
    b, _ = oracle_attention_forward(Attn(), q, k, v, mask)
    assert torch.equal(a, b)
    a, _ = oracle_attention_f32(Attn(), q.bfloat16(), k, v, None)
    assert a.dtype == torch.bfloat16


def test_torch_cpu_decode_path_equals_numpy_oracle():
    """The timed CPU baseline (the reference's torch ops, oracle/torch_cpu.py) computes
    the numpy oracle's int8 decode, to float32 round-off."""
    torch = pytest.importorskip("torch")
    from oracle import torch_cpu
    c = oin.decode_case(3, 1, 16, 8, 700, 128)
    ref = oa.decode_int8(c["q"], c["k_i8"], c["k_sc"], c["v_i8"], c["v_sc"], 2, acc="f64")
    t = {k: torch.from_numpy(np.ascontiguousarray(c[k][0])) for k in
         ("k_i8", "k_sc", "v_i8", "v_sc")}
    q = torch.from_numpy(np.ascontiguousarray(c["q"][0]))[:, None, :].float()
    got = torch_cpu.decode_layer(q, t["k_i8"], t["k_sc"], t["v_i8"], t["v_sc"])[:, 0].numpy()
    np.testing.assert_allclose(got, ref[0], rtol=1e-5, atol=1e-5)
