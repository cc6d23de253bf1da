"""Causal prefill attention over the int8 cache (``hq_prefill_int8``) on the GPU.

Oracle: ``oracle.attention.prefill_int8`` - the prefill branch of the
reference's patched attention (tests/qwen_kvcache_full.py:95-113) over the
dequantized cache its update() returns (:64-65), in float64.  The kernel reads
the same 16-bit K/V/q values and computes in float32, so before its final
rounding to the model dtype it agrees with the oracle to float32 round-off;
the check is |out - ref| <= 1e-3 + 2^-8 |ref| (the last term is the bf16
rounding of the stored output).
"""
import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200 import kernels
from halftone_quantizedkvcache_b200.integration import QuantizedKVCache
from halftone_quantizedkvcache_b200.integration.quantized_attention import (
    quantized_attention_forward)
from oracle import attention as oa
from oracle import inputs as oin
from oracle import quant as oq

pytestmark = pytest.mark.gpu
TDT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def dev(x, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(x))
    return (t.to(TDT[dt]) if dt else t).cuda()


def check(got, ref, what=""):
    got = got.float().cpu().numpy()
    bound = 1e-3 + 2.0 ** -8 * np.abs(ref)
    err = np.abs(got - ref)
    assert np.all(err <= bound), f"{what}: max err {err.max():.3e}, worst ratio {(err / bound).max():.2f}"


@pytest.mark.parametrize("B,Hq,Hkv,Sq,S,dt,sdt,qq", [
    (1, 16, 8, 512, 512, "bf16", "f16", True),     # config 1 prefill
    (2, 16, 8, 100, 137, "bf16", "f32", True),     # multi-token append onto a cache
    (1, 16, 8, 1, 700, "bf16", "f16", True),       # one query: the decode row
    (1, 8, 8, 65, 65, "f16", "f16", True),         # no GQA, ragged q and key tiles
    (1, 32, 8, 130, 300, "bf16", "f16", False),    # n_rep = 4, q used as given
    (2, 4, 2, 3, 3, "bf16", "f32", True),          # tiny
    (4, 16, 8, 640, 640, "bf16", "f16", True),     # grid beyond the resident slots: no cluster split
    (1, 6, 2, 200, 260, "f16", "f32", False),      # n_rep = 3: one head per block
])
def test_prefill_vs_oracle(B, Hq, Hkv, Sq, S, dt, sdt, qq):
    rng = np.random.default_rng(S * 7 + Sq)
    k = oin.outlier_k(rng, B, Hkv, S, 128)
    v = oin.normal(rng, (B, Hkv, S, 128))
    q = oin.normal(rng, (B, Hq, Sq, 128), dt)
    k8, ks = oq.quant_k_perchannel(k)
    v8, vs = oq.quant_v_pertoken(v)
    if sdt == "f16":
        ks, vs = oq.to_f16(ks), oq.to_f16(vs)
    out = kernels.int8_prefill_attn(dev(q, dt), dev(k8), dev(ks), dev(v8), dev(vs), Hq // Hkv,
                                    q_quant=qq)
    torch.cuda.synchronize()
    assert out.shape == (B, Sq, Hq, 128) and out.dtype == TDT[dt]
    ref = oa.prefill_int8(q, k8, ks.astype(np.float32), v8, vs.astype(np.float32), Hq // Hkv,
                          dtype=dt, q_quant=qq)
    check(out, ref, f"B={B} Hq={Hq} Sq={Sq} S={S}")


def test_prefill_status_word_and_repeat():
    """A status word stays 0 on a normal launch; repeated launches give identical rows
    (the cluster merge has a fixed order)."""
    rng = np.random.default_rng(11)
    B, Hq, Hkv, S = 1, 16, 8, 512
    k8, ks = oq.quant_k_perchannel(oin.outlier_k(rng, B, Hkv, S, 128))
    v8, vs = oq.quant_v_pertoken(oin.normal(rng, (B, Hkv, S, 128)))
    q = dev(oin.normal(rng, (B, Hq, S, 128)), "bf16")
    word = torch.zeros(1, dtype=torch.int32, device="cuda")
    args = (q, dev(k8), dev(oq.to_f16(ks)), dev(v8), dev(oq.to_f16(vs)), 2)
    a = kernels.int8_prefill_attn(*args, q_quant=True, status_into=word)
    b = kernels.int8_prefill_attn(*args, q_quant=True, status_into=word)
    torch.cuda.synchronize()
    assert int(word.item()) == 0
    assert torch.equal(a, b)
    with pytest.raises(ValueError):
        kernels.int8_prefill_attn(*args, q_quant=True, status_into=word.to(torch.int64))


def test_prefill_strided_q_and_output():
    """Qwen3 hands q as a [B, Hq, Sq, D] view of [B, Sq, Hq, D]; out may be a view too."""
    rng = np.random.default_rng(5)
    B, Hq, Hkv, S = 1, 16, 8, 200
    k8, ks = oq.quant_k_perchannel(oin.outlier_k(rng, B, Hkv, S, 128))
    v8, vs = oq.quant_v_pertoken(oin.normal(rng, (B, Hkv, S, 128)))
    q_bshd = oin.normal(rng, (B, S, Hq, 128))
    qt = dev(q_bshd, "bf16").transpose(1, 2)
    big = torch.zeros((B, S, Hq, 256), dtype=torch.bfloat16, device="cuda")
    out = big[..., 64:192]
    kernels.int8_prefill_attn(qt, dev(k8), dev(oq.to_f16(ks)), dev(v8), dev(oq.to_f16(vs)), 2,
                              q_quant=True, out=out)
    ref = oa.prefill_int8(q_bshd.transpose(0, 2, 1, 3), k8, oq.to_f16(ks).astype(np.float32), v8,
                          oq.to_f16(vs).astype(np.float32), 2)
    check(out, ref, "strided")
    assert bool((big[..., :64] == 0).all()) and bool((big[..., 192:] == 0).all())


class _Attn:
    num_key_value_groups = 2
    head_dim = 128
    training = False


def _causal_mask(Sq, S, dtype):
    allowed = torch.arange(S)[None, :] <= torch.arange(Sq)[:, None] + (S - Sq)
    m = torch.zeros((Sq, S), dtype=dtype).masked_fill(~allowed, torch.finfo(dtype).min)
    return m[None, None].cuda()


def test_prefill_through_the_cache():
    """fused_prefill=True: the patched attention takes the kernel for a causal
    mask and falls back to the reference math for any other mask."""
    rng = np.random.default_rng(11)
    B, Hq, Hkv, S = 1, 16, 8, 300
    k = oin.outlier_k(rng, B, Hkv, S, 128)
    v = oin.normal(rng, (B, Hkv, S, 128))
    q = oin.normal(rng, (B, Hq, S, 128))
    fused = QuantizedKVCache(mode="fused", fused_prefill=True)
    plain = QuantizedKVCache(mode="fused")
    kf, vf = fused.update(dev(k, "bf16"), dev(v, "bf16"), 0)
    kp, vp = plain.update(dev(k, "bf16"), dev(v, "bf16"), 0)
    mod, mask = _Attn(), _causal_mask(S, S, torch.bfloat16)
    of, _ = quantized_attention_forward(mod, dev(q, "bf16"), kf, vf, mask, scaling=128 ** -0.5)
    op, _ = quantized_attention_forward(mod, dev(q, "bf16"), kp, vp, mask, scaling=128 ** -0.5)
    ref = oa.prefill_int8(q, fused._k_i8[0].cpu().numpy(), fused._k_sc[0].float().cpu().numpy(),
                          fused._v_i8[0].cpu().numpy(), fused._v_sc[0].float().cpu().numpy(), 2)
    check(of, ref, "fused prefill")
    # the reference math rounds its scores to bf16 before the softmax: the kernel
    # is at least as close to the float64 attention as that path is
    err_ours = np.abs(of.float().cpu().numpy() - ref)
    err_refpath = np.abs(op.float().cpu().numpy() - ref)
    assert err_ours.max() <= err_refpath.max() and err_ours.mean() <= err_refpath.mean()
    # a padding-style mask (not causal): both caches take the reference math
    bad = mask.clone()
    bad[..., :5] = torch.finfo(torch.bfloat16).min
    of2, _ = quantized_attention_forward(mod, dev(q, "bf16"), kf, vf, bad, scaling=128 ** -0.5)
    op2, _ = quantized_attention_forward(mod, dev(q, "bf16"), kp, vp, bad, scaling=128 ** -0.5)
    assert torch.equal(of2, op2)


def test_prefill_logits_within_reference_noise():
    """2-layer Qwen3 shape: prefill logits with the fused prefill against the
    reference restatement, within twice its own bf16-vs-float32 drift."""
    from transformers import Qwen3ForCausalLM

    from halftone_quantizedkvcache_b200.integration import installed
    from oracle.hf_reference import (OracleQuantizedKVCache, oracle_attention_forward,
                                     patched_attention, qwen3_config)
    cfg = qwen3_config(num_layers=2)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (2, 96), generator=g).cuda()
    with torch.no_grad(), installed():
        cache = QuantizedKVCache(mode="fused", fused_prefill=True)
        a = model(ids, past_key_values=cache, use_cache=True).logits.float()

    def ref(fp32):
        def fwd(*x, **kw):
            return oracle_attention_forward(*x, fp32_math=fp32, **kw)
        with torch.no_grad(), patched_attention(fwd):
            return model(ids, past_key_values=OracleQuantizedKVCache(), use_cache=True).logits.float()

    b, b32 = ref(False), ref(True)
    err, floor = (a - b).abs(), (b32 - b).abs()
    print(f"prefill logits: ours-vs-oracle max {float(err.max()):.4f}, "
          f"oracle fp32-vs-bf16 max {float(floor.max()):.4f}")
    assert float(err.max()) <= 2.0 * float(floor.max()) + 1e-2
    assert float(err.mean()) <= 2.0 * float(floor.mean()) + 1e-3
