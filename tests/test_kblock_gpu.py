"""Block-wise per-channel K layout on the GPU: write, append and decode parity.

Oracle: ``oracle.blockwise`` (the reference quantizer, reference/page_attention_int8_pytorch.py:23-30,
per block of tokens; a single block is pinned to the reference's golden vectors).
Codes and scales are bit-exact; the decode output is held to max-abs 1e-3 and
relative 1e-3 against the float64 oracle in float32, plus bf16 rounding for bf16 output.
"""
import math

import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200 import kernels
from oracle import blockwise as ob
from oracle import inputs as oin
from oracle import quant as oq

pytestmark = pytest.mark.gpu
TDT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def dev(x, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(x))
    return (t.to(TDT[dt]) if dt else t).cuda()


def make(B, H, S, D, dt, seed=0):
    rng = np.random.default_rng(seed)
    k = oin.outlier_k(rng, B, H, S, D, dt)
    v = oin.normal(rng, (B, H, S, D), dt)
    return k, v


def check_cache(cache, k, v, S, block, v_scale_dt):
    codes, scales = ob.quant_k_blockwise(k[:, :, :S], block)
    nblk = scales.shape[2]
    np.testing.assert_array_equal(cache["k"][:, :, :S].cpu().numpy(), codes)
    np.testing.assert_array_equal(cache["k_scale"][:, :, :nblk].cpu().numpy(), scales)
    vc, vs = oq.quant_v_pertoken(v[:, :, :S])
    np.testing.assert_array_equal(cache["v"][:, :, :S].cpu().numpy(), vc)
    want = vs[..., 0] if v_scale_dt == torch.float32 else oq.to_f16(vs[..., 0])
    np.testing.assert_array_equal(cache["v_scale"][:, :, :S].cpu().numpy(), want)


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("block", [64, 128, 256])
def test_bulk_write_bit_exact(dt, D, block):
    B, H, S = 2, 3, 517
    k, v = make(B, H, S, D, dt)
    c = kernels.kblock_alloc(B, H, S + 40, D, block_tokens=block, dtype=TDT[dt],
                             v_scale_dtype=torch.float32)
    kernels.kblock_write(dev(k, dt), dev(v, dt), 0, c)
    check_cache(c, k, v, S, block, torch.float32)


def test_golden_single_block_through_the_kernel(golden):
    g = golden("quant_golden.npz")
    names = sorted({n.split("/")[0] for n in g.files if "/" in n})
    for name in names:
        dt = str(g[f"{name}/dtype"])
        x = oq.unpack(g[f"{name}/x"], dt)
        B, H, S, D = x.shape
        c = kernels.kblock_alloc(B, H, S, D, block_tokens=256, dtype=TDT[dt])
        kernels.kblock_write(dev(x, dt), dev(x, dt), 0, c)
        np.testing.assert_array_equal(c["k"].cpu().numpy(), g[f"{name}/k_codes"], err_msg=name)
        np.testing.assert_array_equal(c["k_scale"][:, :, :1].cpu().numpy(), g[f"{name}/k_scale"],
                                      err_msg=name)
        np.testing.assert_array_equal(c["v"].cpu().numpy(), g[f"{name}/v_codes"], err_msg=name)
        np.testing.assert_array_equal(c["v_scale"].cpu().numpy(), g[f"{name}/v_scale_f16"][..., 0],
                                      err_msg=name)


@pytest.mark.parametrize("block", [64, 128])
@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_token_appends_equal_bulk(block, dt):
    """Prefill then one token at a time: after every step the cache equals a bulk
    block-wise quantization of the tokens so far (re-coding the open block)."""
    B, H, D, P, S = 2, 2, 128, 70, 70 + 2 * block + 9
    k, v = make(B, H, S, D, dt, seed=4)
    # make later tokens grow the column maxima often
    ramp = np.linspace(1.0, 3.0, S, dtype=np.float32)[None, None, :, None]
    k = oq.cast(k * ramp, dt)
    c = kernels.kblock_alloc(B, H, S, D, block_tokens=block, dtype=TDT[dt])
    kd, vd = dev(k, dt), dev(v, dt)
    kernels.kblock_write(kd[:, :, :P], vd[:, :, :P], 0, c)
    for t in range(P, S):
        kernels.kblock_write(kd[:, :, t:t + 1], vd[:, :, t:t + 1], t, c)
        if t in (P, P + 1, block - 1, block, 2 * block + 3, S - 1):
            check_cache(c, k, v, t + 1, block, torch.float16)


def test_chunked_writes_cross_blocks():
    """Writes of ragged sizes, including one that starts inside a block and ends
    inside a later one (the tail written by a second launch), then appends."""
    B, H, D, block = 1, 4, 128, 64
    sizes = [37, 5, 150, 64, 1, 90, 1, 1, 33]
    S = sum(sizes)
    k, v = make(B, H, S, D, "bf16", seed=7)
    k = oq.cast(k * np.linspace(0.5, 2.0, S, dtype=np.float32)[None, None, :, None], "bf16")
    c = kernels.kblock_alloc(B, H, S, D, block_tokens=block)
    kd, vd = dev(k, "bf16"), dev(v, "bf16")
    pos = 0
    for n in sizes:
        kernels.kblock_write(kd[:, :, pos:pos + n], vd[:, :, pos:pos + n], pos, c)
        pos += n
        check_cache(c, k, v, pos, block, torch.float16)


def test_write_errors():
    c = kernels.kblock_alloc(1, 1, 8, 128, block_tokens=64)
    x = torch.zeros((1, 1, 9, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        kernels.kblock_write(x, x, 0, c)           # past the capacity (the C check: CPU tests)
    with pytest.raises(ValueError):
        kernels.kblock_alloc(1, 1, 8, 128, block_tokens=96)


def _decode_case(B, Hq, Hkv, S, D, block, q_dt, seed):
    k, v = make(B, Hkv, S, D, "bf16", seed)
    q = oin.normal(np.random.default_rng(seed + 1), (B, Hq, D), q_dt)
    return q, k, v


@pytest.mark.parametrize("B,Hq,Hkv,S,D,block", [
    (1, 16, 8, 1, 128, 128), (1, 16, 8, 5, 128, 64), (2, 16, 8, 129, 128, 128),
    (1, 8, 8, 1000, 128, 256), (3, 32, 8, 777, 128, 64), (1, 64, 8, 300, 64, 128),
    (2, 4, 2, 4099, 64, 64), (1, 16, 8, 32768, 128, 128)])
@pytest.mark.parametrize("q_dt,sc", [("f32", torch.float32), ("bf16", torch.float16)])
def test_decode_matches_oracle(B, Hq, Hkv, S, D, block, q_dt, sc):
    q, k, v = _decode_case(B, Hq, Hkv, S, D, block, q_dt, seed=S)
    c = kernels.kblock_alloc(B, Hkv, S + 17, D, block_tokens=block, v_scale_dtype=sc)
    kernels.kblock_write(dev(k, "bf16"), dev(v, "bf16"), 0, c)
    out = kernels.kblock_decode(dev(q, q_dt), c, S).float().cpu().numpy()
    vs = c["v_scale"][:, :, :S].float().cpu().numpy()
    codes, scales = ob.quant_k_blockwise(k, block)
    vc, _ = oq.quant_v_pertoken(v)
    want = ob.decode_blockwise(q, codes, scales, vc, vs, block)
    tol = 1e-3 + (2.0 ** -8 if q_dt == "bf16" else 0.0) * np.abs(want)
    err = np.abs(out - want)
    assert (err <= tol + 1e-3 * np.abs(want)).all(), f"max err {err.max():.3e}"


def test_decode_after_appends_and_dequant():
    B, Hq, Hkv, D, block, P, S = 1, 16, 8, 128, 64, 100, 180
    q, k, v = _decode_case(B, Hq, Hkv, S, D, block, "f32", seed=11)
    c = kernels.kblock_alloc(B, Hkv, S, D, block_tokens=block)
    kd, vd = dev(k, "bf16"), dev(v, "bf16")
    kernels.kblock_write(kd[:, :, :P], vd[:, :, :P], 0, c)
    for t in range(P, S):
        kernels.kblock_write(kd[:, :, t:t + 1], vd[:, :, t:t + 1], t, c)
        if t % 20 == 0 or t == S - 1:
            n = t + 1
            out = kernels.kblock_decode(dev(q, "f32"), c, n).cpu().numpy()
            codes, scales = ob.quant_k_blockwise(k[:, :, :n], block)
            vc, vs = oq.quant_v_pertoken(v[:, :, :n])
            want = ob.decode_blockwise(q, codes, scales, vc, oq.to_f16(vs[..., 0]), block)
            np.testing.assert_allclose(out, want, atol=1e-3, rtol=1e-3)
    deq = kernels.kblock_dequant(c, S).cpu().numpy()
    codes, scales = ob.quant_k_blockwise(k, block)
    np.testing.assert_array_equal(deq, ob.dequant_k_blockwise(codes, scales, block))


def test_decode_sm_scale_and_unsupported():
    B, Hq, Hkv, S, D = 1, 16, 8, 257, 128
    q, k, v = _decode_case(B, Hq, Hkv, S, D, 128, "f32", seed=2)
    c = kernels.kblock_alloc(B, Hkv, S, D)
    kernels.kblock_write(dev(k, "bf16"), dev(v, "bf16"), 0, c)
    out = kernels.kblock_decode(dev(q, "f32"), c, S, sm_scale=0.05).cpu().numpy()
    codes, scales = ob.quant_k_blockwise(k, 128)
    vc, vs = oq.quant_v_pertoken(v)
    want = ob.decode_blockwise(q, codes, scales, vc, oq.to_f16(vs[..., 0]), 128, sm_scale=0.05)
    np.testing.assert_allclose(out, want, atol=1e-3, rtol=1e-3)
    q3 = torch.zeros((1, 24, D), device="cuda")
    with pytest.raises((RuntimeError, ValueError)):
        kernels.kblock_decode(q3, c, S)   # 24 / 8 = 3 query heads per kv head


def test_cache_option_stores_the_blockwise_layout():
    """QuantizedKVCache(k_block_tokens=64): prefill, appends past the first capacity
    (the buffers grow), the stored layout equal to the oracle's bulk quantization."""
    from halftone_quantizedkvcache_b200.integration import QuantizedKVCache
    B, H, D, P, S = 1, 2, 128, 100, 600
    k, v = make(B, H, S, D, "bf16", seed=9)
    k = oq.cast(k * np.linspace(1.0, 2.5, S, dtype=np.float32)[None, None, :, None], "bf16")
    kd, vd = dev(k, "bf16"), dev(v, "bf16")
    cache = QuantizedKVCache(mode="fused", k_block_tokens=64)
    cache.update(kd[:, :, :P], vd[:, :, :P], 0)
    for t in range(P, S):
        kc, _ = cache.update(kd[:, :, t:t + 1], vd[:, :, t:t + 1], 0)
    assert cache.get_seq_length(0) == S and kc.shape[2] == S
    st = cache._kblock[0]
    check_cache(st.c, k, v, S, 64, torch.float16)
    with pytest.raises(ValueError):
        QuantizedKVCache(mode="dequant", k_block_tokens=64)


def test_whole_model_blockwise_is_closer_to_unquantized_than_reference_rule():
    """A 2-layer Qwen3-shaped model (random init, bf16): prefill 64, decode 48.
    The block-wise layout re-scales each block, so decoded K is not clipped to the
    prefill's column maxima the way the reference's retained first scale clips it
    (tests/qwen_kvcache_full.py:54): its logits stay closer to the unquantized model's."""
    from transformers import DynamicCache, Qwen3ForCausalLM

    from halftone_quantizedkvcache_b200.integration import QuantizedKVCache, installed
    from oracle.hf_reference import qwen3_config
    cfg = qwen3_config(num_layers=2)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(1)
    n0, nd = 64, 48
    ids = torch.randint(0, cfg.vocab_size, (1, n0 + nd), generator=g).cuda()

    @torch.no_grad()
    def run(cache):
        out = [model(ids[:, :n0], past_key_values=cache, use_cache=True).logits[:, -1]]
        for t in range(n0, n0 + nd):
            out.append(model(ids[:, t:t + 1], past_key_values=cache, use_cache=True).logits[:, -1])
        return torch.stack(out, 1).float()

    full = run(DynamicCache())
    with installed():
        blk = run(QuantizedKVCache(mode="fused", k_block_tokens=128))
        ref = run(QuantizedKVCache(mode="fused"))
    e_blk = (blk - full)[:, 1:].abs().mean().item()
    e_ref = (ref - full)[:, 1:].abs().mean().item()
    print(f"decode logit error vs unquantized: block-wise {e_blk:.4f}, reference rule {e_ref:.4f}")
    assert torch.isfinite(blk).all()
    assert e_blk < e_ref


def test_wrappers_check_shapes_against_the_cache():
    """The library cannot see buffer sizes: the wrappers reject calls whose counts
    do not match the cache before anything is launched."""
    c = kernels.kblock_alloc(1, 8, 256, 128)
    x = torch.zeros((2, 8, 4, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        kernels.kblock_write(x, x, 0, c)                       # two sequences, cache of one
    y = torch.zeros((1, 8, 4, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        kernels.kblock_write(y, y, 254, c)                     # past the capacity
    kernels.kblock_write(y, y, 0, c)
    q = torch.zeros((2, 16, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        kernels.kblock_decode(q, c, 4)                         # two sequences
    with pytest.raises(ValueError):
        kernels.kblock_decode(q[:1], c, 257)                   # past the capacity
    with pytest.raises(ValueError):
        kernels.kblock_dequant(c, 300)
    assert kernels.kblock_decode(q[:1], c, 4).shape == (1, 16, 128)


@pytest.mark.parametrize("block", [64, 128, 256])
def test_device_length_steps_equal_host_length_steps(block):
    """hq_kblock_write_at + hq_kblock_decode_len (length on the device) against the
    host-length calls, one token per step from a 300-token prefill: the cache is
    bit-exact with the oracle's bulk block-wise quantization after every step and the
    outputs are identical (same split plan, same kernel)."""
    B, Hq, Hkv, D, S0, n = 2, 16, 8, 128, 300, 70
    k, v = make(B, Hkv, S0 + n, D, "bf16", seed=block)
    cap = 512
    host = kernels.kblock_alloc(B, Hkv, cap, D, block_tokens=block, device="cuda")
    devc = kernels.kblock_alloc(B, Hkv, cap, D, block_tokens=block, device="cuda")
    kt, vt = dev(k, "bf16"), dev(v, "bf16")
    kernels.kblock_write(kt[:, :, :S0], vt[:, :, :S0], 0, host)
    kernels.kblock_write(kt[:, :, :S0], vt[:, :, :S0], 0, devc)
    lens = torch.tensor([S0, 0, 0, 0], dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(7)
    for i in range(n):
        L = S0 + i
        kernels.kblock_write(kt[:, :, L:L + 1], vt[:, :, L:L + 1], L, host)
        kernels.kblock_write(kt[:, :, L:L + 1], vt[:, :, L:L + 1], None, devc, lens=lens)
        q = dev(oin.normal(rng, (B, Hq, D)), "bf16")
        a = kernels.kblock_decode(q, host, L + 1)
        b = kernels.kblock_decode(q, devc, L + 1, seq_len=lens, s_plan=L + 1)
        assert torch.equal(a, b), i
    assert lens.tolist()[:3] == [S0 + n, 0, 0]
    for name in ("k", "k_scale", "v", "v_scale"):
        assert torch.equal(host[name], devc[name]), name
    check_cache(devc, k, v, S0 + n, block, torch.float16)


def test_device_length_step_replays_in_a_cuda_graph():
    """One decode step (one-token write at lens[0] + decode over lens[0] tokens) captured
    once and replayed for 100 tokens: the cache stays bit-exact with the oracle's bulk
    block-wise quantization, a full cache writes nothing and sets the status word, and
    every replayed output is within the decode tolerance of the float64 oracle."""
    B, Hq, Hkv, D, S0, n, block = 1, 16, 8, 128, 1000, 100, 128
    cap = S0 + n
    k, v = make(B, Hkv, cap + 1, D, "bf16", seed=3)
    c = kernels.kblock_alloc(B, Hkv, cap, D, block_tokens=block, device="cuda")
    kt, vt = dev(k, "bf16"), dev(v, "bf16")
    kernels.kblock_write(kt[:, :, :S0], vt[:, :, :S0], 0, c)
    lens = torch.tensor([S0, 0, 0, 0], dtype=torch.int32, device="cuda")
    knew = torch.empty((B, Hkv, 1, D), dtype=torch.bfloat16, device="cuda")
    vnew = torch.empty_like(knew)
    q = torch.empty((B, Hq, D), dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(q)
    qs = dev(oin.normal(np.random.default_rng(11), (n + 1, B, Hq, D)), "bf16")

    def step():
        kernels.kblock_write(knew, vnew, None, c, lens=lens)
        kernels.kblock_decode(q, c, cap, seq_len=lens, s_plan=S0, out=out)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        knew.copy_(kt[:, :, S0:S0 + 1])
        vnew.copy_(vt[:, :, S0:S0 + 1])
        q.copy_(qs[0])
        step()                                   # eager: workspaces exist
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step()
        for i in range(1, n):
            knew.copy_(kt[:, :, S0 + i:S0 + i + 1])
            vnew.copy_(vt[:, :, S0 + i:S0 + i + 1])
            q.copy_(qs[i])
            g.replay()
            if i % 33 == 0 or i == n - 1:
                torch.cuda.synchronize()
                L = S0 + i + 1
                codes, scales = ob.quant_k_blockwise(k[:, :, :L], block)
                vc, vs = oq.quant_v_pertoken(v[:, :, :L])
                ref = ob.decode_blockwise(qs[i].float().cpu().numpy(), codes, scales, vc,
                                          oq.to_f16(vs[..., 0]).astype(np.float32), block)
                np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=1e-2, rtol=2.0 ** -7)
        torch.cuda.synchronize()
        assert lens.tolist()[:3] == [cap, 0, 0]
        check_cache(c, k, v, cap, block, torch.float16)
        knew.copy_(kt[:, :, cap:cap + 1])        # one past the capacity: refused on the device
        g.replay()
        torch.cuda.synchronize()
        assert lens.tolist()[0] == cap and lens.tolist()[2] != 0
        del g
    check_cache(c, k, v, cap, block, torch.float16)


def test_whole_model_step_as_one_cuda_graph_with_blockwise_layout():
    """QuantizedKVCache(k_block_tokens=128, device_lengths=True) through HF transformers:
    the full decode step of a random-init 2-layer Qwen3-shaped model captured once as a
    CUDA graph and replayed per token (token id and position in static tensors), against
    the same cache run eagerly with host lengths: the prefill's codes and scales are
    bit-identical, the first logits identical, and the replayed logits stay within a
    small distance of the eager ones (the replayed split plan is the one planned at
    capture, so the float32 sums are grouped differently)."""
    from halftone_quantizedkvcache_b200.integration import QuantizedKVCache, installed
    from test_e2e_qwen3_gpu import build as build_model, tokens
    layers, n0, nd = 2, 200, 40
    model = build_model(layers)
    ids = tokens(model, 1, n0 + nd)
    with torch.no_grad(), installed():
        ref = QuantizedKVCache(mode="fused", k_block_tokens=128)
        want = [model(ids[:, :n0], past_key_values=ref, use_cache=True).logits[:, -1].float()]
        for t in range(n0, n0 + nd):
            want.append(model(ids[:, t:t + 1], past_key_values=ref, use_cache=True).logits[:, -1].float())
        cache = QuantizedKVCache(mode="fused", k_block_tokens=128, device_lengths=True,
                                 capacity=n0 + nd + 128)
        got = [model(ids[:, :n0], past_key_values=cache, use_cache=True).logits[:, -1].float()]
        tok = torch.empty((1, 1), dtype=torch.long, device="cuda")
        pos = torch.empty((1, 1), dtype=torch.long, device="cuda")
        masks = {"full_attention": None}

        def step():
            return model(input_ids=tok, position_ids=pos, attention_mask=masks,
                         past_key_values=cache, use_cache=True).logits[:, -1]

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            tok.copy_(ids[:, n0:n0 + 1])
            pos.fill_(n0)
            got.append(step().float())             # eager step: workspaces exist
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                out = step()
            for t in range(n0 + 1, n0 + nd):
                tok.copy_(ids[:, t:t + 1])
                pos.fill_(t)
                g.replay()
                got.append(out.float().clone())
            torch.cuda.synchronize()
        lens = cache.sync_lengths()
        del g
    assert all(v == n0 + nd for v in lens.values())
    for layer in range(layers):
        a, b = ref._kblock[layer].c, cache._kblock[layer].c
        assert torch.equal(a["k"][:, :, :n0], b["k"][:, :, :n0])
        assert torch.equal(a["v"][:, :, :n0], b["v"][:, :, :n0])
        assert torch.equal(a["v_scale"][:, :, :n0], b["v_scale"][:, :, :n0])
        assert torch.equal(a["k_scale"][:, :, :n0 // 128], b["k_scale"][:, :, :n0 // 128])
    err = (torch.stack(got, 1) - torch.stack(want, 1)).abs()
    assert torch.equal(got[0], want[0])
    print(f"block-wise graph-vs-eager logits: max {float(err.max()):.4f} mean {float(err.mean()):.5f}")
    assert float(err.mean()) < 5e-3 and float(err.max()) < 0.25
