"""Device-resident cache lengths: the decode step (append + int8 decode) as a
replayable CUDA graph.

The reference grows its cache with torch.cat and keeps the length on the host
(tests/qwen_kvcache_full.py:36,51-62), so its step cannot be replayed.  Here a
``QuantizedKVCache(device_lengths=True)`` appends at a device-side length and
the decode kernel reads it.  Checked:
  * eager steps: codes, scales and outputs identical to the host-length cache
    (same split plan, so the same arithmetic);
  * a step captured once and replayed for every later token: codes and scales
    bit-exact with the host-length cache, outputs within the bf16 output
    tolerance of the eager result and within 1e-3 (float32 partials) of the oracle;
  * a full cache: the append writes nothing and reports it, the length stays.
"""
import math

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

B, HQ, HKV, D = 2, 16, 8, 128


class _Attn:
    num_key_value_groups = HQ // HKV
    head_dim = D
    training = False


def bf16(x):
    return torch.from_numpy(np.ascontiguousarray(x)).bfloat16().cuda()


def _step_inputs(rng):
    k = oin.outlier_k(rng, B, HKV, 1, D)
    v = oin.normal(rng, (B, HKV, 1, D))
    q = oin.normal(rng, (B, HQ, 1, D))
    return k, v, q


def _prefill(cache, rng, S0, layer=0):
    k = oin.outlier_k(rng, B, HKV, S0, D)
    v = oin.normal(rng, (B, HKV, S0, D))
    cache.update(bf16(k), bf16(v), layer)
    return k, v


@pytest.mark.parametrize("S0", [1000, 4096])
def test_eager_steps_match_host_length_cache(S0):
    rng = np.random.default_rng(S0)
    dev = QuantizedKVCache(mode="fused", capacity=S0 + 64, device_lengths=True)
    host = QuantizedKVCache(mode="fused")
    k, v = _prefill(dev, np.random.default_rng(1), S0)
    host.update(bf16(k), bf16(v), 0)
    mod = _Attn()
    for _ in range(6):
        kn, vn, q = _step_inputs(rng)
        kd, vd = dev.update(bf16(kn), bf16(vn), 0)
        kh, vh = host.update(bf16(kn), bf16(vn), 0)
        qt = bf16(q)
        od, _ = quantized_attention_forward(mod, qt, kd, vd, None, scaling=1 / math.sqrt(D))
        oh, _ = quantized_attention_forward(mod, qt, kh, vh, None, scaling=1 / math.sqrt(D))
        assert torch.equal(od, oh)
    lens = dev.sync_lengths()
    assert lens[0] == host.get_seq_length(0) == S0 + 6
    for name in ("_k_i8", "_v_i8", "_k_sc", "_v_sc"):
        assert torch.equal(getattr(dev, name)[0], getattr(host, name)[0]), name


def test_graph_replay_matches_eager_and_oracle():
    S0, steps, layers = 3000, 40, 3
    rng = np.random.default_rng(7)
    dev = QuantizedKVCache(mode="fused", capacity=S0 + steps + 64, device_lengths=True)
    host = QuantizedKVCache(mode="fused")
    oracle = oq.QuantizedKVCacheOracle()
    for layer in range(layers):
        k, v = _prefill(dev, np.random.default_rng(10 + layer), S0, layer)
        host.update(bf16(k), bf16(v), layer)
        oracle.update(k, v, layer)
    mod = _Attn()
    scaling = 1 / math.sqrt(D)
    kb = torch.empty((layers, B, HKV, 1, D), dtype=torch.bfloat16, device="cuda")
    vb = torch.empty_like(kb)
    qb = torch.empty((layers, B, HQ, 1, D), dtype=torch.bfloat16, device="cuda")
    ob = torch.empty((layers, B, 1, HQ, D), dtype=torch.bfloat16, device="cuda")

    def step():
        for layer in range(layers):
            kt, vt = dev.update(kb[layer], vb[layer], layer)
            o, _ = quantized_attention_forward(mod, qb[layer], kt, vt, None, scaling=scaling)
            ob[layer].copy_(o)

    def feed():
        ins = [_step_inputs(rng) for _ in range(layers)]
        for layer, (kn, vn, q) in enumerate(ins):
            kb[layer].copy_(bf16(kn))
            vb[layer].copy_(bf16(vn))
            qb[layer].copy_(bf16(q))
        return ins

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ins = feed()
        step()                       # eager warm-up step: workspaces exist before capture
        torch.cuda.synchronize()
        for layer, (kn, vn, q) in enumerate(ins):
            host.update(bf16(kn), bf16(vn), layer)
            oracle.update(kn, vn, layer)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step()                   # recorded only: the device lengths do not move
        worst = 0.0
        for i in range(steps):
            ins = feed()
            g.replay()
            torch.cuda.synchronize()
            for layer, (kn, vn, q) in enumerate(ins):
                kh, vh = host.update(bf16(kn), bf16(vn), layer)
                oh, _ = quantized_attention_forward(mod, bf16(q), kh, vh, None, scaling=scaling)
                torch.testing.assert_close(ob[layer], oh, atol=1e-2, rtol=1e-2)
                oracle.update(kn, vn, layer)
                if i % 13 == 0:  # the float32 result against the oracle
                    part = torch.empty((B, HQ, D + 2), dtype=torch.float32, device="cuda")
                    kk, vv, ks, vs = (torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (
                        oracle._k_i8[layer], oracle._v_i8[layer], oracle._k_sc[layer],
                        oracle._v_sc[layer]))
                    kernels.int8_decode_attn(bf16(q[:, :, 0]), kk, ks, vv, vs, HQ // HKV,
                                             sm_scale=scaling, q_quant=True, partial_out=part)
                    q_in = oa.quant_dequant(q[:, :, 0], (2,), "bf16")  # the per-token q fake quant
                    ref = oa.decode_int8(q_in, oracle._k_i8[layer], oracle._k_sc[layer],
                                         oracle._v_i8[layer], oracle._v_sc[layer], HQ // HKV,
                                         scaling, acc="f64")
                    p = part.cpu().numpy()
                    worst = max(worst, float(np.max(np.abs(p[..., 2:] / p[..., 1:2] - ref))))
                    out_err = float(np.max(np.abs(ob[layer].float().cpu().numpy()[:, 0] - ref)))
                    assert out_err < 2e-2, out_err
        assert worst < 1e-3, worst
    lens = dev.sync_lengths()
    for layer in range(layers):
        assert lens[layer] == S0 + steps + 1
        for name in ("_k_i8", "_v_i8", "_k_sc", "_v_sc"):
            assert torch.equal(getattr(dev, name)[layer], getattr(host, name)[layer]), name
    del g


def test_full_cache_writes_nothing():
    cap = 300
    k8 = torch.full((1, HKV, cap, D), 7, dtype=torch.int8, device="cuda")
    v8 = torch.full_like(k8, 7)
    vs = torch.full((1, HKV, cap, 1), 3.0, dtype=torch.float16, device="cuda")
    lens = torch.tensor([cap - 1, 0, 0, 0], dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(3)
    kn = bf16(oin.outlier_k(rng, 1, HKV, 2, D))
    vn = bf16(oin.normal(rng, (1, HKV, 2, D)))
    kernels.append_kv_at(kn, vn, k8, v8, vs, lens)   # 2 rows at cap - 1: does not fit
    assert lens.tolist() == [cap - 1, 0, -1, 0]
    assert bool((k8 == 7).all()) and bool((v8 == 7).all()) and bool((vs == 3.0).all())
    lens.copy_(torch.tensor([cap - 2, 0, 0, 0], dtype=torch.int32))
    kernels.append_kv_at(kn, vn, k8, v8, vs, lens)   # exactly fits
    assert lens.tolist() == [cap, 0, 0, 0]
    ref_k, _ = oq.quant_k_perchannel(kn.float().cpu().numpy())
    np.testing.assert_array_equal(k8[:, :, cap - 2:].cpu().numpy(), ref_k)
    assert bool((k8[:, :, : cap - 2] == 7).all())


def _attn_step(cache, layer, kn, vn, q):
    kt, vt = cache.update(bf16(kn), bf16(vn), layer)
    o, _ = quantized_attention_forward(_Attn(), bf16(q), kt, vt, None, scaling=1 / math.sqrt(D))
    return o


def test_fused_append_matches_two_launches():
    """fused_append=True: the one-token append runs inside the decode launch; the
    cache is bit-exact with the two-launch path and the outputs agree to float
    round-off (bf16 outputs); a token left pending by an update without an
    attention is written by the next cache access."""
    S0 = 2000
    fused = QuantizedKVCache(mode="fused", capacity=S0 + 64, device_lengths=True, fused_append=True)
    plain = QuantizedKVCache(mode="fused", capacity=S0 + 64, device_lengths=True)
    k, v = _prefill(fused, np.random.default_rng(2), S0)
    plain.update(bf16(k), bf16(v), 0)
    rng = np.random.default_rng(12)
    for i in range(8):
        kn, vn, q = _step_inputs(rng)
        if i == 4:  # an update with no attention after it, then the next step
            fused.update(bf16(kn), bf16(vn), 0)
            plain.update(bf16(kn), bf16(vn), 0)
            kn, vn, q = _step_inputs(rng)
        of = _attn_step(fused, 0, kn, vn, q)
        op = _attn_step(plain, 0, kn, vn, q)
        torch.testing.assert_close(of, op, atol=1e-2, rtol=1e-2)
    lf, lp = fused.sync_lengths(), plain.sync_lengths()
    assert lf == lp and lf[0] == S0 + 9
    for name in ("_k_i8", "_v_i8", "_k_sc", "_v_sc"):
        assert torch.equal(getattr(fused, name)[0], getattr(plain, name)[0]), name


def test_fused_append_graph_replay():
    S0, steps, layers = 1500, 24, 2
    rng = np.random.default_rng(21)
    fused = QuantizedKVCache(mode="fused", capacity=S0 + steps + 64, device_lengths=True,
                             fused_append=True)
    host = QuantizedKVCache(mode="fused")
    oracle = oq.QuantizedKVCacheOracle()
    for layer in range(layers):
        k, v = _prefill(fused, np.random.default_rng(30 + layer), S0, layer)
        host.update(bf16(k), bf16(v), layer)
        oracle.update(k, v, layer)
    kb = torch.empty((layers, B, HKV, 1, D), dtype=torch.bfloat16, device="cuda")
    vb = torch.empty_like(kb)
    qb = torch.empty((layers, B, HQ, 1, D), dtype=torch.bfloat16, device="cuda")
    ob = torch.empty((layers, B, 1, HQ, D), dtype=torch.bfloat16, device="cuda")
    scaling = 1 / math.sqrt(D)

    def step():
        for layer in range(layers):
            kt, vt = fused.update(kb[layer], vb[layer], layer)
            o, _ = quantized_attention_forward(_Attn(), qb[layer], kt, vt, None, scaling=scaling)
            ob[layer].copy_(o)

    def feed():
        ins = [_step_inputs(rng) for _ in range(layers)]
        for layer, (kn, vn, q) in enumerate(ins):
            kb[layer].copy_(bf16(kn))
            vb[layer].copy_(bf16(vn))
            qb[layer].copy_(bf16(q))
        return ins

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ins = feed()
        step()
        torch.cuda.synchronize()
        for layer, (kn, vn, q) in enumerate(ins):
            host.update(bf16(kn), bf16(vn), layer)
            oracle.update(kn, vn, layer)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step()
        for i in range(steps):
            ins = feed()
            g.replay()
            torch.cuda.synchronize()
            for layer, (kn, vn, q) in enumerate(ins):
                oh = _attn_step(host, layer, kn, vn, q)
                torch.testing.assert_close(ob[layer], oh, atol=1e-2, rtol=1e-2)
                oracle.update(kn, vn, layer)
                if i % 11 == 0:
                    q_in = oa.quant_dequant(q[:, :, 0], (2,), "bf16")
                    ref = oa.decode_int8(q_in, oracle._k_i8[layer], oracle._k_sc[layer],
                                         oracle._v_i8[layer], oracle._v_sc[layer], HQ // HKV,
                                         scaling, acc="f64")
                    err = float(np.max(np.abs(ob[layer].float().cpu().numpy()[:, 0] - ref)))
                    assert err < 2e-2, err
        assert kernels.read_status("decode") == 0
    lens = fused.sync_lengths()
    for layer in range(layers):
        assert lens[layer] == S0 + steps + 1
        for name in ("_k_i8", "_v_i8", "_k_sc", "_v_sc"):
            assert torch.equal(getattr(fused, name)[layer], getattr(host, name)[layer]), name
    del g


def test_fused_append_full_cache():
    """At capacity the fused launch writes nothing, keeps the length, attends over
    the cached rows and reports the full cache in the workspace status word."""
    cap = 300
    rng = np.random.default_rng(8)
    k8, ks = oq.quant_k_perchannel(oin.outlier_k(rng, 1, HKV, cap, D))
    v8, vs = oq.quant_v_pertoken(oin.normal(rng, (1, HKV, cap, D)))
    kt, vt = torch.from_numpy(k8).cuda(), torch.from_numpy(v8).cuda()
    kst, vst = torch.from_numpy(oq.to_f16(ks)).cuda(), torch.from_numpy(oq.to_f16(vs)).cuda()
    q = bf16(oin.normal(rng, (1, HQ, D)))
    kn = bf16(oin.outlier_k(rng, 1, HKV, 1, D))
    vn = bf16(oin.normal(rng, (1, HKV, 1, D)))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):      # its own workspace: the status word set here stays local
        lens = torch.tensor([cap - 1, 0, 0, 0], dtype=torch.int32, device="cuda")
        before = kt.clone()
        o1 = kernels.int8_decode_attn(q, kt, kst, vt, vst, HQ // HKV, seq_len=lens,
                                      s_plan=cap - 1, append=(kn, vn))
        assert int(lens[0]) == cap                      # the last row was free: written
        assert torch.equal(kt[:, :, : cap - 1], before[:, :, : cap - 1])
        o2 = kernels.int8_decode_attn(q, kt, kst, vt, vst, HQ // HKV, seq_len=lens,
                                      s_plan=cap, append=(kn, vn))
        assert int(lens[0]) == cap                      # full: nothing written, length kept
        assert kernels.read_status("decode") == -1
        ref = kernels.int8_decode_attn(q, kt, kst, vt, vst, HQ // HKV, seq_len=lens, s_plan=cap)
        torch.testing.assert_close(o2, ref, atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(o1, ref, atol=1e-2, rtol=1e-2)  # same rows both times
        torch.cuda.synchronize()
