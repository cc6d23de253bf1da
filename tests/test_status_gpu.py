"""Kernels whose blocks wait for one another, and the status words of the cache.

The K quantizer (pass B waits for pass A's per-slab counts) and the
sequence-sharded decode (the last block waits for the other ranks' words) are
cooperative launches: a grid that cannot be resident all at once is refused at
launch (cudaErrorCooperativeLaunchTooLarge) and writes nothing.  The grid is
made too large here by planning it for twice the GPU's SMs (hq_set_plan_sms) -
a launch refusal checked by the driver before anything runs, not a fault.

``QuantizedKVCache.check()`` surfaces the status words its kernels report into.
A failing device wait is not provoked on the GPU: the test writes
HQ_ERR_DEVICE_TIMEOUT into a status word the way the kernel would (a fake of the
failing call), then checks that ``check()`` and ``check_status=True`` raise.
"""
import ctypes

import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200 import _lib, kernels
from halftone_quantizedkvcache_b200.integration import QuantizedKVCache, quantized_attention_forward
from oracle import inputs as oin
from oracle import quant as oq

pytestmark = pytest.mark.gpu
TOO_LARGE = 720  # cudaErrorCooperativeLaunchTooLarge


class _Attn:
    num_key_value_groups, head_dim, training = 2, 128, False


@pytest.fixture
def oversized():
    """Grids planned for twice this GPU's SMs, restored afterwards."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    kernels.set_plan_sms(2 * sms)
    try:
        yield
    finally:
        kernels.set_plan_sms(0)


def test_quant_k_refused_when_the_grid_cannot_be_resident(oversized):
    rng = np.random.default_rng(1)
    x = oin.outlier_k(rng, 4, 8, 8192, 128)
    xt = torch.from_numpy(x).bfloat16().cuda()
    q = torch.full(xt.shape, 77, dtype=torch.int8, device="cuda")
    s = torch.full((4, 8, 1, 128), 5.0, dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.HalftoneError) as e:
        kernels.quant_k_perchannel(xt, out=q, scale_dtype=None, scale_f32_out=s)
    assert e.value.status == TOO_LARGE
    torch.cuda.synchronize()
    assert bool((q == 77).all()) and bool((s == 5.0).all())   # nothing written
    kernels.set_plan_sms(0)
    kernels.quant_k_perchannel(xt, out=q, scale_dtype=None, scale_f32_out=s)
    rq, rs = oq.quant_k_perchannel(xt.float().cpu().numpy())
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)


def test_peer_decode_refused_when_the_grid_cannot_be_resident(oversized):
    c = oin.decode_case(3, 1, 16, 8, 32768, 128)
    t = {k: torch.from_numpy(np.ascontiguousarray(c[k])).cuda()
         for k in ("q", "k_i8", "k_sc", "v_i8", "v_sc")}
    q = t["q"].to(torch.bfloat16)
    L = _lib.lib()
    ptr, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
    _lib.check(L.hq_peer_alloc(L.hq_peer_buffer_bytes(1, 1, 16, 8), ctypes.byref(ptr), handle),
               "hq_peer_alloc")
    try:
        peers = ((ctypes.c_void_p * 1)(ptr.value), 1, 0)
        out = torch.full_like(q, 3.0)
        with pytest.raises(_lib.HalftoneError) as e:
            kernels.int8_decode_attn(q, t["k_i8"], t["k_sc"], t["v_i8"], t["v_sc"], peers=peers,
                                     out=out)
        assert e.value.status == TOO_LARGE
        torch.cuda.synchronize()
        assert bool((out == 3.0).all())
        kernels.set_plan_sms(0)
        got = kernels.int8_decode_attn(q, t["k_i8"], t["k_sc"], t["v_i8"], t["v_sc"], peers=peers)
        ref = kernels.int8_decode_attn(q, t["k_i8"], t["k_sc"], t["v_i8"], t["v_sc"])
        assert torch.equal(got, ref)
    finally:
        L.hq_peer_free(ptr.value)


def test_cooperative_quant_k_replays_in_a_cuda_graph():
    rng = np.random.default_rng(2)
    xt = torch.from_numpy(oin.outlier_k(rng, 2, 8, 4096, 128)).bfloat16().cuda()
    q = torch.empty(xt.shape, dtype=torch.int8, device="cuda")
    s = torch.empty((2, 8, 1, 128), dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        kernels.quant_k_perchannel(xt, out=q, scale_dtype=None, scale_f32_out=s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            kernels.quant_k_perchannel(xt, out=q, scale_dtype=None, scale_f32_out=s)
        q.zero_()
        g.replay()
    torch.cuda.synchronize()
    rq, rs = oq.quant_k_perchannel(xt.float().cpu().numpy())
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)
    del g


def _decode_step(cache, rng, layer=0):
    kn = torch.from_numpy(oin.normal(rng, (1, 8, 1, 128))).bfloat16().cuda()
    k, v = cache.update(kn, kn, layer)
    q = torch.from_numpy(oin.normal(rng, (1, 16, 1, 128))).bfloat16().cuda()
    return quantized_attention_forward(_Attn(), q, k, v, None)[0]


def test_cache_check_surfaces_device_status():
    rng = np.random.default_rng(4)
    cache = QuantizedKVCache(mode="fused")
    k = torch.from_numpy(oin.outlier_k(rng, 1, 8, 300, 128)).bfloat16().cuda()
    cache.update(k, k, 0)
    _decode_step(cache, rng)
    cache.check()                                   # all clear
    assert cache._status.decode, "the decode workspace is recorded"
    ws = next(iter(cache._status.decode.values()))
    ws[:4].view(torch.int32).fill_(_lib.ERR_DEVICE_TIMEOUT)   # as a decode that gave up writes it
    with pytest.raises(RuntimeError, match="gave up"):
        cache.check()
    cache.reset_status()
    cache.check()
    cache._status.quant_word(k.device).fill_(_lib.ERR_DEVICE_TIMEOUT)  # a K quantizer that gave up
    with pytest.raises(RuntimeError):
        cache.check()
    cache.reset_status()
    cache.check()


def test_check_status_raises_on_the_next_call():
    rng = np.random.default_rng(5)
    cache = QuantizedKVCache(mode="fused", check_status=True)
    k = torch.from_numpy(oin.outlier_k(rng, 1, 8, 64, 128)).bfloat16().cuda()
    cache.update(k, k, 0)
    _decode_step(cache, rng)                        # checked, clear
    ws = next(iter(cache._status.decode.values()))
    ws[:4].view(torch.int32).fill_(_lib.ERR_DEVICE_TIMEOUT)
    with pytest.raises(RuntimeError):
        _decode_step(cache, rng)
    cache.reset_status()
    _decode_step(cache, rng)
