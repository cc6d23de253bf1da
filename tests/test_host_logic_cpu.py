"""Host-side logic of the later entry points, on CPU (no GPU call is made):
argument checks that return before any launch, the causal-mask test that
routes a prefill to the fused kernel, and the static-scale calibration."""
import ctypes

import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200 import _lib, kernels
from halftone_quantizedkvcache_b200.integration import QuantizedKVCache
from halftone_quantizedkvcache_b200.integration.quantized_attention import _is_causal


def test_new_entry_points_reject_bad_arguments():
    L = _lib.lib()
    st3 = _lib.strides((0, 0, 1), 3)
    st4 = _lib.strides((0, 0, 0, 1), 4)
    kv = _lib.strides((0, 0, 128), 3)
    # hq_decode_int8_ex: unknown flag bits
    args = [16, 1, st3, 16, 16, kv, 16, 16, 0, st3, st3, 1, 16, 8, 64, 128, 0.1, 0, 16, st3, None,
            256, 1 << 20]
    assert L.hq_decode_int8_ex(*args, 4, None) == -1
    # hq_decode_int8_len: no length pointer
    largs = [16, 1, st3, 16, 16, kv, 16, 16, 0, st3, st3, 1, 16, 8, 64, None, 64, 128, 0.1, 0, 16,
             st3, 256, 1 << 20, None]
    assert L.hq_decode_int8_len(*largs) == -1
    # hq_append_kv_at: more than 64 new tokens, or no length buffer
    aargs = [16, 16, 1, st4, st4, 1, 8, 65, 128, 16, st4, 16, st4, None, 16, st3, 300, 16, None]
    assert L.hq_append_kv_at(*aargs) == -1
    aargs[7], aargs[17] = 1, None
    assert L.hq_append_kv_at(*aargs) == -1
    # hq_prefill_int8: null q; head_dim other than 128; f32 q; S < Sq
    pargs = [16, 1, st4, 16, 16, kv, 16, 16, 0, st3, st3, 1, 16, 8, 64, 64, 128, 0.1, 1, 16, st4,
             None, None]
    pargs[0] = None
    assert L.hq_prefill_int8(*pargs) == -1
    pargs[0], pargs[16] = 16, 64
    assert L.hq_prefill_int8(*pargs) == -2
    pargs[16], pargs[1] = 128, 0
    assert L.hq_prefill_int8(*pargs) == -2
    pargs[1], pargs[15] = 1, 32
    assert L.hq_prefill_int8(*pargs) == -1
    # hq_quant_k_static / hq_append_kv_static: null scale, unsupported scale dtype
    assert L.hq_quant_k_static(16, 1, st4, 1, 8, 4, 128, None, 0, st3, 16, st4, None) == -1
    assert L.hq_quant_k_static(16, 1, st4, 1, 8, 4, 128, 16, 3, st3, 16, st4, None) == -2
    assert L.hq_append_kv_static(16, 16, 1, st4, st4, 1, 8, 1, 128, None, 0, st3, 16, st4, 16,
                                 st4, None, 16, st3, None) == -1


def _mask(Sq, S, drop_first=0):
    allowed = torch.arange(S)[None, :] <= torch.arange(Sq)[:, None] + (S - Sq)
    if drop_first:
        allowed[:, :drop_first] = False
    m = torch.zeros((Sq, S), dtype=torch.bfloat16).masked_fill(~allowed, torch.finfo(torch.bfloat16).min)
    return m[None, None]


def test_causal_mask_detection():
    assert _is_causal(_mask(7, 7), 7, 7)
    assert _is_causal(_mask(3, 10), 3, 10)                 # append of 3 onto 7 cached tokens
    assert _is_causal(torch.cat([_mask(3, 10), torch.zeros(1, 1, 3, 4, dtype=torch.bfloat16)], -1),
                      3, 10)                              # wider mask, sliced to S as the reference does
    assert not _is_causal(_mask(7, 7, drop_first=2), 7, 7)  # padding
    assert not _is_causal(torch.zeros(1, 1, 7, 7, dtype=torch.bfloat16), 7, 7)  # full attention
    assert _is_causal(None, 1, 9) and not _is_causal(None, 4, 9)
    soft = _mask(5, 5).float()
    soft[..., 0, 1] = -3.0                                 # a finite bias is not a causal mask
    assert not _is_causal(soft, 5, 5)


def test_calibrate_k_scale_on_host_tensors():
    rng = np.random.default_rng(0)
    xs = [rng.standard_normal((2, 4, n, 64)).astype(np.float32) for n in (5, 17)]
    s = kernels.calibrate_k_scale([torch.from_numpy(x) for x in xs])
    amax = np.maximum(*[np.abs(x).max(axis=(0, 2), keepdims=True) for x in xs])
    np.testing.assert_array_equal(s.numpy(), (amax.astype(np.float64) / 127.0).astype(np.float32))
    with pytest.raises(ValueError):
        kernels.calibrate_k_scale([])


def test_cache_option_combinations():
    with pytest.raises(ValueError):
        QuantizedKVCache(mode="dequant", device_lengths=True)
    with pytest.raises(ValueError):
        QuantizedKVCache(mode="auto", fused_prefill=True)
    with pytest.raises(ValueError):
        QuantizedKVCache(mode="fused", device_lengths=True, static_k_scale=torch.ones(8, 128))


def test_blockwise_entry_points_reject_bad_arguments():
    """hq_kblock_*: argument checks that return before any launch."""
    L = _lib.lib()
    st3 = _lib.strides((0, 0, 128), 3)
    st4 = _lib.strides((0, 0, 128, 1), 4)

    def write(**kw):
        a = dict(k=16, v=16, dt=1, ks=st4, vs=st4, B=1, H=8, pos=0, n=4, D=128, bt=128, kc=16,
                 kqs=st4, ksc=16, kscs=st3, kt=16, kts=st4, vc=16, vqs=st4, v32=None, v16=16,
                 vss=st3, cap=256)
        a.update(kw)
        return L.hq_kblock_write(*a.values(), None)
    assert write(k=None) == -1                 # no K input
    assert write(pos=254) == -1                # past the capacity
    assert write(bt=96) == -2                  # block size not compiled in
    assert write(D=96) == -2
    assert write(dt=3) == -2                   # int8 input
    assert write(v32=16) == -1                 # both V scale dtypes
    assert write(B=70000) == -2                # grid limit
    assert write(B=0) == 0                     # nothing to do

    def decode(**kw):
        a = dict(q=16, qdt=1, qs=st3, kc=16, kqs=st3, ksc=16, kscs=st3, vc=16, vqs=st3, vsc=16,
                 sdt=2, vss=st3, B=1, Hq=16, Hkv=8, S=64, D=128, bt=128, sm=0.1, out=16, os=st3,
                 ws=None, wsb=0)
        a.update(kw)
        return L.hq_kblock_decode(*a.values(), None)
    assert decode(Hq=24) == -2                 # 3 query heads per kv head
    assert decode(sdt=3) == -2                 # int8 V scales
    assert decode(S=0) == -1
    assert decode(B=70000) == -2
    assert decode(B=0) == 0
    assert L.hq_kblock_decode_workspace_bytes(1, 24, 8, 64, 128) == 0
    # device-length variants: no length buffer; the decode serves head_dim 128 and up to
    # 4 q heads per kv head only
    wa = [16, 16, 1, st4, st4, 1, 8, 128, 128, 16, st4, 16, st3, 16, st4, 16, st4, None, 16, st3,
          256, None, None]
    assert L.hq_kblock_write_at(*wa) == -1
    unit = _lib.strides((0, 0, 1), 3)
    da = dict(q=16, qdt=1, qs=unit, kc=16, kqs=st3, ksc=16, kscs=st3, vc=16, vqs=st3, vsc=16,
              sdt=2, vss=st3, B=1, Hq=16, Hkv=8, cap=256, lens=None, plan=64, D=128, bt=128,
              sm=0.1, out=16, os=unit, ws=256, wsb=1 << 20)
    assert L.hq_kblock_decode_len(*da.values(), None) == -1
    da["lens"] = 16
    assert L.hq_kblock_decode_len(*dict(da, D=64).values(), None) == -2
    assert L.hq_kblock_decode_len(*dict(da, Hq=64).values(), None) == -2
    assert L.hq_kblock_dequant(16, st3, 16, st3, 1, 8, 64, 128, 96, 16, 1, st4, None) == -1
    assert L.hq_kblock_dequant(16, st3, 16, st3, 1, 8, 0, 128, 128, 16, 1, st4, None) == 0


def test_blockwise_cache_option_combinations():
    with pytest.raises(ValueError):
        QuantizedKVCache(mode="fused", k_block_tokens=96)
    with pytest.raises(ValueError):
        QuantizedKVCache(mode="auto", k_block_tokens=128)
    with pytest.raises(ValueError):   # the appended token's re-coding is a launch of its own
        QuantizedKVCache(mode="fused", k_block_tokens=128, device_lengths=True, fused_append=True)
    QuantizedKVCache(mode="fused", k_block_tokens=128, device_lengths=True)
    c = QuantizedKVCache(mode="fused", k_block_tokens=64)
    assert c.get_seq_length(0) == 0 and len(c) == 0 and c.storage_bytes() == 0


def test_sharded_write_entry_points_reject_bad_arguments():
    """hq_column_absmax / hq_k_scale_from_amax: argument checks that return before any launch."""
    L = _lib.lib()
    st4 = _lib.strides((0, 0, 128, 1), 4)
    assert L.hq_column_absmax(None, 1, st4, 1, 8, 64, 128, 16, None) == -1   # no input
    assert L.hq_column_absmax(16, 1, st4, 1, 8, 64, 128, None, None) == -1   # no output
    assert L.hq_column_absmax(16, 3, st4, 1, 8, 64, 128, 16, None) == -2     # int8 input
    assert L.hq_column_absmax(16, 1, st4, 1, 8, 64, 96, 16, None) == -2      # head_dim
    assert L.hq_column_absmax(16, 1, st4, 1, 8, -1, 128, 16, None) == -1     # negative S
    assert L.hq_column_absmax(16, 1, st4, 0, 8, 64, 128, 16, None) == 0      # nothing to do
    assert L.hq_k_scale_from_amax(None, 8, 16, None, None) == -1
    assert L.hq_k_scale_from_amax(16, 8, None, None, None) == -1             # no output
    assert L.hq_k_scale_from_amax(16, 0, 16, None, None) == 0
