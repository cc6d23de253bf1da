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
    assert L.hq_decode_int8_ex(*args, 2, None) == -1
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
             None]
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
