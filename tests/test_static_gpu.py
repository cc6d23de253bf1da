"""Static (calibrated) K scales on the GPU: codes bit-exact with the oracle.

Oracle: ``oracle.quant.quant_k_static`` - the code step of ``quantize_int8``
(reference/page_attention_int8_pytorch.py:23-30) with the scale given, pinned to
torch on CPU by tests/test_static_scale_cpu.py.  The reference has no static
path (it is its roadmap item, README.md:140); every other rule of its cache
(V per token, fp16 stored scales) is unchanged.
"""
import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200 import kernels
from halftone_quantizedkvcache_b200.integration import QuantizedKVCache
from oracle import inputs as oin
from oracle import quant as oq

pytestmark = pytest.mark.gpu
TDT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def dev(x, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(x))
    return (t.to(TDT[dt]) if dt else t).cuda()


def calib_scale(rng, B, H, D, dt, shrink=0.7):
    """A scale calibrated on another sample, shrunk so that some values clamp."""
    c = oin.outlier_k(rng, B, H, 300, D, dt)
    return (np.abs(c).max(axis=(0, 2), keepdims=True).astype(np.float32) / np.float32(127)
            * np.float32(shrink)).astype(np.float32)


@pytest.mark.parametrize("shape,dt,sdt", [
    ((2, 8, 1000, 128), "bf16", "f32"),
    ((1, 4, 77, 64), "f16", "f32"),
    ((2, 2, 33, 256), "f32", "f32"),
    ((3, 8, 4096, 128), "bf16", "f16"),
    ((1, 1, 1, 128), "bf16", "f32"),
])
def test_static_codes_vs_oracle(shape, dt, sdt):
    rng = np.random.default_rng(sum(shape))
    B, H, S, D = shape
    x = oin.outlier_k(rng, B, H, S, D, dt)
    s = calib_scale(rng, 1, H, D, dt)
    if sdt == "f16":
        s = oq.to_f16(s).astype(np.float32)
    st = dev(s).to(TDT[sdt])
    q = kernels.quant_k_static(dev(x, dt), st)         # [1, H, 1, D]: broadcast over the batch
    ref = oq.quant_k_static(x, s)
    np.testing.assert_array_equal(q.cpu().numpy(), ref)
    q2 = kernels.quant_k_static(dev(x, dt), st[0, :, 0, :])   # [H, D]
    assert torch.equal(q, q2)


def test_static_per_sequence_scale_and_strided_input():
    rng = np.random.default_rng(3)
    B, S, H, D = 2, 300, 8, 128
    x_bshd = oin.outlier_k(rng, B, S, H, D)
    xt = dev(x_bshd, "bf16").transpose(1, 2)                  # [B, H, S, D] view
    s = np.concatenate([calib_scale(rng, 1, H, D, "bf16", 0.8), calib_scale(rng, 1, H, D, "bf16", 1.2)])
    q = kernels.quant_k_static(xt, dev(s))
    np.testing.assert_array_equal(q.cpu().numpy(), oq.quant_k_static(x_bshd.transpose(0, 2, 1, 3), s))


def test_static_ties_take_the_exact_path():
    s = np.full((1, 1, 1, 128), 0.25, np.float32)
    x = (np.arange(-200, 312, dtype=np.float32).reshape(1, 1, 4, 128) * np.float32(0.125))
    q = kernels.quant_k_static(dev(x, "f32"), dev(s))
    np.testing.assert_array_equal(q.cpu().numpy(), oq.quant_k_static(x, s))


def test_static_append_and_cache():
    rng = np.random.default_rng(9)
    B, H, D = 2, 8, 128
    s = calib_scale(rng, 1, H, D, "bf16", 0.9)
    cache = QuantizedKVCache(mode="fused", static_k_scale=dev(s))
    ref = oq.QuantizedKVCacheOracle()
    ks, vs = [], []
    for n in (100, 1, 3, 70, 1):
        k = oin.outlier_k(rng, B, H, n, D)
        v = oin.normal(rng, (B, H, n, D))
        cache.update(dev(k, "bf16"), dev(v, "bf16"), 0)
        ref.update(k, v, 0)          # for V: the reference rule is unchanged
        ks.append(k)
    kall = np.concatenate(ks, axis=2)
    np.testing.assert_array_equal(cache._k_i8[0].cpu().numpy(), oq.quant_k_static(kall, s))
    np.testing.assert_array_equal(cache._k_sc[0].cpu().numpy(),
                                  np.broadcast_to(oq.to_f16(s), (B, H, 1, D)))
    np.testing.assert_array_equal(cache._v_i8[0].cpu().numpy(), ref._v_i8[0])
    np.testing.assert_array_equal(cache._v_sc[0].cpu().numpy(), ref._v_sc[0])


def test_calibrate_k_scale():
    rng = np.random.default_rng(4)
    xs = [oin.outlier_k(rng, 2, 8, n, 128) for n in (50, 300)]
    s = kernels.calibrate_k_scale([dev(x, "bf16") for x in xs])
    amax = np.maximum(*[np.abs(x).max(axis=(0, 2), keepdims=True) for x in xs])
    np.testing.assert_array_equal(s.cpu().numpy(), (amax.astype(np.float64) / 127.0).astype(np.float32))


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_static_clamp_bounds_and_tiny_scales(dt):
    """Inputs well past the calibrated range (the 16-bit input clamp) and scales so
    small that 127 * s is below the fp16 normal range (the exact path)."""
    rng = np.random.default_rng(17)
    x = oin.normal(rng, (1, 4, 256, 128), dt) * np.float32(3.0)
    x = oq.cast(x, dt)
    s = np.abs(rng.standard_normal((1, 4, 1, 128))).astype(np.float32) * np.float32(0.01) + np.float32(1e-3)
    q = kernels.quant_k_static(dev(x, dt), dev(s))
    ref = oq.quant_k_static(x, s)
    np.testing.assert_array_equal(q.cpu().numpy(), ref)
    assert (np.abs(ref) == 127).mean() > 0.3
    tiny = np.full((1, 4, 1, 128), 1e-7, np.float32)
    xt = oq.cast(oin.normal(rng, (1, 4, 64, 128), dt) * np.float32(1e-5), dt)
    q2 = kernels.quant_k_static(dev(xt, dt), dev(tiny))
    np.testing.assert_array_equal(q2.cpu().numpy(), oq.quant_k_static(xt, tiny))
