"""Exhaustive check of the quantizer arithmetic the CUDA kernels use.

Reference rule (float32 IEEE, reference/page_attention_int8_pytorch.py:23-30):
    scale = RN(amax / 127);  code = rint_half_even(RN(x / scale))
Kernel rule (halftone_quantizedkvcache_b200/csrc/hq_common.cuh, ``Quantizer``):
    r = RN(1 / scale);  k = rint_half_even(x * r)  (exact product, one rounding:
    fma(x, r, 1.5 * 2^23));  d = RN(x * r - k);  if |d| > 0.5 - 2^-15 the
    element is recomputed as rint(RN(x / scale)).

This models the kernel in float64 (every product below is exact in float64)
and checks, for every bf16 and every fp16 magnitude pair (x, amax) with
|x| <= amax, that the kernel rule equals the reference rule.  Exponents do not
matter: scaling x and amax by 2^e scales scale and r exactly (no subnormal
float32 occurs for bf16/fp16 data once amax >= 1e-8), so one binade of amax
covers all of them; the clamped case amax < 1e-8 is enumerated separately.
"""
import numpy as np

THR = np.float32(0.5 - 2.0 ** -15)


def _binade(mbits, e):
    return (1.0 + np.arange(2 ** mbits) / 2.0 ** mbits) * 2.0 ** e


def _check(amaxs, xs_of):
    flagged = total = 0
    for a in amaxs:
        a32 = np.maximum(np.float32(a), np.float32(1e-8))
        s = np.float32(a32 / np.float32(127.0))
        r = np.float32(np.float32(1.0) / s)
        xs = xs_of(a)
        xs = np.concatenate([xs, -xs]).astype(np.float32)
        ref = np.clip(np.rint(xs / s), -127, 127)
        p = xs.astype(np.float64) * np.float64(r)
        k = np.rint(p)
        d = (p - k).astype(np.float32)
        slow = np.abs(d) > THR
        fast = np.where(slow, ref, k)
        np.testing.assert_array_equal(fast, ref)
        assert np.all(np.abs(k[~slow]) <= 127)
        flagged += int(slow.sum())
        total += xs.size
    return flagged / total


def test_bf16_all_pairs():
    def xs_of(a):
        v = np.concatenate([_binade(7, e) for e in range(-16, 1)] + [np.zeros(1)])
        return v[v <= a]
    rate = _check(_binade(7, 0), xs_of)
    assert rate < 5e-3  # the slow path stays rare


def test_bf16_clamped_amax():
    def xs_of(a):
        v = np.concatenate([_binade(7, e) for e in range(-133, -26)] + [np.zeros(1)])
        return v[v < 1e-8]
    _check([0.0, 5e-9], xs_of)


def test_fp16_all_pairs():
    def xs_of(a):
        v = np.concatenate([_binade(10, e) for e in range(-16, 1)] + [np.zeros(1)])
        return v[v <= a]
    rate = _check(_binade(10, 0), xs_of)
    assert rate < 1e-3


def test_plain_reciprocal_would_not_be_exact():
    """Without the residual check, rint(x * r) differs from the reference."""
    mism = 0
    for a in _binade(7, 0):
        s = np.float32(np.float32(a) / np.float32(127.0))
        r = np.float32(np.float32(1.0) / s)
        v = np.concatenate([_binade(7, e) for e in range(-8, 1)]).astype(np.float32)
        v = v[v <= a]
        mism += int(np.count_nonzero(np.rint(v / s) != np.rint(v.astype(np.float64) * np.float64(r))))
    assert mism > 0
