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
import pytest

THR = np.float32(0.5 - 2.0 ** -15)


def _binade(mbits, e):
    return (1.0 + np.arange(2 ** mbits) / 2.0 ** mbits) * 2.0 ** e


def _check(amaxs, xs_of, rcp_ulps=0):
    flagged = total = 0
    for a in amaxs:
        a32 = np.maximum(np.float32(a), np.float32(1e-8))
        s = np.float32(a32 / np.float32(127.0))
        r = np.float32(np.float32(1.0) / s)
        for _ in range(abs(rcp_ulps)):  # a reciprocal approximation up to one ulp off
            r = np.nextafter(r, np.float32(np.inf if rcp_ulps > 0 else -np.inf))
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


@pytest.mark.parametrize("ulps", [0, -1, 1])
def test_bf16_all_pairs(ulps):
    def xs_of(a):
        v = np.concatenate([_binade(7, e) for e in range(-16, 1)] + [np.zeros(1)])
        return v[v <= a]
    rate = _check(_binade(7, 0), xs_of, ulps)
    assert rate < 5e-3  # the slow path stays rare


def test_bf16_clamped_amax():
    def xs_of(a):
        v = np.concatenate([_binade(7, e) for e in range(-133, -26)] + [np.zeros(1)])
        return v[v < 1e-8]
    _check([0.0, 5e-9], xs_of)


@pytest.mark.parametrize("ulps", [0, -1, 1])
def test_fp16_all_pairs(ulps):
    def xs_of(a):
        v = np.concatenate([_binade(10, e) for e in range(-16, 1)] + [np.zeros(1)])
        return v[v <= a]
    rate = _check(_binade(10, 0), xs_of, ulps)
    assert rate < 1e-3


@pytest.mark.parametrize("bits", [7, 10])
def test_scale_without_divide_for_16bit_amax(bits):
    """scale = q + fma(-q, 127, amax) * c with q = amax * c, c = RN(1/127), equals
    RN(amax / 127) for every bf16 (7-bit) and fp16 (10-bit) mantissa; exponents
    scale both sides exactly.  The FMA is modelled exactly with fractions."""
    from fractions import Fraction

    def rn32(fr):
        f = np.float32(float(fr))
        cands = [np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))]
        return min(cands, key=lambda v: (abs(Fraction(float(v)) - fr),
                                         int(np.float32(v).view(np.uint32)) & 1))
    c = np.float32(1) / np.float32(127)
    assert int(c.view(np.uint32)) == 0x3C010204
    for m in range(2 ** bits):
        a = np.float32(1 + m / 2 ** bits)
        q = np.float32(a * c)
        r = rn32(Fraction(float(a)) - 127 * Fraction(float(q)))
        s = rn32(Fraction(float(q)) + Fraction(float(r)) * Fraction(float(c)))
        assert s == np.float32(a / np.float32(127)), m


def test_balanced_limb_digits():
    """The decode kernel writes q * k_scale and p * v_scale as x = 65536 a + 256 b + c
    with int8 digits; every |x| <= 127 * 65793 must split without overflow."""
    KL = 127 * 65793
    xs = np.concatenate([np.arange(-KL, -KL + 70000), np.arange(-70000, 70000),
                         np.arange(KL - 70000, KL + 1),
                         np.random.default_rng(0).integers(-KL, KL + 1, 1_000_000)]).astype(np.int64)
    c = ((xs + 128) & 255) - 128
    x1 = (xs - c) >> 8
    b = ((x1 + 128) & 255) - 128
    a = (x1 - b) >> 8
    assert np.array_equal(65536 * a + 256 * b + c, xs)
    for d in (a, b, c):
        assert d.min() >= -128 and d.max() <= 127


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


def _fma32(a, b, c):
    """RN32(a * b + c) elementwise for float32 arrays.  a * b is exact in float64;
    when the float64 sum lands next to a float32 rounding boundary the value is
    recomputed exactly with fractions, so the model is exact."""
    from fractions import Fraction
    t = a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)
    r = t.astype(np.float32)
    rr = r.astype(np.float64)
    lo = np.nextafter(r, np.float32(-np.inf)).astype(np.float64)
    hi = np.nextafter(r, np.float32(np.inf)).astype(np.float64)
    near = ((np.abs(t - (rr + lo) / 2) <= np.abs(rr) * 2.0 ** -50) |
            (np.abs(t - (rr + hi) / 2) <= np.abs(rr) * 2.0 ** -50))
    for i in np.nonzero(near)[0]:
        fr = Fraction(float(a[i])) * Fraction(float(b[i])) + Fraction(float(c[i]))
        f = np.float32(float(fr))
        cands = [np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))]
        r[i] = min(cands, key=lambda v: (abs(Fraction(float(v)) - fr),
                                         int(np.float32(v).view(np.uint32)) & 1))
    return r


def _markstein(xs, s, y, steps):
    S = np.full(xs.size, s, np.float32)
    Y = np.full(xs.size, y, np.float32)
    q = (xs.astype(np.float64) * np.float64(y)).astype(np.float32)
    for _ in range(steps):
        q = _fma32(_fma32(-q, S, xs), Y, q)
    return q


def _markstein_check(amaxs, xs_of, steps=1):
    """Codes of the kernel quotient (``steps`` FMA corrections) equal the reference's."""
    for a in amaxs:
        s = np.float32(np.maximum(np.float32(a), np.float32(1e-8)) / np.float32(127))
        y = np.float32(np.float32(1) / s)
        xs = xs_of(a)
        xs = np.concatenate([xs, -xs]).astype(np.float32)
        np.testing.assert_array_equal(np.rint(_markstein(xs, s, y, steps)), np.rint(xs / s))


@pytest.mark.parametrize("bits", [7, 10])
def test_branch_free_quotient_16bit(bits):
    """The 16-bit quantize kernels compute the code as rint(q1) with q0 = x * y,
    q1 = fma(fma(-q0, s, x), y, q0), y = RN(1 / s) (hq_common.cuh, quot_pair):
    for every bf16 / fp16 pair (x, amax), |x| <= amax, rint(q1) equals the
    reference code rint(RN(x / s)) (q1 itself may differ from the IEEE quotient
    in its last bit, never across a rounding boundary of the code)."""
    def xs_of(a):
        v = np.concatenate([_binade(bits, e) for e in range(-16, 1)] + [np.zeros(1)])
        return v[v <= a]
    _markstein_check(_binade(bits, 0), xs_of)


def test_uncorrected_quotient_would_not_be_exact():
    """Without the correction step (rint(RN(x * y))) some bf16 codes differ:
    the FMA step is needed."""
    bad = 0
    for a in _binade(7, 0):
        s = np.float32(np.float32(a) / np.float32(127))
        y = np.float32(np.float32(1) / s)
        v = np.concatenate([_binade(7, e) for e in range(-16, 1)])
        xs = v[v <= a].astype(np.float32)
        bad += int(np.count_nonzero(np.rint(_markstein(xs, s, y, 0)) != np.rint(xs / s)))
    assert bad > 0


def test_branch_free_quotient_clamped_amax():
    """amax < 1e-8 (scale from the clamp): codes match for every bf16 |x| < 1e-8.
    Quotients of x below ~4e-37 lose their last bit to subnormal intermediates;
    they are < 1e-26, far from any rounding boundary of the code."""
    def xs_of(a):
        v = np.concatenate([_binade(7, e) for e in range(-133, -26)] + [np.zeros(1)])
        return v[v < 1e-8]
    _markstein_check([0.0], xs_of)
