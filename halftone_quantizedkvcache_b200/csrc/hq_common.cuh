// Shared device helpers for the Halftone int8 KV-cache kernels (sm_100a).
//
// Contents:
//   * element-type traits (bf16 / f16 / f32 inputs, int8 codes);
//   * the guarded symmetric-int8 quantizer used by every quantize-on-write
//     kernel (bit-exact with the float32 IEEE reference rule
//     scale = max(amax, 1e-8) / 127, code = clamp(rint(x / scale), -127, 127));
//   * int8 -> float conversion by byte permute (Kim et al., "Who Says
//     Elephants Can't Run", 2022: place the biased byte under the exponent of
//     2^23 and subtract);
//   * packed f32x2 arithmetic (sm_100 `fma.rn.f32x2` / `add.rn.f32x2`);
//   * mbarrier + cp.async.bulk (1-D TMA) helpers with bounded waits.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/halftone_b200.h"

namespace hq {

// ---------------------------------------------------------------- element types
template <int DT> struct Elem;
template <> struct Elem<HQ_DTYPE_F32> {
  using T = float;
  static constexpr int kBytes = 4;
  __device__ __forceinline__ static float to_f32(T v) { return v; }
  __device__ __forceinline__ static T from_f32(float v) { return v; }
};
template <> struct Elem<HQ_DTYPE_BF16> {
  using T = __nv_bfloat16;
  static constexpr int kBytes = 2;
  __device__ __forceinline__ static float to_f32(T v) { return __bfloat162float(v); }
  __device__ __forceinline__ static T from_f32(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<HQ_DTYPE_F16> {
  using T = __half;
  static constexpr int kBytes = 2;
  __device__ __forceinline__ static float to_f32(T v) { return __half2float(v); }
  __device__ __forceinline__ static T from_f32(float v) { return __float2half_rn(v); }
};

// Unpack one 16-byte vector of DT elements into floats (8 for 16-bit types, 4 for f32).
template <int DT> struct Vec16;
template <> struct Vec16<HQ_DTYPE_BF16> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <> struct Vec16<HQ_DTYPE_F16> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 p = __half22float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
};
template <> struct Vec16<HQ_DTYPE_F32> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
};

// ---------------------------------------------------------------- quantizer
// Reference rule (float32 IEEE):  scale = max(amax, 1e-8f) / 127  (true divide)
//                                 code  = clamp(rint_even(RN(x / scale)), -127, 127)
//
// Fast path: r = RN(1 / scale) once per row / column; per element one FFMA
// y = x * r + 1.5 * 2^23 rounds the exact product x * r to an integer k
// (ties to even), and d = fma(x, r, -k) is its exact-product residual.
// |x * r - RN(x / scale)| <= 127.5 * 2^-24 + 2^-18 < 2^-15 for |x| <= amax,
// so k can differ from the reference code only when |d| > 0.5 - 2^-15; those
// elements (about 1e-3 of bf16 inputs) redo the true IEEE divide.  The
// equivalence is checked exhaustively for every bf16 and fp16 (x, amax) pair by
// tests/test_quant_rounding_model.py and on the GPU by the parity tests.
//
// For 16-bit inputs the kernels skip the guard altogether: with the exact
// reciprocal y = RN(1/scale), Markstein's division with two correction steps
//   q0 = x*y, r0 = fma(-q0, s, x), q1 = fma(r0, y, q0), r1 = fma(-q1, s, x),
//   q2 = fma(r1, y, q1)
// returns the IEEE quotient RN(x/s) for every bf16 and fp16 x with |x| <= amax
// (checked exhaustively by the model test), so the code is rint(q2) with no
// branch.  amax itself has 8 (bf16) or 11 (fp16) significant bits, and
// scale = RN(amax / 127) needs no divide either: q = amax * RN(1/127), then one
// FMA correction q + fma(-q, 127, amax) * RN(1/127), exact for every such
// mantissa; the clamp value 1e-8 (not 16-bit representable) takes the divide.
constexpr float kInv127 = 0.007874015718698502f;  // RN(1/127), 0x3c010204

struct Quantizer {
  float scale;  // RN(amax / 127)
  float rcp;    // RN(1 / scale)
  __device__ __forceinline__ static Quantizer from_amax(float amax) {
    Quantizer q;
    q.scale = __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f);
    q.rcp = __frcp_rn(q.scale);
    return q;
  }
  // amax must be a bf16 or fp16 value (or below 1e-8)
  __device__ __forceinline__ static Quantizer from_amax16(float amax) {
    Quantizer q;
    if (amax >= 1e-8f) {
      const float s0 = amax * kInv127;
      q.scale = __fmaf_rn(__fmaf_rn(-s0, 127.0f, amax), kInv127, s0);
    } else {
      q.scale = __fdiv_rn(1e-8f, 127.0f);
    }
    q.rcp = __frcp_rn(q.scale);
    return q;
  }
  // Returns the code as an int in [-127, 127].
  __device__ __forceinline__ int code(float x) const {
    const float kMagic = 12582912.0f;  // 1.5 * 2^23
    float y = __fmaf_rn(x, rcp, kMagic);
    float k = y - kMagic;
    float d = __fmaf_rn(x, rcp, -k);
    int c = static_cast<int>(__float_as_uint(y) - 0x4B400000u);
    if (fabsf(d) > 0.499969482421875f) {  // 0.5 - 2^-15: redo with the IEEE divide
      float e = rintf(__fdiv_rn(x, scale));
      e = fminf(fmaxf(e, -127.0f), 127.0f);
      c = static_cast<int>(e);
    }
    return c;
  }
};

__device__ __forceinline__ uint32_t pack4_s8(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xffu) | ((static_cast<uint32_t>(b) & 0xffu) << 8) |
         ((static_cast<uint32_t>(c) & 0xffu) << 16) | (static_cast<uint32_t>(d) << 24);
}

// ---------------------------------------------------------------- int8 -> f32
// Byte i of w (a signed int8) becomes float exactly: flip the sign bit
// (b + 128 as an unsigned byte), place it in the low mantissa byte of 2^23,
// and subtract 2^23 + 128.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Converts 4 int8 in w to 4 floats, returned as two packed f32x2 (lo pair, hi pair).
struct F2 {
  unsigned long long v;
};
__device__ __forceinline__ F2 f2_make(float a, float b) {
  F2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_split(F2 x, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x.v));
}
__device__ __forceinline__ F2 f2_fma(F2 a, F2 b, F2 c) {
  F2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return d;
}
__device__ __forceinline__ F2 f2_add(F2 a, F2 b) {
  F2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d.v) : "l"(a.v), "l"(b.v));
  return d;
}
__device__ __forceinline__ F2 f2_mul(F2 a, F2 b) {
  F2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d.v) : "l"(a.v), "l"(b.v));
  return d;
}

__device__ __forceinline__ F2 f2_sub(F2 a, F2 b) {
  F2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d.v) : "l"(a.v), "l"(b.v));
  return d;
}
__device__ __forceinline__ uint32_t f2_lo_bits(F2 x) { return static_cast<uint32_t>(x.v); }
__device__ __forceinline__ uint32_t f2_hi_bits(F2 x) { return static_cast<uint32_t>(x.v >> 32); }

// Packed form of Quantizer::code for two elements with reciprocals r.  The low
// byte of each float of y is the code (y = 1.5 * 2^23 + k, |k| <= 127); dev
// accumulates the largest |residual| so the caller can take the exact path
// for the whole vector when any element lies within 2^-15 of a tie.
__device__ __forceinline__ F2 quant_pair(F2 x, F2 r, float& dev) {
  const F2 m2 = f2_make(12582912.0f, 12582912.0f);
  const F2 y = f2_fma(x, r, m2);
  const F2 d = f2_fma(x, r, f2_sub(m2, y));  // x*r - k, exact product, one rounding
  float d0, d1;
  f2_split(d, d0, d1);
  dev = fmaxf(dev, fmaxf(fabsf(d0), fabsf(d1)));
  return y;
}
constexpr float kTieGuard = 0.499969482421875f;  // 0.5 - 2^-15

// Low bytes of four floats -> one word of int8 codes.
__device__ __forceinline__ uint32_t pack_low_bytes(F2 a, F2 b) {
  const uint32_t t0 = prmt(f2_lo_bits(a), f2_hi_bits(a), 0x0040u);
  const uint32_t t1 = prmt(f2_lo_bits(b), f2_hi_bits(b), 0x0040u);
  return prmt(t0, t1, 0x5410u);
}

// Quotient x / s for a pair of 16-bit inputs (ns = -s, y = RN(1/s)): q0 = x * y
// and one FMA residual correction.  The result can differ from the IEEE
// quotient RN(x / s) in its last bit, but never across a rounding boundary of
// the code: rint(q1) == rint(RN(x / s)) for every bf16 and fp16 x with
// |x| <= amax (checked exhaustively on the host, tests/test_quant_rounding_model.py).
__device__ __forceinline__ F2 quot_pair(F2 x, F2 ns, F2 y) {
  const F2 q0 = f2_mul(x, y);
  return f2_fma(f2_fma(q0, ns, x), y, q0);
}
// rint(q) (half to even) as the low byte of q + 1.5 * 2^23
__device__ __forceinline__ F2 round_magic(F2 q) {
  return f2_add(q, f2_make(12582912.0f, 12582912.0f));
}

// max(|acc|, |w|) per 16-bit lane (the sign bit of the result is meaningless)
template <int DT>
__device__ __forceinline__ uint32_t absmax_x2(uint32_t acc, uint32_t w);
template <>
__device__ __forceinline__ uint32_t absmax_x2<HQ_DTYPE_BF16>(uint32_t acc, uint32_t w) {
  uint32_t d;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(acc), "r"(w));
  return d;
}
template <>
__device__ __forceinline__ uint32_t absmax_x2<HQ_DTYPE_F16>(uint32_t acc, uint32_t w) {
  uint32_t d;
  asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(d) : "r"(acc), "r"(w));
  return d;
}
// the larger magnitude of the two halves, as float
template <int DT>
__device__ __forceinline__ float absmax_of_x2(uint32_t w);
template <>
__device__ __forceinline__ float absmax_of_x2<HQ_DTYPE_BF16>(uint32_t w) {
  return fmaxf(fabsf(__uint_as_float(w << 16)), fabsf(__uint_as_float(w & 0xffff0000u)));
}
template <>
__device__ __forceinline__ float absmax_of_x2<HQ_DTYPE_F16>(uint32_t w) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
  return fmaxf(fabsf(f.x), fabsf(f.y));
}

__device__ __forceinline__ void s8x4_to_f2x2(uint32_t w, F2& lo, F2& hi) {
  const uint32_t kExp = 0x4B000000u;
  const uint32_t u = w ^ 0x80808080u;
  F2 a, b;
  a.v = (static_cast<unsigned long long>(prmt(u, kExp, 0x7651u)) << 32) | prmt(u, kExp, 0x7650u);
  b.v = (static_cast<unsigned long long>(prmt(u, kExp, 0x7653u)) << 32) | prmt(u, kExp, 0x7652u);
  const F2 bias = f2_make(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
  lo = f2_add(a, bias);
  hi = f2_add(b, bias);
}

// bf16 pair word -> packed f32x2 (exact)
__device__ __forceinline__ F2 bf16x2_to_f2(uint32_t w) {
  F2 r;
  r.v = (static_cast<unsigned long long>(w & 0xffff0000u) << 32) | (w << 16);
  return r;
}
__device__ __forceinline__ F2 f16x2_to_f2(uint32_t w) {
  __half2 h = *reinterpret_cast<const __half2*>(&w);
  float2 p = __half22float2(h);
  return f2_make(p.x, p.y);
}

// ---------------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// raises the transaction bytes the current phase waits for, without arriving
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// 16-byte global -> shared copy; src_bytes 0 fills the slot with zeros
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes,
                                           uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(src_bytes), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// 16-byte global -> shared copy (L2 only)
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}

// Bounded wait: returns false after kSpinLimit polls (each try_wait itself
// suspends for a hardware-defined interval), never hangs.
constexpr uint32_t kSpinLimit = 1u << 22;
// Nanoseconds of the GPU's global timer.
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// 1-D bulk copy global -> this CTA's shared memory (no tensor map); `bytes` and
// both addresses must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Records a device-side error in the caller's status word (first error wins).
__device__ __forceinline__ void report_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

}  // namespace hq
