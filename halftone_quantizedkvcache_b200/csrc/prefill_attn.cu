// Causal prefill attention over an int8 KV cache (sm_100a).
//
// Reference semantics: the prefill branch of quantized_attention_forward
// (tests/qwen_kvcache_full.py:95-113) over the dequantized cache that
// QuantizedKVCache.update returns (:64-65): q per-token fake quantization
// (:19-23, dims (3,)), K = dtype(code * k_scale[d]), V = dtype(code * v_scale[s]),
// GQA by repeat_interleave, softmax(q K^T * scaling + causal mask) in float32,
// P V, output [B, Sq, Hq, D].  Query i of an Sq-token step attends to keys
// 0 .. S - Sq + i (the newest Sq of S cached tokens are the queries).
//
// The reference materialises the dequantized cache and runs it through ~15
// torch kernels; here one launch reads the int8 codes once per q tile:
//
//   * grid = (q tiles of 64 rows, q head, batch), the longest (last) q tiles
//     first; 8 warps: warps w and w + 4 share q rows 16 w .. 16 w + 15 and take
//     alternate key tiles (two tiles per step), then merge their softmax states
//     in shared memory - the causal rows of the last q tile cost half the steps;
//   * q rows are fake-quantized in the prologue and kept in shared memory as
//     bf16/f16 (A-fragments by ldmatrix in every key tile);
//   * 64-token K/V tiles: int8 codes are loaded into registers one tile ahead,
//     dequantized exactly as the reference's update() does (float product,
//     rounded to the model dtype) and stored to shared memory with a 16-byte
//     XOR swizzle (conflict-free ldmatrix);
//   * S = q K^T and O += P V on the tensor cores (mma.sync m16n8k16, float32
//     accumulation) with an online float32 softmax; P is split into a high
//     and a low 16-bit part (two MMAs), so the probabilities keep ~16 bits
//     instead of the 8 of a single bf16 rounding.
// The inputs of both products are exactly the reference's 16-bit values, so
// the result differs from the float32 math of record only by accumulation
// order and the 2^-16 relative rounding of P.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>

#include "hq_common.cuh"

namespace hq {
namespace pre {

constexpr int kD = 128;
constexpr int kThreads = 256;
constexpr int kRows = 64;    // q rows per block (16 per warp)
constexpr int kKeys = 64;    // keys per tile
constexpr int kRowB = kD * 2;  // bytes of one 16-bit row
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kSmem = (kRows + 4 * kKeys) * kRowB + kD * 4;  // q, 2 K tiles, 2 V tiles, K scales

struct Params {
  const void* q;
  int64_t qsb, qsh, qsi;       // q [B, Hq, Sq, D] element strides
  const int8_t* k;
  const int8_t* v;
  int64_t kvsb, kvsh, kvss;    // codes [B, Hkv, S, D]
  const void* ksc;
  const void* vsc;
  int64_t kscb, ksch, kscd, vscb, vsch, vscs;
  void* out;
  int64_t osb, osh, osi;       // out [B, Sq, Hq, D] addressed as (b, h, i)
  int Hq, Hkv, Sq, S;
  float qk_scale;              // sm_scale * log2(e)
  int q_quant;
};

template <int DT> struct T16;
template <> struct T16<HQ_DTYPE_BF16> {
  using T = __nv_bfloat16;
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};
template <> struct T16<HQ_DTYPE_F16> {
  using T = __half;
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static float round(float x) { return __half2float(__float2half_rn(x)); }
};

template <int DT>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (DT == HQ_DTYPE_BF16) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
// byte offset of 16-byte chunk c (0..15) of row r in a tile of 256-byte rows
__device__ __forceinline__ uint32_t sw(int r, int c) {
  return static_cast<uint32_t>(r * kRowB + ((c ^ (r & 7)) << 4));
}

// Dequantizes 16 codes (one 16-byte piece) with per-element float scales and
// stores them as 16-bit values (two swizzled chunks of row r, chunks 2p, 2p+1).
template <int DT>
__device__ __forceinline__ void dq_store(unsigned char* tile, int r, int p, const uint4& codes,
                                         const float* sc) {
  const uint32_t w[4] = {codes.x, codes.y, codes.z, codes.w};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int32_t x = static_cast<int32_t>(w[i]);
    const float c0 = static_cast<float>(static_cast<int8_t>(x & 0xff));
    const float c1 = static_cast<float>(static_cast<int8_t>((x >> 8) & 0xff));
    const float c2 = static_cast<float>(static_cast<int8_t>((x >> 16) & 0xff));
    const float c3 = static_cast<float>(x >> 24);
    o[2 * i] = T16<DT>::pack(c0 * sc[4 * i], c1 * sc[4 * i + 1]);
    o[2 * i + 1] = T16<DT>::pack(c2 * sc[4 * i + 2], c3 * sc[4 * i + 3]);
  }
  *reinterpret_cast<uint4*>(tile + sw(r, 2 * p)) = make_uint4(o[0], o[1], o[2], o[3]);
  *reinterpret_cast<uint4*>(tile + sw(r, 2 * p + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
}

template <int DT, int SDT>
__global__ void __launch_bounds__(kThreads) prefill_kernel(const Params p) {
  using E = T16<DT>;
  using SE = Elem<SDT>;
  using QT = typename E::T;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* qs = smem_raw;                    // 16 KB: the q tile
  unsigned char* ks = qs + kRows * kRowB;          // 2 x 16 KB: dequantized K tiles
  unsigned char* vs = ks + 2 * kKeys * kRowB;      // 2 x 16 KB: dequantized V tiles
  float* ksc = reinterpret_cast<float*>(vs + 2 * kKeys * kRowB);  // K scales of the kv head
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rw = warp & 3, kp = warp >> 2;  // q rows 16 rw .., key tiles of parity kp
  const int g = lane >> 2, t = lane & 3;
  const int n_qt = (p.Sq + kRows - 1) / kRows;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);  // longest rows first
  const int hq = blockIdx.y, b = blockIdx.z;
  const int nrep = p.Hq / p.Hkv, hk = hq / nrep;
  const int i0 = qt * kRows;
  const int off = p.S - p.Sq;  // key index of query 0

  // ---- q tile: 4 threads per row, 32 elements each; per-row fake quantization
  {
    const int r = tid >> 2, quarter = tid & 3;
    const int i = i0 + r;
    const QT* src = reinterpret_cast<const QT*>(p.q) + b * p.qsb + hq * p.qsh +
                    static_cast<int64_t>(i < p.Sq ? i : 0) * p.qsi + quarter * 32;
    float x[32];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 w = i < p.Sq ? *reinterpret_cast<const uint4*>(src + 8 * c) : make_uint4(0, 0, 0, 0);
      float f[8];
      Vec16<DT>::unpack(w, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[8 * c + e] = f[e];
    }
    if (p.q_quant) {
      float m = 0.0f;
#pragma unroll
      for (int e = 0; e < 32; ++e) m = fmaxf(m, fabsf(x[e]));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      const Quantizer qz = Quantizer::from_amax(m);
#pragma unroll
      for (int e = 0; e < 32; ++e) x[e] = E::round(static_cast<float>(qz.code(x[e])) * qz.scale);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 w;
      w.x = E::pack(x[8 * c], x[8 * c + 1]);
      w.y = E::pack(x[8 * c + 2], x[8 * c + 3]);
      w.z = E::pack(x[8 * c + 4], x[8 * c + 5]);
      w.w = E::pack(x[8 * c + 6], x[8 * c + 7]);
      *reinterpret_cast<uint4*>(qs + sw(r, quarter * 4 + c)) = w;
    }
  }
  // ---- K scales of the kv head, one per channel
  {
    const auto* kp = reinterpret_cast<const typename SE::T*>(p.ksc) + b * p.kscb + hk * p.ksch;
    if (tid < kD) ksc[tid] = SE::to_f32(kp[tid * p.kscd]);
  }
  // dequantization: threads 0-127 fill the even tile of a step, 128-255 the odd one
  const int half = tid >> 7;
  const int pc = tid & 7;         // 16-byte piece of a code row (channels 16 pc .. 16 pc + 15)
  const int rr = (tid & 127) >> 3;  // rows rr, rr + 16, rr + 32, rr + 48 of the tile
  const int last_key = min(p.S - 1, off + min(i0 + kRows, p.Sq) - 1);
  const int n_kt = last_key >= 0 ? last_key / kKeys + 1 : 0;
  const int8_t* kbase = p.k + b * p.kvsb + hk * p.kvsh;
  const int8_t* vbase = p.v + b * p.kvsb + hk * p.kvsh;
  const auto* vsp = reinterpret_cast<const typename SE::T*>(p.vsc) + b * p.vscb + hk * p.vsch;
  uint4 kc[4], vc[4];
  float vsc[4];
  auto load_tile = [&](int kt) {  // this thread's rows of tile kt
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int s = kt * kKeys + rr + 16 * j;
      const bool in = s < p.S;
      kc[j] = in ? *reinterpret_cast<const uint4*>(kbase + s * p.kvss + 16 * pc) : make_uint4(0, 0, 0, 0);
      vc[j] = in ? *reinterpret_cast<const uint4*>(vbase + s * p.kvss + 16 * pc) : make_uint4(0, 0, 0, 0);
      vsc[j] = in ? SE::to_f32(vsp[s * p.vscs]) : 0.0f;
    }
  };
  const int n_steps = (n_kt + 1) / 2;  // two key tiles per step
  if (n_steps > 0) load_tile(half);
  __syncthreads();  // q tile and K scales complete

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.0f, l_hi = 0.0f;
  const int row_lo = i0 + rw * 16 + g, row_hi = row_lo + 8;  // query indices
  const int lim_lo = row_lo < p.Sq ? off + row_lo : -1;        // last key of each row
  const int lim_hi = row_hi < p.Sq ? off + row_hi : -1;

  unsigned char* kst = ks + kp * kKeys * kRowB;  // this warp's K / V tile of each step
  unsigned char* vst = vs + kp * kKeys * kRowB;
  for (int step = 0; step < n_steps; ++step) {
    // dequantize the two tiles held in registers into shared memory
    __syncthreads();  // the previous step's reads are done
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = rr + 16 * j;
      dq_store<DT>(ks + half * kKeys * kRowB, r, pc, kc[j], ksc + 16 * pc);
      float vv[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) vv[e] = vsc[j];
      dq_store<DT>(vs + half * kKeys * kRowB, r, pc, vc[j], vv);
    }
    __syncthreads();
    if (step + 1 < n_steps) load_tile(2 * (step + 1) + half);  // in flight during the math
    const int kt = 2 * step + kp;

    // ---- S = q K^T for 64 keys: 8 n-tiles of 8 keys
    float sacc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      // q A-fragment of this warp's 16 rows, channels 16 kk .. 16 kk + 15
      uint32_t qa[4];
      ldsm4(smem_u32(qs) + sw(rw * 16 + (lane & 15), 2 * kk + (lane >> 4)), qa);
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of n-tiles
        uint32_t bfr[4];
        const int key = np * 16 + ((lane >> 4) << 3) + (lane & 7);
        ldsm4(smem_u32(kst) + sw(key, 2 * kk + ((lane >> 3) & 1)), bfr);
        mma16816<DT>(sacc[2 * np], qa, bfr[0], bfr[1]);
        mma16816<DT>(sacc[2 * np + 1], qa, bfr[2], bfr[3]);
      }
    }
    // ---- online softmax (base 2), causal and ragged masks
    const int key0 = kt * kKeys;
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = key0 + 8 * n + 2 * t + e;
        sacc[n][e] = key <= lim_lo ? sacc[n][e] * p.qk_scale : -INFINITY;
        sacc[n][2 + e] = key <= lim_hi ? sacc[n][2 + e] * p.qk_scale : -INFINITY;
        mx_lo = fmaxf(mx_lo, sacc[n][e]);
        mx_hi = fmaxf(mx_hi, sacc[n][2 + e]);
      }
    }
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
    const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    const float a_lo = mn_lo == -INFINITY ? 1.0f : exp2f(m_lo - mn_lo);
    const float a_hi = mn_hi == -INFINITY ? 1.0f : exp2f(m_hi - mn_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    l_lo *= a_lo;
    l_hi *= a_hi;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= a_lo;
      o[n][1] *= a_lo;
      o[n][2] *= a_hi;
      o[n][3] *= a_hi;
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float plo = sacc[n][e] == -INFINITY ? 0.0f : exp2f(sacc[n][e] - mn_lo);
        const float phi = sacc[n][2 + e] == -INFINITY ? 0.0f : exp2f(sacc[n][2 + e] - mn_hi);
        sacc[n][e] = plo;
        sacc[n][2 + e] = phi;
        l_lo += plo;
        l_hi += phi;
      }
    }
    // ---- O += P V: P as high + low 16-bit parts (A-fragments from the S accumulators)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per k-step
      uint32_t ph[4], pl[4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float* c = sacc[2 * kk + h];
        const float h0 = E::round(c[0]), h1 = E::round(c[1]);
        const float h2 = E::round(c[2]), h3 = E::round(c[3]);
        ph[2 * h] = E::pack(h0, h1);          // row g, keys 2t, 2t+1 (+8 for h = 1)
        ph[2 * h + 1] = E::pack(h2, h3);      // row g + 8
        pl[2 * h] = E::pack(c[0] - h0, c[1] - h1);
        pl[2 * h + 1] = E::pack(c[2] - h2, c[3] - h3);
      }
      // fragment order a0..a3 = (g, k lo), (g+8, k lo), (g, k hi), (g+8, k hi)
      const uint32_t ah[4] = {ph[0], ph[1], ph[2], ph[3]};
      const uint32_t al[4] = {pl[0], pl[1], pl[2], pl[3]};
#pragma unroll
      for (int np = 0; np < 8; ++np) {  // pairs of 8-channel n-tiles
        uint32_t bfr[4];
        const int key = 16 * kk + (((lane >> 3) & 1) << 3) + (lane & 7);
        ldsm4t(smem_u32(vst) + sw(key, 2 * np + (lane >> 4)), bfr);
        mma16816<DT>(o[2 * np], ah, bfr[0], bfr[1]);
        mma16816<DT>(o[2 * np], al, bfr[0], bfr[1]);
        mma16816<DT>(o[2 * np + 1], ah, bfr[2], bfr[3]);
        mma16816<DT>(o[2 * np + 1], al, bfr[2], bfr[3]);
      }
    }
  }
  // ---- merge the odd-tile warps' state into the even-tile warps (same rows)
  __syncthreads();  // every warp is done with the tiles: reuse K / V as scratch
  float* mo = reinterpret_cast<float*>(ks);            // [4 warps][16][4][32 lanes]
  float* ml = reinterpret_cast<float*>(vs);            // [4 warps][4][32 lanes]
  if (kp == 1) {
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) mo[((rw * 16 + n) * 4 + e) * 32 + lane] = o[n][e];
    ml[(rw * 4 + 0) * 32 + lane] = m_lo;
    ml[(rw * 4 + 1) * 32 + lane] = m_hi;
    ml[(rw * 4 + 2) * 32 + lane] = l_lo;
    ml[(rw * 4 + 3) * 32 + lane] = l_hi;
  }
  __syncthreads();
  if (kp == 1) return;
  {
    const float m2_lo = ml[(rw * 4 + 0) * 32 + lane], m2_hi = ml[(rw * 4 + 1) * 32 + lane];
    const float mn_lo = fmaxf(m_lo, m2_lo), mn_hi = fmaxf(m_hi, m2_hi);
    const float a_lo = m_lo == -INFINITY ? 0.0f : exp2f(m_lo - mn_lo);
    const float a_hi = m_hi == -INFINITY ? 0.0f : exp2f(m_hi - mn_hi);
    const float b_lo = m2_lo == -INFINITY ? 0.0f : exp2f(m2_lo - mn_lo);
    const float b_hi = m2_hi == -INFINITY ? 0.0f : exp2f(m2_hi - mn_hi);
    l_lo = l_lo * a_lo + ml[(rw * 4 + 2) * 32 + lane] * b_lo;
    l_hi = l_hi * a_hi + ml[(rw * 4 + 3) * 32 + lane] * b_hi;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] = o[n][0] * a_lo + mo[((rw * 16 + n) * 4 + 0) * 32 + lane] * b_lo;
      o[n][1] = o[n][1] * a_lo + mo[((rw * 16 + n) * 4 + 1) * 32 + lane] * b_lo;
      o[n][2] = o[n][2] * a_hi + mo[((rw * 16 + n) * 4 + 2) * 32 + lane] * b_hi;
      o[n][3] = o[n][3] * a_hi + mo[((rw * 16 + n) * 4 + 3) * 32 + lane] * b_hi;
    }
  }
  // ---- normalise and store [b, i, hq, :]
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float inv_lo = l_lo > 0.0f ? 1.0f / l_lo : 0.0f;
  const float inv_hi = l_hi > 0.0f ? 1.0f / l_hi : 0.0f;
  QT* out = reinterpret_cast<QT*>(p.out) + b * p.osb + hq * p.osh;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int d = 8 * n + 2 * t;
    if (row_lo < p.Sq)
      *reinterpret_cast<uint32_t*>(out + row_lo * p.osi + d) = E::pack(o[n][0] * inv_lo, o[n][1] * inv_lo);
    if (row_hi < p.Sq)
      *reinterpret_cast<uint32_t*>(out + row_hi * p.osi + d) = E::pack(o[n][2] * inv_hi, o[n][3] * inv_hi);
  }
}

// Sets the kernel's dynamic shared-memory limit once per device, then launches.
template <int DT, int SDT>
int launch(const Params& p, dim3 grid, cudaStream_t st) {
  static std::atomic<uint64_t> ready{0};  // bit d: the attribute is set on device d
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t(1) << dev) : 0;
  if (!bit || !(ready.load(std::memory_order_acquire) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel<DT, SDT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    ready.fetch_or(bit, std::memory_order_acq_rel);
  }
  prefill_kernel<DT, SDT><<<grid, kThreads, kSmem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}

}  // namespace pre
}  // namespace hq

using namespace hq;

extern "C" int hq_prefill_int8(const void* q, int q_dtype, const int64_t q_strides[4],
                               const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                               const void* k_scale, const void* v_scale, int scale_dtype,
                               const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                               int Hq, int Hkv, int Sq, int S, int D, float sm_scale, int q_quant,
                               void* out, const int64_t out_strides[4], hq_stream_t stream) {
  if (!q || !k || !v || !k_scale || !v_scale || !out || !q_strides || !kv_strides ||
      !ksc_strides || !vsc_strides || !out_strides || B < 0 || Hq <= 0 || Hkv <= 0 || Sq < 0 ||
      S < Sq)
    return HQ_ERR_INVALID_ARGUMENT;
  if (D != pre::kD || Hq % Hkv || Hq > 65535 || B > 65535 ||
      (q_dtype != HQ_DTYPE_BF16 && q_dtype != HQ_DTYPE_F16) ||
      (scale_dtype != HQ_DTYPE_F32 && scale_dtype != HQ_DTYPE_F16))
    return HQ_ERR_UNSUPPORTED;
  // 16-byte rows: q rows and code rows are read as 16-byte vectors
  auto al = [](const void* x, uintptr_t a) { return reinterpret_cast<uintptr_t>(x) % a == 0; };
  if (q_strides[3] != 1 || out_strides[3] != 1 || kv_strides[2] % 16 || kv_strides[0] % 16 ||
      kv_strides[1] % 16 || !al(k, 16) || !al(v, 16) || !al(q, 16) || q_strides[0] % 8 ||
      q_strides[1] % 8 || q_strides[2] % 8 || !al(out, 4) || out_strides[0] % 2 ||
      out_strides[1] % 2 || out_strides[2] % 2)
    return HQ_ERR_INVALID_ARGUMENT;
  if (B == 0 || Sq == 0) return HQ_OK;
  pre::Params p{};
  p.q = q;
  p.qsb = q_strides[0];
  p.qsh = q_strides[1];
  p.qsi = q_strides[2];
  p.k = k;
  p.v = v;
  p.kvsb = kv_strides[0];
  p.kvsh = kv_strides[1];
  p.kvss = kv_strides[2];
  p.ksc = k_scale;
  p.vsc = v_scale;
  p.kscb = ksc_strides[0];
  p.ksch = ksc_strides[1];
  p.kscd = ksc_strides[2];
  p.vscb = vsc_strides[0];
  p.vsch = vsc_strides[1];
  p.vscs = vsc_strides[2];
  p.out = out;
  p.osb = out_strides[0];
  p.osh = out_strides[1];
  p.osi = out_strides[2];
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.Sq = Sq;
  p.S = S;
  p.qk_scale = sm_scale * pre::kLog2e;
  p.q_quant = q_quant;
  dim3 grid((Sq + pre::kRows - 1) / pre::kRows, Hq, B);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (q_dtype == HQ_DTYPE_BF16)
    return scale_dtype == HQ_DTYPE_F16 ? pre::launch<HQ_DTYPE_BF16, HQ_DTYPE_F16>(p, grid, st)
                                       : pre::launch<HQ_DTYPE_BF16, HQ_DTYPE_F32>(p, grid, st);
  return scale_dtype == HQ_DTYPE_F16 ? pre::launch<HQ_DTYPE_F16, HQ_DTYPE_F16>(p, grid, st)
                                     : pre::launch<HQ_DTYPE_F16, HQ_DTYPE_F32>(p, grid, st);
}
