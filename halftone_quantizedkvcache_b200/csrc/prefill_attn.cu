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
// torch kernels; here one launch reads the int8 codes.  Two kernels share the
// work decomposition:
//
//   * even group sizes (every Qwen3 shape): prefill_umma_kernel (namespace um,
//     below) - a block takes 64 query rows of the two q heads that share a kv
//     head (128 rows = 128 tensor-memory lanes, one per thread), S = Q K^T and
//     O += P V are tcgen05.mma products in tensor memory, Q arrives by TMA in
//     the swizzled layout the MMA reads and is fake-quantized in place;
//   * odd group sizes: prefill_kernel - a block takes 64 query rows of one q
//     head, 8 warps (warps w and w + 4 share 16 rows and take alternate key
//     tiles), S and P V on mma.sync m16n8k16 with ldmatrix A/B fragments.
//
// Shared by both:
//   * the 64-token key tiles that a q tile's causal rows reach are dealt round
//     robin to the C blocks of a thread-block cluster (C = 1, 2, 4 or 8, chosen
//     on the host so that the grid fills the resident block slots of the GPU;
//     the longest q tiles are scheduled first).  Each block runs an online
//     softmax over its tiles; the cluster then merges the C partial states
//     through distributed shared memory: every block leaves its unnormalised
//     output rows and (max, sum) in its own shared memory, and after a cluster
//     barrier block c merges rows c R / C .. (c + 1) R / C of all C blocks and
//     stores them.  No workspace, no second launch;
//   * code tiles (64 tokens x 128 bytes of K and of V) arrive by TMA
//     (cp.async.bulk.tensor) with mbarrier completion and bounded waits; all
//     threads dequantize them exactly as the reference's update() does (float
//     product rounded to the model dtype) into swizzled 16-bit tiles;
//   * q rows are fake-quantized per row (the reference's per-token rule) with a
//     branch-free exact quotient;
//   * the online softmax runs in float32 with the scale folded into the
//     exponent; P is split into a high and a low 16-bit part (two MMAs), so the
//     probabilities keep ~16 bits instead of the 8 of a single bf16 rounding.
// The inputs of both products are exactly the reference's 16-bit values, so
// the result differs from the float32 math of record only by accumulation
// order and the 2^-16 relative rounding of P.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>

#include "decode_common.cuh"
#include "hq_common.cuh"

namespace hq {
namespace pre {

constexpr int kD = 128;
constexpr int kRows = 64;    // q rows per head per block (16 per warp)
constexpr int kKeys = 64;    // keys per tile
constexpr int kRowB = kD * 2;  // bytes of one 16-bit row
constexpr int kMaxCluster = 8;
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  const void* q;
  int64_t qsb, qsh, qsi;       // q [B, Hq, Sq, D] element strides
  int q_heads_inner;           // q tensor map dims (D, Hq, Sq, B) instead of (D, Sq, Hq, B)
  const void* ksc;
  const void* vsc;
  int64_t kscb, ksch, kscd, vscb, vsch, vscs;
  void* out;
  int64_t osb, osh, osi;       // out [B, Sq, Hq, D] addressed as (b, h, i)
  int Hq, Hkv, Sq, S;
  int n_qt;                    // q tiles
  int n_chunks;                // blocks per cluster: key tiles dealt round robin
  float qk_scale;              // sm_scale * log2(e)
  int q_quant;
  int* status;                 // optional: HQ_ERR_DEVICE_TIMEOUT when a bounded wait gave up
};

// Shared memory of a block (bytes): G q tiles, the dequantized K and V tiles,
// the two-stage ring of code tiles, the K scales, two mbarriers.  After the
// key loop the front is reused for the partial state the cluster merges.
template <int G>
struct Cfg {
  static constexpr int kWarps = 4 * G;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kR = G * kRows;                      // q rows of the block
  static constexpr int kCode = kKeys * kD;                  // one int8 code tile
  static constexpr int kOffK = kR * kRowB;
  static constexpr int kOffV = kOffK + kKeys * kRowB;
  static constexpr int kOffRing = kOffV + kKeys * kRowB;    // stage s: K codes, V codes
  static constexpr int kOffKsc = kOffRing + 2 * 2 * kCode;  // K scales; merge weights later
  static constexpr int kOffBar = kOffKsc + kD * 4;
  static constexpr int kSmem = kOffBar + 2 * 8;
  static constexpr int kPieces = kKeys * (kD / 16) / kThreads;  // 16-code pieces per thread
  // partial state: rows of kPartStride floats (conflict-free float2 stores), then (m, l)
  static constexpr int kPartStride = kD + 8;
  static constexpr int kOffML = kR * kPartStride * 4;
  static_assert(kOffML + kR * 8 <= kOffKsc, "the partial state overlaps the K scales");
  static_assert(kOffRing % 128 == 0 && kCode % 128 == 0, "TMA destinations");
  static_assert(kR <= kD, "the merge weights (rows x blocks = kR) fit the K-scale slot");
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

// Dequantizes 16 codes (one 16-byte piece: channels 16 p .. 16 p + 15 of row r) with
// the scales sc (per channel: 8 pairs; per row: one pair repeated) into two swizzled
// chunks of a 16-bit tile: the float product code * scale (exact codes from a byte
// permute, packed f32x2 multiplies) rounded to the model dtype, as the reference's
// update() computes it.
template <int DT, bool PER_CHANNEL>
__device__ __forceinline__ void dq_piece(unsigned char* tile, int r, int p, const uint4& codes,
                                         const F2* sc) {
  const uint32_t w[4] = {codes.x, codes.y, codes.z, codes.w};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    F2 lo, hi;
    s8x4_to_f2x2(w[i], lo, hi);
    lo = f2_mul(lo, sc[PER_CHANNEL ? 2 * i : 0]);
    hi = f2_mul(hi, sc[PER_CHANNEL ? 2 * i + 1 : 0]);
    float a, b;
    f2_split(lo, a, b);
    o[2 * i] = T16<DT>::pack(a, b);
    f2_split(hi, a, b);
    o[2 * i + 1] = T16<DT>::pack(a, b);
  }
  *reinterpret_cast<uint4*>(tile + sw(r, 2 * p)) = make_uint4(o[0], o[1], o[2], o[3]);
  *reinterpret_cast<uint4*>(tile + sw(r, 2 * p + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
}

__device__ __forceinline__ float ex2_ftz(float x) {  // 2^x; -inf -> +0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// P = hi + lo with hi = RN16(P), lo = RN16(P - hi), for two probabilities: the two
// 16-bit pair words of the A-fragments.
template <int DT>
__device__ __forceinline__ void split_hilo(float a, float b, uint32_t& hw, uint32_t& lw);
template <>
__device__ __forceinline__ void split_hilo<HQ_DTYPE_BF16>(float a, float b, uint32_t& hw,
                                                          uint32_t& lw) {
  hw = T16<HQ_DTYPE_BF16>::pack(a, b);
  const F2 h = bf16x2_to_f2(hw);
  float da, db;
  f2_split(f2_sub(f2_make(a, b), h), da, db);
  lw = T16<HQ_DTYPE_BF16>::pack(da, db);
}
template <>
__device__ __forceinline__ void split_hilo<HQ_DTYPE_F16>(float a, float b, uint32_t& hw,
                                                         uint32_t& lw) {
  hw = T16<HQ_DTYPE_F16>::pack(a, b);
  const F2 h = f16x2_to_f2(hw);
  float da, db;
  f2_split(f2_sub(f2_make(a, b), h), da, db);
  lw = T16<HQ_DTYPE_F16>::pack(da, db);
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}
// address of the same shared-memory location in block `rank` of the cluster
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 dsmem_ld4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(a)
               : "memory");
  return v;
}
__device__ __forceinline__ float2 dsmem_ld2(uint32_t a) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a) : "memory");
  return v;
}
// code tiles are read by every block of the q tiles and head groups of a kv head
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Fake quantization of two 16-bit values (the reference's per-token rule on q, whose
// row maximum is itself a 16-bit value): the quotient x / s by the reciprocal and one
// FMA residual correction (rint of it equals rint(RN(x / s)) for every bf16 and fp16
// |x| <= amax), rounded half to even by adding 1.5 * 2^23, then RN16(code * s).  No
// branch and no divide.
template <int DT>
__device__ __forceinline__ uint32_t fq_pair(uint32_t w, F2 ns2, F2 r2, F2 s2) {
  const F2 m2 = f2_make(12582912.0f, 12582912.0f);
  const F2 x = DT == HQ_DTYPE_BF16 ? bf16x2_to_f2(w) : f16x2_to_f2(w);
  const F2 k = f2_sub(round_magic(quot_pair(x, ns2, r2)), m2);
  float a, c;
  f2_split(f2_mul(k, s2), a, c);
  return T16<DT>::pack(a, c);
}

template <int DT, int SDT, int G>
__global__ void __launch_bounds__(Cfg<G>::kThreads, 2)
    prefill_kernel(const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv,
                   const Params p) {
  using C = Cfg<G>;
  using E = T16<DT>;
  using SE = Elem<SDT>;
  using QT = typename E::T;
  constexpr int T = C::kThreads;
  constexpr int NP = C::kPieces;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* qs = smem_raw;
  unsigned char* kts = smem_raw + C::kOffK;
  unsigned char* vts = smem_raw + C::kOffV;
  unsigned char* ring = smem_raw + C::kOffRing;
  float* ksc = reinterpret_cast<float*>(smem_raw + C::kOffKsc);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + C::kOffBar);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hl = warp >> 2, rw = warp & 3;  // head within the block, 16-row group
  const int g = lane >> 2, t = lane & 3;
  const int nc = p.n_chunks;
  const int chunk = static_cast<int>(blockIdx.x) % nc;  // rank in the cluster
  const int qt = p.n_qt - 1 - static_cast<int>(blockIdx.x) / nc;  // longest rows first
  const int nrep = p.Hq / p.Hkv, groups = nrep / G;
  const int hk = blockIdx.y / groups;
  const int hq0 = hk * nrep + (blockIdx.y % groups) * G;
  const int b = blockIdx.z;
  const int i0 = qt * kRows;
  const int off = p.S - p.Sq;  // key index of query 0
  const int last_key = min(p.S - 1, off + min(i0 + kRows, p.Sq) - 1);
  const int n_kt = last_key / kKeys + 1;
  const int n_my = n_kt > chunk ? (n_kt - 1 - chunk) / nc + 1 : 0;  // this block's key tiles
  const uint64_t pol = l2_evict_last();

  auto issue = [&](int j) {  // thread 0: this block's tile j into stage j & 1
    const int st = j & 1, kt = chunk + j * nc;
    unsigned char* dst = ring + st * 2 * C::kCode;
    mbar_arrive_expect_tx(&full[st], 2 * C::kCode);
    dec::mmak::tma_load_4d(dst, &mk, 0, kt * kKeys, hk, b, &full[st], pol);
    dec::mmak::tma_load_4d(dst + C::kCode, &mv, 0, kt * kKeys, hk, b, &full[st], pol);
  };
  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0)
    for (int j = 0; j < min(2, n_my); ++j) issue(j);

  // V scales of this thread's code rows, one tile ahead
  const auto* vsp = reinterpret_cast<const typename SE::T*>(p.vsc) + b * p.vscb + hk * p.vsch;
  float vsr[NP];
  auto load_vs = [&](int j) {
    const int s0 = (chunk + j * nc) * kKeys;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const int s = s0 + ((tid + i * T) >> 3);
      vsr[i] = s < p.S ? SE::to_f32(vsp[s * p.vscs]) : 0.0f;
    }
  };
  if (n_my > 0) load_vs(0);

  // ---- q tiles: 4 threads per row, 32 elements each; per-row fake quantization
  {
    const int quarter = tid & 3;
#pragma unroll 1
    for (int rr = tid >> 2; rr < C::kR; rr += T / 4) {
      const int h = rr / kRows, i = i0 + rr % kRows;
      const QT* src = reinterpret_cast<const QT*>(p.q) + b * p.qsb + (hq0 + h) * p.qsh +
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
        const Quantizer qz = Quantizer::from_amax16(m);
        const float M = 12582912.0f;
#pragma unroll
        for (int e = 0; e < 32; ++e) {  // exact quotient (16-bit inputs), half-to-even code
          const float q0 = x[e] * qz.rcp;
          const float q1 = __fmaf_rn(__fmaf_rn(q0, -qz.scale, x[e]), qz.rcp, q0);
          x[e] = ((q1 + M) - M) * qz.scale;
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 w;
        w.x = E::pack(x[8 * c], x[8 * c + 1]);
        w.y = E::pack(x[8 * c + 2], x[8 * c + 3]);
        w.z = E::pack(x[8 * c + 4], x[8 * c + 5]);
        w.w = E::pack(x[8 * c + 6], x[8 * c + 7]);
        *reinterpret_cast<uint4*>(qs + sw(rr, quarter * 4 + c)) = w;
      }
    }
  }
  // ---- K scales of the kv head, one per channel
  {
    const auto* kp = reinterpret_cast<const typename SE::T*>(p.ksc) + b * p.kscb + hk * p.ksch;
    if (tid < kD) ksc[tid] = SE::to_f32(kp[tid * p.kscd]);
  }
  __syncthreads();  // q tiles and K scales complete

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.0f, l_hi = 0.0f;
  const int row_lo = i0 + rw * 16 + g, row_hi = row_lo + 8;  // query indices
  const int lim_lo = row_lo < p.Sq ? off + row_lo : -1;        // last key of each row
  const int lim_hi = row_hi < p.Sq ? off + row_hi : -1;
  const uint32_t qaddr = smem_u32(qs + hl * kRows * kRowB);
  const float qk = p.qk_scale;
  // the smallest key limit of the warp's rows (-1 when a row lies past Sq)
  const int wlim = i0 + rw * 16 + 15 < p.Sq ? off + i0 + rw * 16 : -1;

  int j = 0;
  bool failed = false;
  for (; j < n_my; ++j) {
    // ---- dequantize stage j & 1 into the 16-bit tiles
    const bool ok = mbar_wait(&full[j & 1], (j >> 1) & 1);
    if (ok) {
      const unsigned char* kc = ring + (j & 1) * 2 * C::kCode;
      const unsigned char* vc = kc + C::kCode;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        const int pi = tid + i * T, r = pi >> 3, pc = pi & 7;
        dq_piece<DT, true>(kts, r, pc, *reinterpret_cast<const uint4*>(kc + r * kD + pc * 16),
                           reinterpret_cast<const F2*>(ksc + 16 * pc));
        const F2 vs2 = f2_make(vsr[i], vsr[i]);
        dq_piece<DT, false>(vts, r, pc, *reinterpret_cast<const uint4*>(vc + r * kD + pc * 16), &vs2);
      }
    }
    if (__syncthreads_or(!ok)) {  // tiles ready; stage j & 1 consumed
      failed = true;
      break;
    }
    if (tid == 0 && j + 2 < n_my) issue(j + 2);
    if (j + 1 < n_my) load_vs(j + 1);
    const int kt = chunk + j * nc;

    // ---- S = q K^T for 64 keys: 8 n-tiles of 8 keys
    float sacc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t qa[4];
      ldsm4(qaddr + sw(rw * 16 + (lane & 15), 2 * kk + (lane >> 4)), qa);
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of n-tiles
        uint32_t bfr[4];
        const int key = np * 16 + ((lane >> 4) << 3) + (lane & 7);
        ldsm4(smem_u32(kts) + sw(key, 2 * kk + ((lane >> 3) & 1)), bfr);
        mma16816<DT>(sacc[2 * np], qa, bfr[0], bfr[1]);
        mma16816<DT>(sacc[2 * np + 1], qa, bfr[2], bfr[3]);
      }
    }
    // ---- online softmax (base 2): raw scores, the scale folded into the exponent;
    // masks only where a key of the tile lies past the warp's first row limit
    const int key0 = kt * kKeys;
    if (key0 + kKeys - 1 > wlim) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = key0 + 8 * n + 2 * t + e;
          if (key > lim_lo) sacc[n][e] = -INFINITY;
          if (key > lim_hi) sacc[n][2 + e] = -INFINITY;
        }
      }
    }
    float mx_lo = m_lo, mx_hi = m_hi;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      mx_lo = fmaxf(mx_lo, fmaxf(sacc[n][0], sacc[n][1]));
      mx_hi = fmaxf(mx_hi, fmaxf(sacc[n][2], sacc[n][3]));
    }
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
    // new running maxima (raw units); a row with no key so far keeps its state
    const float a_lo = mx_lo == -INFINITY ? 1.0f : ex2_ftz((m_lo - mx_lo) * qk);
    const float a_hi = mx_hi == -INFINITY ? 1.0f : ex2_ftz((m_hi - mx_hi) * qk);
    const float nb_lo = mx_lo == -INFINITY ? 0.0f : -mx_lo * qk;
    const float nb_hi = mx_hi == -INFINITY ? 0.0f : -mx_hi * qk;
    m_lo = mx_lo;
    m_hi = mx_hi;
    {
      const F2 alo = f2_make(a_lo, a_lo), ahi = f2_make(a_hi, a_hi);
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        float x0, x1;
        f2_split(f2_mul(f2_make(o[n][0], o[n][1]), alo), x0, x1);
        o[n][0] = x0;
        o[n][1] = x1;
        f2_split(f2_mul(f2_make(o[n][2], o[n][3]), ahi), x0, x1);
        o[n][2] = x0;
        o[n][3] = x1;
      }
    }
    F2 ls_lo = f2_make(l_lo * a_lo, 0.0f), ls_hi = f2_make(l_hi * a_hi, 0.0f);
    // ---- O += P V: P as high + low 16-bit parts (A-fragments from the S accumulators)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per k-step
      uint32_t ah[4], al[4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float* c = sacc[2 * kk + h];
        const float p0 = ex2_ftz(__fmaf_rn(c[0], qk, nb_lo)), p1 = ex2_ftz(__fmaf_rn(c[1], qk, nb_lo));
        const float p2 = ex2_ftz(__fmaf_rn(c[2], qk, nb_hi)), p3 = ex2_ftz(__fmaf_rn(c[3], qk, nb_hi));
        ls_lo = f2_add(ls_lo, f2_make(p0, p1));
        ls_hi = f2_add(ls_hi, f2_make(p2, p3));
        // fragment order a0..a3 = (g, k lo), (g+8, k lo), (g, k hi), (g+8, k hi)
        split_hilo<DT>(p0, p1, ah[2 * h], al[2 * h]);
        split_hilo<DT>(p2, p3, ah[2 * h + 1], al[2 * h + 1]);
      }
#pragma unroll
      for (int np = 0; np < 8; ++np) {  // pairs of 8-channel n-tiles
        uint32_t bfr[4];
        const int key = 16 * kk + (((lane >> 3) & 1) << 3) + (lane & 7);
        ldsm4t(smem_u32(vts) + sw(key, 2 * np + (lane >> 4)), bfr);
        mma16816<DT>(o[2 * np], ah, bfr[0], bfr[1]);
        mma16816<DT>(o[2 * np + 1], ah, bfr[2], bfr[3]);
        mma16816<DT>(o[2 * np], al, bfr[0], bfr[1]);
        mma16816<DT>(o[2 * np + 1], al, bfr[2], bfr[3]);
      }
    }
    {
      float x0, x1;
      f2_split(ls_lo, x0, x1);
      l_lo = x0 + x1;
      f2_split(ls_hi, x0, x1);
      l_hi = x0 + x1;
    }
    __syncthreads();  // the tiles are read before the next dequantization
  }
  if (failed) {
    if (tid == 0) report_error(p.status, HQ_ERR_DEVICE_TIMEOUT);
    // the copies still in flight land before the block moves on (bounded again);
    // the block then contributes an empty state
    for (int jj = j; jj < min(n_my, j + 2); ++jj) mbar_wait(&full[jj & 1], (jj >> 1) & 1);
    m_lo = m_hi = -INFINITY;
    l_lo = l_hi = 0.0f;
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  }
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);

  if (nc == 1) {
    // ---- the block holds every key tile of its rows: normalise and store [b, i, hq, :]
    const float inv_lo = l_lo > 0.0f ? 1.0f / l_lo : 0.0f;
    const float inv_hi = l_hi > 0.0f ? 1.0f / l_hi : 0.0f;
    QT* out = reinterpret_cast<QT*>(p.out) + b * p.osb + (hq0 + hl) * p.osh;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int d = 8 * n + 2 * t;
      if (row_lo < p.Sq)
        *reinterpret_cast<uint32_t*>(out + row_lo * p.osi + d) = E::pack(o[n][0] * inv_lo, o[n][1] * inv_lo);
      if (row_hi < p.Sq)
        *reinterpret_cast<uint32_t*>(out + row_hi * p.osi + d) = E::pack(o[n][2] * inv_hi, o[n][3] * inv_hi);
    }
    return;
  }

  // ---- cluster merge: the partial state of every block in its own shared memory
  __syncthreads();  // every warp is done with the q / K / V tiles
  float* part = reinterpret_cast<float*>(smem_raw);
  float2* ml = reinterpret_cast<float2*>(smem_raw + C::kOffML);
  {
    const int pr_lo = hl * kRows + rw * 16 + g, pr_hi = pr_lo + 8;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      *reinterpret_cast<float2*>(part + pr_lo * C::kPartStride + 8 * n + 2 * t) = make_float2(o[n][0], o[n][1]);
      *reinterpret_cast<float2*>(part + pr_hi * C::kPartStride + 8 * n + 2 * t) = make_float2(o[n][2], o[n][3]);
    }
    if (t == 0) {
      ml[pr_lo] = make_float2(m_lo * qk, l_lo);  // maxima in base-2 exponent units
      ml[pr_hi] = make_float2(m_hi * qk, l_hi);
    }
  }
  cluster_sync_all();  // every block's partial state is visible to the cluster
  const int rows = C::kR / nc, r0 = chunk * rows;
  float* wt = ksc;  // [rows][nc] merge weights, 1 / sum folded in
  if (tid < rows) {
    float mj[kMaxCluster], lj[kMaxCluster];
    float M = -INFINITY;
#pragma unroll
    for (int c = 0; c < kMaxCluster; ++c) {
      if (c < nc) {
        const float2 v = dsmem_ld2(dsmem_addr(ml + r0 + tid, c));
        mj[c] = v.x;
        lj[c] = v.y;
        M = fmaxf(M, v.x);
      }
    }
    float L = 0.0f;
#pragma unroll
    for (int c = 0; c < kMaxCluster; ++c) {
      if (c < nc) {
        mj[c] = (M == -INFINITY || mj[c] == -INFINITY) ? 0.0f : exp2f(mj[c] - M);
        L += mj[c] * lj[c];
      }
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
    for (int c = 0; c < kMaxCluster; ++c)
      if (c < nc) wt[tid * nc + c] = mj[c] * inv;
  }
  __syncthreads();
  QT* out = reinterpret_cast<QT*>(p.out) + b * p.osb;
#pragma unroll 1
  for (int it = tid; it < rows * (kD / 4); it += T) {
    const int r = it / (kD / 4), d4 = it % (kD / 4);
    const int pr = r0 + r;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int c = 0; c < kMaxCluster; ++c) {
      if (c < nc) {
        const float w = wt[r * nc + c];
        const float4 v = dsmem_ld4(dsmem_addr(part + pr * C::kPartStride + 4 * d4, c));
        acc.x += w * v.x;
        acc.y += w * v.y;
        acc.z += w * v.z;
        acc.w += w * v.w;
      }
    }
    const int i = i0 + pr % kRows;
    if (i < p.Sq) {
      QT* dst = out + (hq0 + pr / kRows) * p.osh + i * p.osi + 4 * d4;
      reinterpret_cast<uint32_t*>(dst)[0] = E::pack(acc.x, acc.y);
      reinterpret_cast<uint32_t*>(dst)[1] = E::pack(acc.z, acc.w);
    }
  }
  cluster_sync_all();  // no block leaves while the others may still read its shared memory
}

// ================================================================ tcgen05 version
// Used when the group size is even (two q heads of one kv head per block).
// 128 q rows (row r = 64 h + i: head h of the pair, query i of the q tile) sit
// on the 128 lanes of tensor memory; 4 warps, thread r owns row r.  Per key
// tile: S = Q K^T (128 x 64 float32) and O += P V (128 x 128 float32) are
// tcgen05.mma products issued by one thread into tensor memory (S: columns
// 0..63, O: columns 128..255); Q, the dequantized K and V tiles and P (high
// and low 16-bit parts) sit in shared memory in the 128-byte-swizzled layouts
// the MMA reads (K-major for Q, K and P; MN-major for V, whose rows are
// tokens).  Completion of the copies and of the MMAs is tracked by mbarriers
// with bounded waits.  Each thread runs the online softmax of its own row from
// a tcgen05.ld of S; O is rescaled in tensor memory when a row maximum grows by
// more than 2^8 in probability.  Q arrives by TMA in the layout the MMA reads and
// is fake-quantized in place, one row per thread.
namespace um {

constexpr int kThreads = 128;
constexpr int kR = 128;                  // q rows of a block
constexpr int kPieces = kKeys * (kD / 16) / kThreads;  // 16-code pieces per thread and tile
static_assert((kThreads / 8) * kPieces == kKeys, "rows (tid >> 3) + 16 i cover the tile once");
constexpr int kOffQ = 0;                 // 2 column blocks x 128 rows x 128 B
constexpr int kOffK = 32768;             // 2 column blocks x 64 rows x 128 B; P high part later
constexpr int kOffV = kOffK + 16384;     // 2 column blocks x 64 rows x 128 B
constexpr int kOffPl = kOffV + 16384;    // 128 rows x 128 B
constexpr int kOffCk = kOffPl + 16384;   // K codes of a tile (64 x 128 B)
constexpr int kOffCv = kOffCk + 8192;    // V codes
constexpr int kOffBar = kOffCv + 8192;   // fullK, fullV, s_done, pv_done, fullQ
constexpr int kOffTmem = kOffBar + 40;   // tensor-memory base written by tcgen05.alloc
constexpr int kSmem = 1024 + kOffTmem + 16;  // 1024: alignment of the swizzled tiles
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0, kColO = 128;
constexpr int kPartStride = kD + 8;      // cluster merge: partial rows (floats)
constexpr int kOffML = kR * kPartStride * 4;
static_assert(kOffML + kR * 8 <= kOffCk, "the partial state overlaps the code staging");
static_assert(kSmem + 1024 <= 233472 / 2, "two blocks per SM");

// 128-byte-swizzled tile of 128-byte rows: byte offset of 16-byte chunk c of row r
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

// shared-memory matrix descriptor: 128-byte swizzle, version 1
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}
// instruction descriptor, kind::f16: float32 accumulator, A and B of the model dtype
template <int DT>
__host__ __device__ constexpr uint32_t idesc(int M, int N, bool b_mn_major) {
  return (1u << 4) | (uint32_t(DT == HQ_DTYPE_BF16 ? 1 : 0) << 7) |
         (uint32_t(DT == HQ_DTYPE_BF16 ? 1 : 0) << 10) | (uint32_t(b_mn_major ? 1 : 0) << 16) |
         (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t id,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(id), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 32 consecutive float32 columns of this thread's lane, the load awaited in the same
// statement (the registers are not read before they are valid)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];\n\ttcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16 codes of one piece dequantized into two 16-byte chunks cc, cc + 1 of row r of a
// 128-byte-swizzled column block (the float product code * scale rounded to the model
// dtype, as the reference's update() computes it)
template <int DT, bool PER_CHANNEL>
__device__ __forceinline__ void dq_piece_sw(unsigned char* blk, int r, int cc, const uint4& codes,
                                            const F2* sc) {
  const uint32_t w[4] = {codes.x, codes.y, codes.z, codes.w};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    F2 lo, hi;
    s8x4_to_f2x2(w[i], lo, hi);
    lo = f2_mul(lo, sc[PER_CHANNEL ? 2 * i : 0]);
    hi = f2_mul(hi, sc[PER_CHANNEL ? 2 * i + 1 : 0]);
    float a, b;
    f2_split(lo, a, b);
    o[2 * i] = T16<DT>::pack(a, b);
    f2_split(hi, a, b);
    o[2 * i + 1] = T16<DT>::pack(a, b);
  }
  *reinterpret_cast<uint4*>(blk + sw128(r, cc)) = make_uint4(o[0], o[1], o[2], o[3]);
  *reinterpret_cast<uint4*>(blk + sw128(r, cc + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
}

// Merge of rows chunk R / NC .. of the cluster's partial states, pulled from every
// block's shared memory: (row, 4 channels) items, consecutive threads on consecutive
// channels of a row (coalesced remote reads), every load of a thread's items issued at
// once and in flight while the row weights are formed (threads < rows, into wt); then
// the weighted sums, stored as [b, i, hq, :].
template <int DT, int NC>
__device__ __forceinline__ void merge_pull(const float* part, const float2* ml, float* wt,
                                           int chunk, int tid, int i0, int hq0, int Sq,
                                           typename T16<DT>::T* out_b, int64_t osh, int64_t osi) {
  constexpr int rows = kR / NC, NQ = rows * (kD / 4) / kThreads;
  const int r0 = chunk * rows;
  float4 v[NQ][NC];
#pragma unroll
  for (int k = 0; k < NQ; ++k) {
    const int it = tid + kThreads * k, pr = r0 + (it >> 5), d4 = it & 31;
#pragma unroll
    for (int c = 0; c < NC; ++c)
      v[k][c] = dsmem_ld4(dsmem_addr(part + pr * kPartStride + 4 * d4, c));
  }
  if (tid < rows) {
    float2 mv[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) mv[c] = dsmem_ld2(dsmem_addr(ml + r0 + tid, c));
    float M = -INFINITY;
#pragma unroll
    for (int c = 0; c < NC; ++c) M = fmaxf(M, mv[c].x);
    float w[NC], L = 0.0f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      w[c] = (M == -INFINITY || mv[c].x == -INFINITY) ? 0.0f : exp2f(mv[c].x - M);
      L += w[c] * mv[c].y;
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
    for (int c = 0; c < NC; ++c) wt[tid * NC + c] = w[c] * inv;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < NQ; ++k) {
    const int it = tid + kThreads * k, rr = it >> 5, d4 = it & 31, pr = r0 + rr;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const float w = wt[rr * NC + c];
      acc.x += w * v[k][c].x;
      acc.y += w * v[k][c].y;
      acc.z += w * v[k][c].z;
      acc.w += w * v[k][c].w;
    }
    const int i = i0 + (pr & 63);
    if (i < Sq) {
      auto* dst = out_b + (hq0 + (pr >> 6)) * osh + i * osi + 4 * d4;
      reinterpret_cast<uint32_t*>(dst)[0] = T16<DT>::pack(acc.x, acc.y);
      reinterpret_cast<uint32_t*>(dst)[1] = T16<DT>::pack(acc.z, acc.w);
    }
  }
}

template <int DT, int SDT>
__global__ void __launch_bounds__(kThreads, 2)
    prefill_umma_kernel(const __grid_constant__ CUtensorMap mk,
                        const __grid_constant__ CUtensorMap mv,
                        const __grid_constant__ CUtensorMap mq, const Params p) {
  using E = T16<DT>;
  using SE = Elem<SDT>;
  using QT = typename E::T;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* qs = smem + kOffQ;
  unsigned char* kts = smem + kOffK;
  unsigned char* ph = smem + kOffK;  // P high part: the K tile is free once S is read
  unsigned char* vts = smem + kOffV;
  unsigned char* pl = smem + kOffPl;
  unsigned char* ck = smem + kOffCk;
  unsigned char* cv = smem + kOffCv;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full_k = bars;
  uint64_t* full_v = bars + 1;
  uint64_t* s_done = bars + 2;
  uint64_t* pv_done = bars + 3;
  uint64_t* full_q = bars + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int nc = p.n_chunks;
  const int chunk = static_cast<int>(blockIdx.x) % nc;
  const int qt = p.n_qt - 1 - static_cast<int>(blockIdx.x) / nc;  // longest rows first
  const int nrep = p.Hq / p.Hkv, groups = nrep / 2;
  const int hk = blockIdx.y / groups;
  const int hq0 = hk * nrep + (blockIdx.y % groups) * 2;
  const int b = blockIdx.z;
  const int i0 = qt * kRows;
  const int off = p.S - p.Sq;
  const int last_key = min(p.S - 1, off + min(i0 + kRows, p.Sq) - 1);
  const int n_kt = last_key / kKeys + 1;
  const int n_my = n_kt > chunk ? (n_kt - 1 - chunk) / nc + 1 : 0;
  const uint64_t pol = l2_evict_last();

  auto issue_k = [&](int j) {
    mbar_arrive_expect_tx(full_k, kKeys * kD);
    dec::mmak::tma_load_4d(ck, &mk, 0, (chunk + j * nc) * kKeys, hk, b, full_k, pol);
  };
  auto issue_v = [&](int j) {
    mbar_arrive_expect_tx(full_v, kKeys * kD);
    dec::mmak::tma_load_4d(cv, &mv, 0, (chunk + j * nc) * kKeys, hk, b, full_v, pol);
  };
  if (tid == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    // the block's q rows by TMA, straight into the swizzled K-major Q tile: per head of
    // the pair, two boxes of 64 rows x 64 channels (rows past Sq read as zeros)
    mbar_arrive_expect_tx(full_q, kR * kD * 2);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
      for (int cb = 0; cb < 2; ++cb) {
        unsigned char* dst = smem + kOffQ + cb * (kR * 128) + hh * (kRows * 128);
        if (p.q_heads_inner)
          dec::mmak::tma_load_4d(dst, &mq, 64 * cb, hq0 + hh, i0, b, full_q, pol);
        else
          dec::mmak::tma_load_4d(dst, &mq, 64 * cb, i0, hq0 + hh, b, full_q, pol);
      }
  }
  if (warp == 0) {  // tensor memory: S and O
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  if (tid == 0 && n_my > 0) {
    issue_k(0);
    issue_v(0);
  }

  // this thread's dequantization pieces: rows (tid >> 3) + 16 i (i < kPieces), channels
  // 16 pc .. 16 pc + 15
  const int pc = tid & 7, prow = tid >> 3;
  F2 ksc2[8];
  {
    const auto* kp = reinterpret_cast<const typename SE::T*>(p.ksc) + b * p.kscb + hk * p.ksch;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      ksc2[e] = f2_make(SE::to_f32(kp[(16 * pc + 2 * e) * p.kscd]),
                        SE::to_f32(kp[(16 * pc + 2 * e + 1) * p.kscd]));
  }
  const auto* vsp = reinterpret_cast<const typename SE::T*>(p.vsc) + b * p.vscb + hk * p.vsch;
  float vsr[kPieces];
  auto load_vs = [&](int j) {
    const int s0 = (chunk + j * nc) * kKeys + prow;
#pragma unroll
    for (int i = 0; i < kPieces; ++i) {
      const int s = s0 + 16 * i;
      vsr[i] = s < p.S ? SE::to_f32(vsp[s * p.vscs]) : 0.0f;
    }
  };
  if (n_my > 0) load_vs(0);

  // ---- q: this thread's row of the Q tile (16 chunks of 16 bytes, swizzled), fake
  // quantized in place per row (the reference's per-token rule); compact loops
  {
    const int qr = tid;
    const bool ok_q = mbar_wait(full_q, 0);
    if (!ok_q) report_error(p.status, HQ_ERR_DEVICE_TIMEOUT);
    if (p.q_quant && ok_q) {
      float m = 0.0f;
#pragma unroll 4
      for (int c = 0; c < 16; ++c) {
        const uint4 w = *reinterpret_cast<const uint4*>(qs + (c >> 3) * (kR * 128) + sw128(qr, c & 7));
        m = fmaxf(m, fmaxf(fmaxf(absmax_of_x2<DT>(w.x), absmax_of_x2<DT>(w.y)),
                           fmaxf(absmax_of_x2<DT>(w.z), absmax_of_x2<DT>(w.w))));
      }
      const Quantizer qz = Quantizer::from_amax16(m);
      const F2 r2 = f2_make(qz.rcp, qz.rcp), s2 = f2_make(qz.scale, qz.scale);
      const F2 ns2 = f2_make(-qz.scale, -qz.scale);
#pragma unroll 4
      for (int c = 0; c < 16; ++c) {
        uint4* at = reinterpret_cast<uint4*>(qs + (c >> 3) * (kR * 128) + sw128(qr, c & 7));
        uint4 w = *at;
        w.x = fq_pair<DT>(w.x, ns2, r2, s2);
        w.y = fq_pair<DT>(w.y, ns2, r2, s2);
        w.z = fq_pair<DT>(w.z, ns2, r2, s2);
        w.w = fq_pair<DT>(w.w, ns2, r2, s2);
        *at = w;
      }
    }
  }
  fence_async_smem();  // Q is read by the tensor cores
  const int r = tid, i_row = i0 + (r & 63);  // this thread's row

  // descriptors: K-major tiles advance 32 bytes per 16-element k-step inside a
  // 128-byte column block, then by the block; V (MN-major) by 16 token rows
  const uint32_t qa = smem_u32(qs), ka = smem_u32(kts), va = smem_u32(vts);
  const uint32_t pha = smem_u32(ph), pla = smem_u32(pl);
  constexpr uint32_t id_s = idesc<DT>(128, 64, false);
  constexpr uint32_t id_o = idesc<DT>(128, 128, true);
  const float qk = p.qk_scale;
  const int lim = i_row < p.Sq ? off + i_row : -1;  // last key of the row
  float m_run = -INFINITY, l_run = 0.0f;
  // issued copies / products (uniform over the block) and completions this thread saw
  int k_iss = n_my > 0 ? 1 : 0, v_iss = k_iss, s_iss = 0, pv_iss = 0;
  int k_wt = 0, v_wt = 0, s_wt = 0, pv_wt = 0;
  bool ok = true;
  int j = 0;
  for (; j < n_my; ++j) {
    const int kt = chunk + j * nc;
    // the previous P V has finished reading V and P (P's high part lies in the K tile)
    if (ok && pv_wt < pv_iss) {
      ok = mbar_wait(pv_done, pv_wt & 1);
      pv_wt += ok;
    }
    if (ok) {
      ok = mbar_wait(full_k, k_wt & 1);
      k_wt += ok;
    }
    if (ok) {
#pragma unroll
      for (int i = 0; i < kPieces; ++i) {
        const int rr = prow + 16 * i;
        const uint4 c = *reinterpret_cast<const uint4*>(ck + rr * kD + pc * 16);
        dq_piece_sw<DT, true>(kts + (pc >> 2) * (kKeys * 128), rr, (2 * pc) & 7, c, ksc2);
      }
    }
    fence_async_smem();
    tc_fence_before();
    if (__syncthreads_or(!ok)) break;
    if (j + 1 < n_my) {
      if (tid == 0) issue_k(j + 1);
      ++k_iss;
    }
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16(tmem + kColS, sdesc(qa + (kk >> 2) * (kR * 128) + (kk & 3) * 32, 16, 1024),
                sdesc(ka + (kk >> 2) * (kKeys * 128) + (kk & 3) * 32, 16, 1024), id_s, kk > 0);
      mma_commit(s_done);
    }
    ++s_iss;
    // ---- V tile while S is computed
    if (ok) {
      ok = mbar_wait(full_v, v_wt & 1);
      v_wt += ok;
    }
    if (ok) {
#pragma unroll
      for (int i = 0; i < kPieces; ++i) {
        const int rr = prow + 16 * i;
        const uint4 c = *reinterpret_cast<const uint4*>(cv + rr * kD + pc * 16);
        const F2 s2 = f2_make(vsr[i], vsr[i]);
        dq_piece_sw<DT, false>(vts + (pc >> 2) * (kKeys * 128), rr, (2 * pc) & 7, c, &s2);
      }
    }
    if (j + 1 < n_my) load_vs(j + 1);
    // ---- softmax of this row
    if (ok) {
      ok = mbar_wait(s_done, s_wt & 1);
      s_wt += ok;
    }
    tc_fence_after();
    float s[64];
    {
      float t0[32], t1[32];
      tmem_ld32(tmem + lane_base + kColS, t0);
      tmem_ld32(tmem + lane_base + kColS + 32, t1);
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        s[e] = t0[e];
        s[32 + e] = t1[e];
      }
    }
    const int key0 = kt * kKeys;
    if (key0 + kKeys - 1 > lim) {
#pragma unroll
      for (int e = 0; e < 64; ++e)
        if (key0 + e > lim) s[e] = -INFINITY;
    }
    float mx;
    {  // row maximum as a tree (short dependency chain)
      float t[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) t[e] = fmaxf(fmaxf(s[e], s[e + 16]), fmaxf(s[e + 32], s[e + 48]));
#pragma unroll
      for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int e = 0; e < w; ++e) t[e] = fmaxf(t[e], t[e + w]);
      mx = fmaxf(m_run, t[0]);
    }
    // the running maximum moves only when the row maximum grows by more than 2^8 in
    // probability: P stays below 256 (exact in its high and low parts), O and l keep
    // a common scale, and O in tensor memory is rarely rescaled
    float a = 1.0f;
    if (mx != -INFINITY && (m_run == -INFINITY || (mx - m_run) * qk > 8.0f)) {
      a = ex2_ftz((m_run - mx) * qk);
      m_run = mx;
    }
    const float nb = m_run == -INFINITY ? 0.0f : -m_run * qk;
    // O *= a in tensor memory (the previous P V has completed) when the maximum moved
    if (j > 0 && __any_sync(0xffffffffu, a != 1.0f)) {
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_base + kColO + 32 * c, o);
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] *= a;
        tmem_st32(tmem + lane_base + kColO + 32 * c, o);
      }
      tmem_wait_st();
    }
    // P = 2^(s qk - m qk): high and low 16-bit parts, K-major rows of 64 keys
    F2 ls[4];  // four partial sums of pairs (short dependency chains)
#pragma unroll
    for (int e = 0; e < 4; ++e) ls[e] = f2_make(0.0f, 0.0f);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p0 = ex2_ftz(__fmaf_rn(s[8 * c + 2 * e], qk, nb));
        const float p1 = ex2_ftz(__fmaf_rn(s[8 * c + 2 * e + 1], qk, nb));
        ls[e] = f2_add(ls[e], f2_make(p0, p1));
        split_hilo<DT>(p0, p1, hw[e], lw[e]);
      }
      *reinterpret_cast<uint4*>(ph + sw128(r, c)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(pl + sw128(r, c)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    {
      float x0, x1;
      f2_split(f2_add(f2_add(ls[0], ls[1]), f2_add(ls[2], ls[3])), x0, x1);
      l_run = l_run * a + (x0 + x1);
    }
    fence_async_smem();
    tc_fence_before();
    if (__syncthreads_or(!ok)) break;
    if (j + 1 < n_my) {
      if (tid == 0) issue_v(j + 1);
      ++v_iss;
    }
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t dv = sdesc(va + kk * 16 * 128, kKeys * 128, 1024);
        mma_f16(tmem + kColO, sdesc(pha + kk * 32, 16, 1024), dv, id_o, (j > 0 || kk > 0) ? 1u : 0u);
        mma_f16(tmem + kColO, sdesc(pla + kk * 32, 16, 1024), dv, id_o, 1u);
      }
      mma_commit(pv_done);
    }
    ++pv_iss;
  }
  // every copy and product in flight completes before the block moves on (each wait
  // bounded): in the normal case this is the wait for the last P V
  bool done = mbar_wait(full_q, 0);
  for (; k_wt < k_iss; ++k_wt) done = mbar_wait(full_k, k_wt & 1) && done;
  for (; v_wt < v_iss; ++v_wt) done = mbar_wait(full_v, v_wt & 1) && done;
  for (; s_wt < s_iss; ++s_wt) done = mbar_wait(s_done, s_wt & 1) && done;
  for (; pv_wt < pv_iss; ++pv_wt) done = mbar_wait(pv_done, pv_wt & 1) && done;
  if (j < n_my || !done) {  // a bounded wait gave up: the rows contribute nothing
    report_error(p.status, HQ_ERR_DEVICE_TIMEOUT);
    m_run = -INFINITY;
    l_run = 0.0f;
  }
  tc_fence_after();
  const bool have = n_my > 0 && l_run > 0.0f;

  if (nc == 1) {
    // ---- normalise this row into the (free) Q tile, swizzled; then store [b, i, hq, :]
    // with consecutive threads on consecutive words of a row (coalesced)
    const float inv = have ? 1.0f / l_run : 0.0f;
    __syncthreads();  // no thread still reads Q
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float o[32];
      tmem_ld32(tmem + lane_base + kColO + 32 * c, o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {  // 16-byte chunk 4 c + e of the row
        const int ch = 4 * c + e;
        *reinterpret_cast<uint4*>(qs + (ch >> 3) * (kR * 128) + sw128(r, ch & 7)) =
            make_uint4(E::pack(o[8 * e] * inv, o[8 * e + 1] * inv),
                       E::pack(o[8 * e + 2] * inv, o[8 * e + 3] * inv),
                       E::pack(o[8 * e + 4] * inv, o[8 * e + 5] * inv),
                       E::pack(o[8 * e + 6] * inv, o[8 * e + 7] * inv));
      }
    }
    __syncthreads();
    QT* out_b = reinterpret_cast<QT*>(p.out) + b * p.osb;
#pragma unroll 4
    for (int k = 0; k < kR * (kD / 2) / kThreads; ++k) {  // words (element pairs) of the tile
      const int wi = tid + kThreads * k, rr = wi >> 6, pw = wi & 63;
      const int i = i0 + (rr & 63);
      if (i < p.Sq) {
        const int ch = pw >> 2;
        const uint32_t v = *reinterpret_cast<const uint32_t*>(
            qs + (ch >> 3) * (kR * 128) + sw128(rr, ch & 7) + (pw & 3) * 4);
        reinterpret_cast<uint32_t*>(out_b + (hq0 + (rr >> 6)) * p.osh + i * p.osi)[pw] = v;
      }
    }
  } else {
    // ---- cluster merge through distributed shared memory
    float* part = reinterpret_cast<float*>(smem);
    float2* ml = reinterpret_cast<float2*>(smem + kOffML);
    __syncthreads();  // no thread still reads the tiles the partial state overwrites
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float o[32];
      tmem_ld32(tmem + lane_base + kColO + 32 * c, o);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        *reinterpret_cast<float4*>(part + r * kPartStride + 32 * c + 4 * e) =
            have ? make_float4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3])
                 : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    ml[r] = make_float2(have ? m_run * qk : -INFINITY, have ? l_run : 0.0f);
    cluster_sync_all();
    QT* out_b = reinterpret_cast<QT*>(p.out) + b * p.osb;
    float* wt = reinterpret_cast<float*>(smem + kOffCk);  // [rows][nc]; codes no longer needed
    if (nc == 2)
      merge_pull<DT, 2>(part, ml, wt, chunk, tid, i0, hq0, p.Sq, out_b, p.osh, p.osi);
    else if (nc == 4)
      merge_pull<DT, 4>(part, ml, wt, chunk, tid, i0, hq0, p.Sq, out_b, p.osh, p.osi);
    else
      merge_pull<DT, 8>(part, ml, wt, chunk, tid, i0, hq0, p.Sq, out_b, p.osh, p.osi);
    cluster_sync_all();  // no block leaves while the others may still read its shared memory
  }
  // ---- release the tensor memory
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

template <int DT, int SDT>
int launch(const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mq, const Params& p,
           dim3 grid, cudaStream_t st) {
  auto kern = prefill_umma_kernel<DT, SDT>;
  static std::atomic<uint64_t> ready{0};  // bit d: the attribute is set on device d
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t(1) << dev) : 0;
  if (!bit || !(ready.load(std::memory_order_acquire) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    ready.fetch_or(bit, std::memory_order_acq_rel);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(p.n_chunks);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mk, mv, mq, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return static_cast<int>(e);
  }
  return HQ_OK;
}

}  // namespace um

// int8 codes [B, Hkv, S, 128] with byte strides (sb, sh, ss): boxes of 64 tokens x
// 128 bytes, zero fill past S.
inline int encode_code_map(CUtensorMap* m, const void* base, int64_t sb, int64_t sh, int64_t ss,
                           int S, int Hkv, int B) {
  auto enc = dec::encode_fn();
  if (!enc) return HQ_ERR_UNSUPPORTED;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(S),
                        static_cast<cuuint64_t>(Hkv), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(ss), static_cast<cuuint64_t>(sh),
                           static_cast<cuuint64_t>(sb)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(kD), static_cast<cuuint32_t>(kKeys), 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? HQ_OK : HQ_ERR_INVALID_ARGUMENT;
}

// q [B, Hq, Sq, 128] of a 16-bit dtype with element strides (sb, sh, si): boxes of 64
// channels x 64 rows, 128-byte swizzle (the K-major layout tcgen05.mma reads), zero
// fill past Sq.  The dims run in increasing stride: (D, Sq, Hq, B), or (D, Hq, Sq, B)
// when heads are closer than rows (q viewed from [B, Sq, Hq, D]); both give the same
// shared-memory image of a box.
inline int encode_q_map(CUtensorMap* m, const void* base, int dt, int64_t sb, int64_t sh,
                        int64_t si, int Sq, int Hq, int B, int* heads_inner) {
  auto enc = dec::encode_fn();
  if (!enc) return HQ_ERR_UNSUPPORTED;
  const bool hi = sh < si;
  *heads_inner = hi ? 1 : 0;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(hi ? Hq : Sq),
                        static_cast<cuuint64_t>(hi ? Sq : Hq), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>((hi ? sh : si) * 2),
                           static_cast<cuuint64_t>((hi ? si : sh) * 2),
                           static_cast<cuuint64_t>(sb * 2)};
  cuuint32_t box[4] = {64, hi ? 1u : 64u, hi ? 64u : 1u, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(m, dt == HQ_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   4, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? HQ_OK : HQ_ERR_INVALID_ARGUMENT;
}

// Sets the kernel's dynamic shared-memory limit once per device, then launches the
// grid with clusters of `nc` blocks along x.
template <int DT, int SDT, int G>
int launch(const CUtensorMap& mk, const CUtensorMap& mv, const Params& p, dim3 grid,
           cudaStream_t st) {
  using C = Cfg<G>;
  auto kern = prefill_kernel<DT, SDT, G>;
  static std::atomic<uint64_t> ready{0};  // bit d: the attribute is set on device d
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t(1) << dev) : 0;
  if (!bit || !(ready.load(std::memory_order_acquire) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    ready.fetch_or(bit, std::memory_order_acq_rel);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(p.n_chunks);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mk, mv, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return static_cast<int>(e);
  }
  return HQ_OK;
}

// Blocks per cluster: double while every q tile still has tiles for each block and
// the grid fits the resident slots (2 blocks per SM).
inline int plan_chunks(int n_qt, int S, int head_groups, int B) {
  const int max_kt = (S - 1) / kKeys + 1;
  const int64_t units = static_cast<int64_t>(n_qt) * head_groups * B;
  const int64_t slots = 2 * static_cast<int64_t>(current_sm_count());
  int nc = 1;
  while (nc < kMaxCluster && 2 * nc <= max_kt && units * 2 * nc <= slots) nc *= 2;
  return nc;
}

template <int DT, int SDT>
int dispatch(const CUtensorMap& mk, const CUtensorMap& mv, Params& p, int B, cudaStream_t st) {
  const int nrep = p.Hq / p.Hkv;
  const int G = nrep % 2 == 0 ? 2 : 1;
  p.n_qt = (p.Sq + kRows - 1) / kRows;
  p.n_chunks = plan_chunks(p.n_qt, p.S, p.Hq / G, B);
  dim3 grid(p.n_qt * p.n_chunks, p.Hq / G, B);
  if (G == 1) return launch<DT, SDT, 1>(mk, mv, p, grid, st);
  CUtensorMap mq;
  const int rc = encode_q_map(&mq, p.q, DT, p.qsb, p.qsh, p.qsi, p.Sq, p.Hq, B, &p.q_heads_inner);
  if (rc != HQ_OK) return rc;
  return um::launch<DT, SDT>(mk, mv, mq, p, grid, st);
}

}  // namespace pre
}  // namespace hq

using namespace hq;

extern "C" int hq_prefill_int8(const void* q, int q_dtype, const int64_t q_strides[4],
                               const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                               const void* k_scale, const void* v_scale, int scale_dtype,
                               const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                               int Hq, int Hkv, int Sq, int S, int D, float sm_scale, int q_quant,
                               void* out, const int64_t out_strides[4], int* status,
                               hq_stream_t stream) {
  if (!q || !k || !v || !k_scale || !v_scale || !out || !q_strides || !kv_strides ||
      !ksc_strides || !vsc_strides || !out_strides || B < 0 || Hq <= 0 || Hkv <= 0 || Sq < 0 ||
      S < Sq)
    return HQ_ERR_INVALID_ARGUMENT;
  if (D != pre::kD || Hq % Hkv || Hq > 65535 || B > 65535 ||
      (q_dtype != HQ_DTYPE_BF16 && q_dtype != HQ_DTYPE_F16) ||
      (scale_dtype != HQ_DTYPE_F32 && scale_dtype != HQ_DTYPE_F16))
    return HQ_ERR_UNSUPPORTED;
  // 16-byte rows: q rows are read as 16-byte vectors, code tiles by TMA (16-byte
  // aligned base and strides)
  auto al = [](const void* x, uintptr_t a) { return reinterpret_cast<uintptr_t>(x) % a == 0; };
  if (q_strides[3] != 1 || out_strides[3] != 1 || kv_strides[2] % 16 || kv_strides[0] % 16 ||
      kv_strides[1] % 16 || kv_strides[2] < pre::kD || !al(k, 16) || !al(v, 16) || !al(q, 16) ||
      q_strides[0] % 8 || q_strides[1] % 8 || q_strides[2] % 8 || !al(out, 4) ||
      out_strides[0] % 2 || out_strides[1] % 2 || out_strides[2] % 2)
    return HQ_ERR_INVALID_ARGUMENT;
  if (B == 0 || Sq == 0) return HQ_OK;
  CUtensorMap mk, mv;
  int rc = pre::encode_code_map(&mk, k, kv_strides[0], kv_strides[1], kv_strides[2], S, Hkv, B);
  if (rc == HQ_OK)
    rc = pre::encode_code_map(&mv, v, kv_strides[0], kv_strides[1], kv_strides[2], S, Hkv, B);
  if (rc != HQ_OK) return rc;
  pre::Params p{};
  p.q = q;
  p.qsb = q_strides[0];
  p.qsh = q_strides[1];
  p.qsi = q_strides[2];
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
  p.status = status;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (q_dtype == HQ_DTYPE_BF16)
    return scale_dtype == HQ_DTYPE_F16 ? pre::dispatch<HQ_DTYPE_BF16, HQ_DTYPE_F16>(mk, mv, p, B, st)
                                       : pre::dispatch<HQ_DTYPE_BF16, HQ_DTYPE_F32>(mk, mv, p, B, st);
  return scale_dtype == HQ_DTYPE_F16 ? pre::dispatch<HQ_DTYPE_F16, HQ_DTYPE_F16>(mk, mv, p, B, st)
                                     : pre::dispatch<HQ_DTYPE_F16, HQ_DTYPE_F32>(mk, mv, p, B, st);
}
