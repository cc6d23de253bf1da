// Quantize-on-write kernels (sm_100a): symmetric int8, K per channel, V per token.
//
// Reference semantics: quantize_int8 (reference/page_attention_int8_pytorch.py:23-30)
// with reduce dim 2 (K) / 3 (V) of [B, H, S, D], as used by QuantizedKVCache.update
// (tests/qwen_kvcache_full.py:41-47).  The reference's fused Triton kernels
// (src/kernels/quant_kv_triton.py:16-87) run one program per column / row and,
// for K, read each column twice with a 256-byte stride.  Here:
//
//   * V per token: each row of D elements is read once with 16-byte vector
//     loads by 4-8 lanes holding several vectors each, reduced with 2-3 warp
//     shuffle rounds, and written as packed int8 (8 codes per 16-byte input
//     vector).
//   * K per channel: teams of blocks take one (b, h) slab at a time; pass A
//     publishes the column maxima, pass B re-reads the chunks from L2 and
//     writes codes, so HBM sees 1 read + 1 int8 write per element; on large
//     inputs the two blocks of an SM split the passes (one HBM-bound, one
//     compute-bound).
//   * Append: one block per (b, h) quantizes the few new tokens of K (per
//     channel over the new tokens; scale not stored) and V (per token; scale
//     stored), exactly as the reference's update() does on a non-empty layer.
#include <algorithm>
#include <atomic>
#include <cstdio>

#include "hq_common.cuh"

namespace hq {

constexpr int kThreads = 256;

// ------------------------------------------------------------------ V per token
template <int DT, int D>
struct VShape {
  static constexpr int kVecElems = 16 / Elem<DT>::kBytes;   // elements per 16-byte vector
  static constexpr int kVecPerRow = D / kVecElems;
  // few lanes per row, several vectors per lane: the row maximum then costs 2-3
  // shuffle rounds per row instead of 4-5 (at most 8 vectors in flight per lane)
  static constexpr int kLanesPerRow =
      kVecPerRow <= 4 ? kVecPerRow : (kVecPerRow / 8 > 4 ? kVecPerRow / 8 : 4);
  static constexpr int kVecPerLane = kVecPerRow / kLanesPerRow;
  static constexpr int kRowsPerWarp = 32 / kLanesPerRow;
};

template <int N>
__device__ __forceinline__ void store_codes(int8_t* dst, const int* c);
template <>
__device__ __forceinline__ void store_codes<8>(int8_t* dst, const int* c) {
  uint2 w;
  w.x = pack4_s8(c[0], c[1], c[2], c[3]);
  w.y = pack4_s8(c[4], c[5], c[6], c[7]);
  *reinterpret_cast<uint2*>(dst) = w;
}
template <>
__device__ __forceinline__ void store_codes<4>(int8_t* dst, const int* c) {
  *reinterpret_cast<uint32_t*>(dst) = pack4_s8(c[0], c[1], c[2], c[3]);
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Unpacks a 16-byte vector into packed float pairs (4 pairs for 16-bit types, 2 for f32).
template <int DT>
__device__ __forceinline__ void vec_to_f2(const uint4& v, F2* f);
template <>
__device__ __forceinline__ void vec_to_f2<HQ_DTYPE_BF16>(const uint4& v, F2* f) {
  f[0] = bf16x2_to_f2(v.x);
  f[1] = bf16x2_to_f2(v.y);
  f[2] = bf16x2_to_f2(v.z);
  f[3] = bf16x2_to_f2(v.w);
}
template <>
__device__ __forceinline__ void vec_to_f2<HQ_DTYPE_F16>(const uint4& v, F2* f) {
  f[0] = f16x2_to_f2(v.x);
  f[1] = f16x2_to_f2(v.y);
  f[2] = f16x2_to_f2(v.z);
  f[3] = f16x2_to_f2(v.w);
}
template <>
__device__ __forceinline__ void vec_to_f2<HQ_DTYPE_F32>(const uint4& v, F2* f) {
  f[0].v = (static_cast<unsigned long long>(v.y) << 32) | v.x;
  f[1].v = (static_cast<unsigned long long>(v.w) << 32) | v.z;
}

// Quantizes one 16-byte vector (VE elements) with per-element quantizers qz
// (pairs: ns2 = -scale, rcp2 = RN(1/scale)) and stores its VE codes at dst.
// 16-bit inputs: exact quotient, no branch.  f32 inputs: one-FFMA fast path
// guarded by the tie check, exact divide for the (rare) flagged vector.
template <int DT>
__device__ __forceinline__ void quant_vec_store(const uint4& v, const F2* ns2, const F2* rcp2,
                                                const Quantizer* qz, int8_t* dst) {
  constexpr int VE = Vec16<DT>::N;
  F2 x[VE / 2];
  vec_to_f2<DT>(v, x);
  F2 y[VE / 2];
  if constexpr (DT != HQ_DTYPE_F32) {
#pragma unroll
    for (int p = 0; p < VE / 2; ++p) y[p] = round_magic(quot_pair(x[p], ns2[p], rcp2[p]));
  } else {
    float dev = 0.0f;
#pragma unroll
    for (int p = 0; p < VE / 2; ++p) y[p] = quant_pair(x[p], rcp2[p], dev);
    if (dev > kTieGuard) {  // rare: some element sits next to a rounding tie
      float f[VE];
      Vec16<DT>::unpack(v, f);
      int c[VE];
#pragma unroll
      for (int e = 0; e < VE; ++e) c[e] = qz[e].code(f[e]);
      store_codes<VE>(dst, c);
      return;
    }
  }
  if constexpr (VE == 8) {
    uint2 w;
    w.x = pack_low_bytes(y[0], y[1]);
    w.y = pack_low_bytes(y[2], y[3]);
    *reinterpret_cast<uint2*>(dst) = w;
  } else {
    *reinterpret_cast<uint32_t*>(dst) = pack_low_bytes(y[0], y[1]);
  }
}

template <int DT>
__device__ __forceinline__ Quantizer quantizer_for(float amax) {
  return DT == HQ_DTYPE_F32 ? Quantizer::from_amax(amax) : Quantizer::from_amax16(amax);
}

// |x| maximum over one 16-byte vector, folded into a running float maximum
template <int DT>
__device__ __forceinline__ float vec_absmax(const uint4& v, float m) {
  if constexpr (DT == HQ_DTYPE_F32) {
    float f[4];
    Vec16<DT>::unpack(v, f);
    return fmaxf(fmaxf(m, fmaxf(fabsf(f[0]), fabsf(f[1]))), fmaxf(fabsf(f[2]), fabsf(f[3])));
  } else {
    const uint32_t a = absmax_x2<DT>(absmax_x2<DT>(v.x, v.y), absmax_x2<DT>(v.z, v.w));
    return fmaxf(m, absmax_of_x2<DT>(a));
  }
}

// grid = (token blocks, slabs); each warp quantizes kIters groups of
// kRowsPerWarp rows, all of whose loads are issued before any compute.
template <int DT, int D>
__global__ void __launch_bounds__(kThreads) quant_v_kernel(
    const char* __restrict__ x, int64_t xsb, int64_t xsh, int64_t xss, int H, int S, int n_slabs,
    int8_t* __restrict__ q, int64_t qsb, int64_t qsh, int64_t qss, float* __restrict__ sc32,
    __half* __restrict__ sc16, int64_t ssb, int64_t ssh, int64_t sss) {
  using Sh = VShape<DT, D>;
  constexpr int EB = Elem<DT>::kBytes;
  constexpr int VE = Sh::kVecElems;
  constexpr int IT = Sh::kVecPerLane >= 4 ? 1 : 4 / Sh::kVecPerLane;
  constexpr int kRowsPerWarp = Sh::kRowsPerWarp * IT;
  constexpr int kRowsPerBlock = (kThreads / 32) * kRowsPerWarp;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane % Sh::kLanesPerRow;
  for (int slab = blockIdx.y; slab < n_slabs; slab += gridDim.y) {
    const int b = slab / H, h = slab - (slab / H) * H;
    const char* base = x + (static_cast<int64_t>(b) * xsb + static_cast<int64_t>(h) * xsh) * EB;
    int8_t* qbase = q + static_cast<int64_t>(b) * qsb + static_cast<int64_t>(h) * qsh;
    const int s0 = blockIdx.x * kRowsPerBlock + warp * kRowsPerWarp + lane / Sh::kLanesPerRow;
    uint4 vec[IT][Sh::kVecPerLane];
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int s = s0 + it * Sh::kRowsPerWarp;
#pragma unroll
      for (int i = 0; i < Sh::kVecPerLane; ++i)
        vec[it][i] = s < S ? ldg_stream(base + static_cast<int64_t>(s) * xss * EB +
                                        (sub + i * Sh::kLanesPerRow) * 16)
                           : make_uint4(0, 0, 0, 0);
    }
    // row maxima of the IT row groups, then one quantizer per row computed by
    // lane sub == it of the row's lanes and broadcast to them
    float amax[IT];
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      float m = 0.0f;
#pragma unroll
      for (int i = 0; i < Sh::kVecPerLane; ++i) m = vec_absmax<DT>(vec[it][i], m);
#pragma unroll
      for (int off = Sh::kLanesPerRow / 2; off > 0; off >>= 1)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      amax[it] = m;
    }
    const int my_it = sub % IT;
    float my_amax = amax[0];
#pragma unroll
    for (int it = 1; it < IT; ++it) my_amax = my_it == it ? amax[it] : my_amax;
    const Quantizer mine = quantizer_for<DT>(my_amax);
    const int my_s = s0 + my_it * Sh::kRowsPerWarp;
    if (sub < IT && my_s < S) {
      const int64_t so = static_cast<int64_t>(b) * ssb + static_cast<int64_t>(h) * ssh +
                         static_cast<int64_t>(my_s) * sss;
      if (sc32) sc32[so] = mine.scale;
      if (sc16) sc16[so] = __float2half_rn(mine.scale);
    }
    const int group_base = lane - sub;
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int s = s0 + it * Sh::kRowsPerWarp;
      Quantizer qz = mine;  // one row group: every lane holds its row's maximum
      if constexpr (IT > 1) {
        qz.scale = __shfl_sync(0xffffffffu, mine.scale, group_base + it);
        qz.rcp = __shfl_sync(0xffffffffu, mine.rcp, group_base + it);
      }
      if (s >= S) continue;
      Quantizer qzv[VE];
      F2 rcp2[VE / 2], ns2[VE / 2];
#pragma unroll
      for (int e = 0; e < VE; ++e) qzv[e] = qz;
#pragma unroll
      for (int p = 0; p < VE / 2; ++p) {
        rcp2[p] = f2_make(qz.rcp, qz.rcp);
        ns2[p] = f2_make(-qz.scale, -qz.scale);
      }
#pragma unroll
      for (int i = 0; i < Sh::kVecPerLane; ++i)
        quant_vec_store<DT>(vec[it][i], ns2, rcp2, qzv,
                            qbase + static_cast<int64_t>(s) * qss + (sub + i * Sh::kLanesPerRow) * VE);
    }
  }
}

// ------------------------------------------------------------------ K per channel
// A (b, h) slab of S x D is cut into chunks of kRowsPerChunk whole rows (32 KB
// of input).  Each slab is processed in two passes over its chunks:
//   A  read the chunks and fold column maxima in registers; reduce over the
//      block and publish to the slab's global maxima (one atomicMax per column,
//      waited for), then count the block for the slab;
//   B  once every A block of the slab is counted, re-read the chunks - from L2,
//      they were read moments before - and write codes.
// The persistent grid (every block resident) is split into teams; team t
// handles slabs t, t + T, ..., and a team block takes one contiguous run of
// each slab's chunks.  Paired grids (large inputs): the two blocks of a pair
// (blockIdx i and i + G/2 - normally the two blocks of one SM) split the
// passes: the first runs pass A only (HBM-bound), the second pass B only
// (compute-bound), so every SM keeps both kinds of work in flight; the A side
// runs at most two slabs ahead of the B side (bounded L2 footprint: T slabs
// being re-read and T being read, T chosen to fit kTeamBytes).  Small grids:
// every block runs A then B of its run, waiting for its team in between.
// Waits are bounded and only point to lower slab indices (no cycle); a block
// that gives up sets the status word and skips its codes.
// Chunks stream through a kKStages-deep shared-memory ring with cp.async that
// runs ahead across pass and slab boundaries.
constexpr int kKStages = 3;
constexpr size_t kTeamBytes = size_t(64) << 20;  // input of the slabs in flight

template <int DT, int D>
struct KShape {
  static constexpr int kVecElems = 16 / Elem<DT>::kBytes;
  static constexpr int kVecPerRow = D / kVecElems;             // column groups
  static constexpr int kRowSlots = kThreads / kVecPerRow;      // rows per pass
  static constexpr int kPasses = 8;
  static constexpr int kRowsPerChunk = kRowSlots * kPasses;    // 32 KB of input
  static constexpr int kWarps = kThreads / 32;
  // rows of the block-level max table: one per warp when a warp spans whole
  // rows, else one per row slot
  static constexpr int kRedRows = kVecPerRow <= 32 ? kWarps : kRowSlots;
  static constexpr int kStageVecs = kThreads * kPasses;        // 16-byte slots per stage
  static constexpr size_t kTableOff = size_t(kKStages) * kStageVecs * 16;
  static constexpr size_t kQsOff = kTableOff + size_t(kRedRows) * D * 4;
  static constexpr size_t kSmem = kQsOff + size_t(D) * 8;
};

constexpr int kMaxSmIds = 1024;  // per-SM arrival counters (paired grids)

struct KWorkspace {
  int* status;        // [1]
  int* roles;         // [2] blocks that took role A / role B (paired grids)
  int* sm_slot;       // [kMaxSmIds] blocks that started on each SM (paired grids)
  int* a_done;        // [B*H] A blocks that published the slab's maxima
  int* b_done;        // [B*H] B blocks that finished the slab (paired grids)
  unsigned* amax;     // [B*H*D] column absmax as float bits (all >= 0)
};

struct KPlan {
  int n_slabs, n_chunks, teams;
  int paired;         // blocks i < G/2 run pass A, blocks i >= G/2 pass B
};

// bounded wait until *cnt >= target (thread-uniform call by one thread)
__device__ __forceinline__ bool wait_count(const int* cnt, int target) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    int c;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(c) : "l"(cnt) : "memory");
    if (c >= target) return true;
    __nanosleep(64);
  }
  return false;
}

__host__ __device__ inline size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// L2 policies: A reads keep their chunk in L2 for the B re-read, B reads mark it
// as last use.
__device__ __forceinline__ uint64_t l2_policy_keep() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_drop() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

template <int DT, int D>
__global__ void __launch_bounds__(kThreads, 2) quant_k_kernel(
    const char* __restrict__ x, int64_t xsb, int64_t xsh, int64_t xss, int H, int S, KPlan pl,
    int8_t* __restrict__ q, int64_t qsb, int64_t qsh, int64_t qss, float* __restrict__ sc32,
    __half* __restrict__ sc16, KWorkspace ws) {
  using Sh = KShape<DT, D>;
  constexpr int EB = Elem<DT>::kBytes;
  constexpr int VE = Sh::kVecElems;
  constexpr int NS = kKStages;
  extern __shared__ __align__(128) unsigned char smem[];
  uint4* stages = reinterpret_cast<uint4*>(smem);
  float* table = reinterpret_cast<float*>(smem + Sh::kTableOff);  // [kRedRows][D]
  float* qr = reinterpret_cast<float*>(smem + Sh::kQsOff);
  float* qn = qr + D;
  __shared__ int s_ok;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int cg = tid % Sh::kVecPerRow;      // column group: columns cg*VE .. +VE
  const int rs = tid / Sh::kVecPerRow;      // row slot
  const int red_row = Sh::kVecPerRow <= 32 ? warp : rs;
  const bool red_writer = Sh::kVecPerRow <= 32 ? lane < Sh::kVecPerRow : true;
  const int T = pl.teams;
  const int half = pl.paired ? gridDim.x / 2 : gridDim.x;   // blocks per role
  int idx = blockIdx.x, role = 0;
  if (pl.paired) {
    // the first block to start on an SM runs pass A, the second pass B, so that
    // each SM holds one HBM-bound and one compute-bound block; the index within
    // the role comes from a counter (a full role hands the block to the other)
    __shared__ int s_role[2];
    if (tid == 0) {
      unsigned smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      int r = smid < kMaxSmIds ? (atomicAdd(ws.sm_slot + smid, 1) & 1) : 0;
      int i = atomicAdd(ws.roles + r, 1);
      if (i >= half) {
        r ^= 1;
        i = atomicAdd(ws.roles + r, 1);
      }
      s_role[0] = r;
      s_role[1] = i;
    }
    __syncthreads();
    role = s_role[0];
    idx = s_role[1];
  }
  const bool run_a = !pl.paired || role == 0;
  const bool run_b = !pl.paired || role == 1;
  const int team = idx % T, rank = idx / T;
  const int members = (half - team + T - 1) / T;   // role blocks of the team
  const int lo = static_cast<int>(static_cast<int64_t>(pl.n_chunks) * rank / members);
  const int hi = static_cast<int>(static_cast<int64_t>(pl.n_chunks) * (rank + 1) / members);
  const int n_k = team < pl.n_slabs ? (pl.n_slabs - team + T - 1) / T : 0;
  const uint64_t pol_keep = l2_policy_keep(), pol_drop = l2_policy_drop();

  // prefetch cursor over (slab k of the team, pass, chunk r): the passes this
  // block runs, A before B for each slab
  int pf_k = 0, pf_pass = run_a ? 0 : 1, pf_r = lo;
  const bool empty = lo >= hi;
  auto issue = [&](int stage) {
    if (!empty && pf_k < n_k) {
      const int slab = team + pf_k * T;
      const int b = slab / H, h = slab - (slab / H) * H;
      const char* base = x + (static_cast<int64_t>(b) * xsb + static_cast<int64_t>(h) * xsh) * EB + cg * 16;
      const int row0 = pf_r * Sh::kRowsPerChunk;
      const uint64_t pol = pf_pass == 0 ? pol_keep : pol_drop;
      uint4* dst = stages + stage * Sh::kStageVecs + tid;
#pragma unroll
      for (int p = 0; p < Sh::kPasses; ++p) {
        const int s = row0 + p * Sh::kRowSlots + rs;
        const char* src = s < S ? base + static_cast<int64_t>(s) * xss * EB : base;
        cp_async16(dst + p * kThreads, src, s < S ? 16 : 0, pol);
      }
      if (++pf_r >= hi) {
        pf_r = lo;
        if (pf_pass == 0 && run_b) {
          pf_pass = 1;
        } else {
          pf_pass = run_a ? 0 : 1;
          ++pf_k;
        }
      }
    }
    cp_async_commit();
  };

  for (int k = 0; k < NS - 1; ++k) issue(k);
  int it = 0;  // chunks consumed (ring position)
  for (int k = 0; k < n_k; ++k) {
    const int slab = team + k * T;
    const int64_t col0 = static_cast<int64_t>(slab) * D;
    bool ok = true;
    if (run_a) {
      // paired: stay at most two slabs ahead of the B side
      if (pl.paired && k >= 2) {
        if (tid == 0) {
          const bool seen = wait_count(ws.b_done + (slab - 2 * T), members);
          if (!seen) report_error(ws.status, HQ_ERR_DEVICE_TIMEOUT);
        }
        __syncthreads();
      }
      // ---- A: column maxima of this block's run
      float cmax[VE];
#pragma unroll
      for (int e = 0; e < VE; ++e) cmax[e] = 0.0f;
      for (int r = lo; r < hi; ++r, ++it) {
        issue((it + NS - 1) % NS);
        cp_async_wait<NS - 1>();  // this thread's copies of chunk `it` have landed
        const uint4* st = stages + (it % NS) * Sh::kStageVecs + tid;
        if constexpr (DT == HQ_DTYPE_F32) {
#pragma unroll
          for (int p = 0; p < Sh::kPasses; ++p) {
            float f[VE];
            Vec16<DT>::unpack(st[p * kThreads], f);
#pragma unroll
            for (int e = 0; e < VE; ++e) cmax[e] = fmaxf(cmax[e], fabsf(f[e]));
          }
        } else {
          uint4 m = st[0];
#pragma unroll
          for (int p = 1; p < Sh::kPasses; ++p) {
            const uint4 d = st[p * kThreads];
            m.x = absmax_x2<DT>(m.x, d.x);
            m.y = absmax_x2<DT>(m.y, d.y);
            m.z = absmax_x2<DT>(m.z, d.z);
            m.w = absmax_x2<DT>(m.w, d.w);
          }
          float f[VE];
          Vec16<DT>::unpack(m, f);
#pragma unroll
          for (int e = 0; e < VE; ++e) cmax[e] = fmaxf(cmax[e], fabsf(f[e]));
        }
      }
      // lanes of one warp that share a column group differ in bits >= log2(kVecPerRow)
#pragma unroll
      for (int off = Sh::kVecPerRow; off < 32; off <<= 1)
#pragma unroll
        for (int e = 0; e < VE; ++e) cmax[e] = fmaxf(cmax[e], __shfl_xor_sync(0xffffffffu, cmax[e], off));
      if (red_writer) {
#pragma unroll
        for (int e = 0; e < VE; ++e) table[red_row * D + cg * VE + e] = cmax[e];
      }
      __syncthreads();  // block table complete; qs of the previous slab no longer read
      float m = 0.0f;
      if (tid < D) {
        m = table[tid];
#pragma unroll
        for (int w = 1; w < Sh::kRedRows; ++w) m = fmaxf(m, table[w * D + tid]);
      }
      if (members == 1 && !pl.paired) {
        // the whole slab is this block's run: the block maximum is final
        if (tid < D) {
          const Quantizer qz = quantizer_for<DT>(m);
          qr[tid] = qz.rcp;
          qn[tid] = -qz.scale;
          if (sc32) sc32[col0 + tid] = qz.scale;
          if (sc16) sc16[col0 + tid] = __float2half_rn(qz.scale);
        }
        __syncthreads();  // qs ready; table free for the next slab
      } else {
        // publish; the returned old value is awaited, so the maximum is
        // performed in L2 before this block is counted
        if (tid < D && m > 0.0f) {
          const unsigned old = atomicMax(ws.amax + col0 + tid, __float_as_uint(m));
          if (old == 0xffffffffu) s_ok = 0;  // never: maxima are >= 0; forces the wait
        }
        __syncthreads();  // table free for the next slab
        if (tid == 0) {
          __threadfence();
          atomicAdd(ws.a_done + slab, 1);
        }
      }
    }
    if (run_b) {
      if (pl.paired || members > 1) {
        // every A block of the slab has published: quantizers from the maxima
        if (tid == 0) {
          const bool seen = wait_count(ws.a_done + slab, members);
          if (!seen) report_error(ws.status, HQ_ERR_DEVICE_TIMEOUT);
          s_ok = seen;
        }
        __syncthreads();
        ok = s_ok != 0;  // gave up: status word set, this slab's codes are not written
        if (ok && tid < D) {
          const Quantizer qz = quantizer_for<DT>(__uint_as_float(__ldcg(ws.amax + col0 + tid)));
          qr[tid] = qz.rcp;
          qn[tid] = -qz.scale;
          if (rank == 0) {  // one block per slab writes the scale outputs
            if (sc32) sc32[col0 + tid] = qz.scale;
            if (sc16) sc16[col0 + tid] = __float2half_rn(qz.scale);
          }
        }
        __syncthreads();  // qs ready
      }
      // ---- B: codes of the run
      Quantizer qz[VE];
      F2 rcp2[VE / 2], ns2[VE / 2];
      {
        const float4* r4 = reinterpret_cast<const float4*>(qr + cg * VE);
        const float4* n4 = reinterpret_cast<const float4*>(qn + cg * VE);
#pragma unroll
        for (int e = 0; e < VE / 4; ++e) {
          const float4 r = r4[e], n = n4[e];
          rcp2[2 * e] = f2_make(r.x, r.y);
          rcp2[2 * e + 1] = f2_make(r.z, r.w);
          ns2[2 * e] = f2_make(n.x, n.y);
          ns2[2 * e + 1] = f2_make(n.z, n.w);
          qz[4 * e + 0] = {-n.x, r.x};
          qz[4 * e + 1] = {-n.y, r.y};
          qz[4 * e + 2] = {-n.z, r.z};
          qz[4 * e + 3] = {-n.w, r.w};
        }
      }
      const int b = slab / H, h = slab - (slab / H) * H;
      int8_t* qbase = q + static_cast<int64_t>(b) * qsb + static_cast<int64_t>(h) * qsh + cg * VE;
      for (int r = lo; r < hi; ++r, ++it) {
        issue((it + NS - 1) % NS);
        cp_async_wait<NS - 1>();
        const uint4* st = stages + (it % NS) * Sh::kStageVecs + tid;
        if (ok) {
          const int row0 = r * Sh::kRowsPerChunk;
#pragma unroll
          for (int p = 0; p < Sh::kPasses; ++p) {
            const int s = row0 + p * Sh::kRowSlots + rs;
            if (s < S) quant_vec_store<DT>(st[p * kThreads], ns2, rcp2, qz, qbase + static_cast<int64_t>(s) * qss);
          }
        }
      }
      if (pl.paired) {
        __syncthreads();  // qs is rewritten for the next slab; the run is consumed
        if (tid == 0) atomicAdd(ws.b_done + slab, 1);
      }
    }
  }
  cp_async_wait<0>();
}

// ------------------------------------------------------------------ K per channel, static scales
// Codes for given (calibrated) per-channel scales: q = clamp(rint(x / s[d]), +-127),
// the reference's quantize_int8 rule (reference/page_attention_int8_pytorch.py:23-30)
// with the scale supplied instead of found.  No maximum is searched, so it is a
// single streaming pass like the V kernel.  Values beyond the calibrated range
// clamp to +-127; NaN inputs give an unspecified code.
//
// rint(x * RN(1/s)) equals rint(RN(x / s)) whenever the exact residual
// x * RN(1/s) - k stays within 0.5 - 2^-15 of the integer k and |k| <= 128 (the
// reciprocal's relative error moves the quotient by at most 128 * 2^-24 there);
// other elements take the IEEE divide, and |k| > 128 clamps either way.
__device__ __forceinline__ int static_code(float x, float s, float rcp) {
  float k = rintf(x * rcp);
  if (fabsf(k) <= 128.0f && fabsf(__fmaf_rn(x, rcp, -k)) > kTieGuard) k = rintf(__fdiv_rn(x, s));
  if (k != k) k = 0.0f;
  return static_cast<int>(fminf(fmaxf(k, -127.0f), 127.0f));
}

// One 16-byte vector with per-element static scales (sc, rc = RN(1/sc); r2 the
// reciprocals as pairs).  16-bit inputs: packed x * r + 1.5 * 2^23 (the code in
// the low byte), clamped to +-127, with the exact path for the whole vector
// when any residual lies within 2^-15 of a tie; f32 inputs element by element.
template <int DT>
__device__ __forceinline__ void static_vec_store(const uint4& v, const F2* r2, const float* sc,
                                                 const float* rc, int8_t* dst) {
  constexpr int VE = Vec16<DT>::N;
  if constexpr (DT != HQ_DTYPE_F32) {
    F2 x[VE / 2], y[VE / 2];
    vec_to_f2<DT>(v, x);
    float dev = 0.0f;
#pragma unroll
    for (int p = 0; p < VE / 2; ++p) y[p] = quant_pair(x[p], r2[p], dev);
    if (dev <= kTieGuard) {
      const float lo = 12582912.0f - 127.0f, hi = 12582912.0f + 127.0f;
#pragma unroll
      for (int p = 0; p < VE / 2; ++p) {
        float a, b;
        f2_split(y[p], a, b);
        y[p] = f2_make(fminf(fmaxf(a, lo), hi), fminf(fmaxf(b, lo), hi));
      }
      uint2 w;
      w.x = pack_low_bytes(y[0], y[1]);
      w.y = pack_low_bytes(y[2], y[3]);
      *reinterpret_cast<uint2*>(dst) = w;
      return;
    }
  }
  float f[VE];
  Vec16<DT>::unpack(v, f);
  int c[VE];
#pragma unroll
  for (int e = 0; e < VE; ++e) c[e] = static_code(f[e], sc[e], rc[e]);
  store_codes<VE>(dst, c);
}

// grid = (row blocks, slabs); each thread quantizes one 16-byte vector of IT rows.
template <int DT, int D, int SDT>
__global__ void __launch_bounds__(kThreads) quant_k_static_kernel(
    const char* __restrict__ x, int64_t xsb, int64_t xsh, int64_t xss, int H, int S, int n_slabs,
    const void* __restrict__ scale, int64_t ssb, int64_t ssh, int64_t ssd, int8_t* __restrict__ q,
    int64_t qsb, int64_t qsh, int64_t qss) {
  constexpr int EB = Elem<DT>::kBytes;
  constexpr int VE = 16 / EB;
  constexpr int VPR = D / VE;
  constexpr int RS = kThreads / VPR;
  constexpr int IT = 4;
  const int cg = threadIdx.x % VPR, rs = threadIdx.x / VPR;
  const auto* sp = reinterpret_cast<const typename Elem<SDT>::T*>(scale);
  for (int slab = blockIdx.y; slab < n_slabs; slab += gridDim.y) {
    const int b = slab / H, h = slab - (slab / H) * H;
    float sc[VE], rc[VE];
    F2 r2[VE / 2];
#pragma unroll
    for (int e = 0; e < VE; ++e) {
      sc[e] = Elem<SDT>::to_f32(sp[b * ssb + h * ssh + (cg * VE + e) * ssd]);
      rc[e] = __frcp_rn(sc[e]);
    }
#pragma unroll
    for (int p = 0; p < VE / 2; ++p) r2[p] = f2_make(rc[2 * p], rc[2 * p + 1]);
    const char* base = x + (static_cast<int64_t>(b) * xsb + static_cast<int64_t>(h) * xsh) * EB + cg * 16;
    int8_t* qbase = q + static_cast<int64_t>(b) * qsb + static_cast<int64_t>(h) * qsh + cg * VE;
    for (int r0 = blockIdx.x * RS * IT; r0 < S; r0 += gridDim.x * RS * IT) {
      uint4 v[IT];
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int s = r0 + it * RS + rs;
        v[it] = s < S ? ldg_stream(base + static_cast<int64_t>(s) * xss * EB) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int s = r0 + it * RS + rs;
        if (s < S) static_vec_store<DT>(v[it], r2, sc, rc, qbase + static_cast<int64_t>(s) * qss);
      }
    }
  }
}

// ------------------------------------------------------------------ append
// One block of D threads per (b, h); thread d owns channel d.
template <int DT, int D>
__global__ void __launch_bounds__(D) append_kernel(
    const char* __restrict__ k, const char* __restrict__ v, int64_t ksb, int64_t ksh, int64_t kss,
    int64_t vsb, int64_t vsh, int64_t vss, int H, int S_new, int8_t* __restrict__ kq,
    int64_t kqb, int64_t kqh, int64_t kqs, int8_t* __restrict__ vq, int64_t vqb, int64_t vqh,
    int64_t vqs, float* __restrict__ vs32, __half* __restrict__ vs16, int64_t vssb, int64_t vssh,
    int64_t vsss, int* __restrict__ lens, int cap, const void* __restrict__ kst, int kst_f16,
    int64_t kstb, int64_t ksth, int64_t kstd) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int kW = D / 32;
  __shared__ float wmax[kW];
  __shared__ int s_row0;
  const int d = threadIdx.x;
  const int64_t b = blockIdx.x / H, h = blockIdx.x % H;
  // device-resident length: the new rows go to lens[0] .. lens[0] + S_new - 1
  int64_t row0 = 0;
  if (lens) {
    if (d == 0) s_row0 = __ldcg(lens);
    __syncthreads();
    row0 = s_row0;
    if (row0 < 0 || row0 + S_new > cap) {  // full cache: nothing is written
      if (d == 0) report_error(lens + 2, HQ_ERR_INVALID_ARGUMENT);
      return;
    }
    kq += row0 * kqs;
    vq += row0 * vqs;
    if (vs32) vs32 += row0 * vsss;
    if (vs16) vs16 += row0 * vsss;
  }
  const T* kp = reinterpret_cast<const T*>(k) + b * ksb + h * ksh + d;
  const T* vp = reinterpret_cast<const T*>(v) + b * vsb + h * vsh + d;
  if (kst) {
    // K with the given static per-channel scale of channel d
    const int64_t si = b * kstb + h * ksth + d * kstd;
    const float sk = kst_f16 ? __half2float(reinterpret_cast<const __half*>(kst)[si])
                             : reinterpret_cast<const float*>(kst)[si];
    const float rk = __frcp_rn(sk);
    for (int s = 0; s < S_new; ++s)
      kq[b * kqb + h * kqh + s * kqs + d] = static_cast<int8_t>(static_code(E::to_f32(kp[s * kss]), sk, rk));
  } else {
    // K: per-channel over the S_new new tokens
    float amax = 0.0f;
    for (int s = 0; s < S_new; ++s) amax = fmaxf(amax, fabsf(E::to_f32(kp[s * kss])));
    const Quantizer qk = Quantizer::from_amax(amax);
    for (int s = 0; s < S_new; ++s)
      kq[b * kqb + h * kqh + s * kqs + d] = static_cast<int8_t>(qk.code(E::to_f32(kp[s * kss])));
  }
  // V: per token over D
  for (int s = 0; s < S_new; ++s) {
    const float xv = E::to_f32(vp[s * vss]);
    float m = fabsf(xv);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((d & 31) == 0) wmax[d >> 5] = m;
    __syncthreads();
    m = wmax[0];
#pragma unroll
    for (int w = 1; w < kW; ++w) m = fmaxf(m, wmax[w]);
    __syncthreads();
    const Quantizer qv = Quantizer::from_amax(m);
    vq[b * vqb + h * vqh + s * vqs + d] = static_cast<int8_t>(qv.code(xv));
    if (d == 0) {
      const int64_t so = b * vssb + h * vssh + s * vsss;
      if (vs32) vs32[so] = qv.scale;
      if (vs16) vs16[so] = __float2half_rn(qv.scale);
    }
  }
  if (lens) {
    // every block has read lens[0]; the last one to arrive advances it
    __syncthreads();
    if (d == 0) {
      __threadfence();
      if (atomicAdd(lens + 1, 1) == static_cast<int>(gridDim.x) - 1) {
        lens[1] = 0;
        lens[0] = static_cast<int>(row0) + S_new;
      }
    }
  }
}

// ------------------------------------------------------------------ dequant
template <int SDT, int ODT>
__global__ void __launch_bounds__(kThreads) dequant_kernel(
    const int8_t* __restrict__ q, int64_t qsb, int64_t qsh, int64_t qss, int H, int S, int D,
    const void* __restrict__ scale, int64_t ssb, int64_t ssh, int64_t ssx, int per_channel,
    void* __restrict__ out, int64_t osb, int64_t osh, int64_t oss, int64_t n) {
  using SE = Elem<SDT>;
  using OE = Elem<ODT>;
  const auto* sc = reinterpret_cast<const typename SE::T*>(scale);
  auto* o = reinterpret_cast<typename OE::T*>(out);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t d = i % D;
    const int64_t r = i / D;
    const int64_t s = r % S, bh = r / S;
    const int64_t h = bh % H, b = bh / H;
    const float c = static_cast<float>(q[b * qsb + h * qsh + s * qss + d]);
    const float f = SE::to_f32(sc[b * ssb + h * ssh + (per_channel ? d : s) * ssx]);
    o[b * osb + h * osh + s * oss + d] = OE::from_f32(c * f);
  }
}

// ------------------------------------------------------------------ host helpers
// Per-device number of SMs the grids are planned for (0: the device's own).
static std::atomic<int> g_plan_sms[64];

int sm_count(int dev) {
  static std::atomic<int> cache[64];
  if (dev < 0 || dev >= 64) return 148;
  const int planned = g_plan_sms[dev].load(std::memory_order_relaxed);
  if (planned > 0) return planned;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
    v = 148;
  cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

int current_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  return sm_count(dev);
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static int finish_launch() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}

template <int DT, int D>
static int launch_quant_v(const void* x, const int64_t* xs, int B, int H, int S, int8_t* q,
                          const int64_t* qs, float* s32, uint16_t* s16, const int64_t* ss,
                          cudaStream_t st) {
  using Sh = VShape<DT, D>;
  constexpr int IT = Sh::kVecPerLane >= 4 ? 1 : 4 / Sh::kVecPerLane;
  constexpr int kRowsPerBlock = (kThreads / 32) * Sh::kRowsPerWarp * IT;
  const int n_slabs = B * H;
  const int64_t z[3] = {0, 0, 0};
  if (!ss) ss = z;
  dim3 grid((S + kRowsPerBlock - 1) / kRowsPerBlock, n_slabs < 65535 ? n_slabs : 65535);
  quant_v_kernel<DT, D><<<grid, kThreads, 0, st>>>(
      static_cast<const char*>(x), xs[0], xs[1], xs[2], H, S, n_slabs, q, qs[0], qs[1], qs[2], s32,
      reinterpret_cast<__half*>(s16), ss[0], ss[1], ss[2]);
  return finish_launch();
}

template <int DT, int D>
static int launch_quant_k(const void* x, const int64_t* xs, int B, int H, int S, int8_t* q,
                          const int64_t* qs, float* s32, uint16_t* s16, void* wsp,
                          cudaStream_t st) {
  using Sh = KShape<DT, D>;
  auto kern = quant_k_kernel<DT, D>;
  constexpr size_t smem = Sh::kSmem;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<int> occ_cache[64];
  int per_sm = (dev >= 0 && dev < 64) ? occ_cache[dev].load(std::memory_order_relaxed) : 0;
  cudaError_t e;
  if (per_sm <= 0) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (per_sm <= 0) return HQ_ERR_UNSUPPORTED;
    if (dev >= 0 && dev < 64) occ_cache[dev].store(per_sm, std::memory_order_relaxed);
  }
  KPlan pl;
  pl.n_slabs = B * H;
  pl.n_chunks = (S + Sh::kRowsPerChunk - 1) / Sh::kRowsPerChunk;
  // Blocks wait for one another: the grid never exceeds what is resident at
  // once.  Paired when every role block still gets >= 2 chunks per slab pass on
  // average; teams: as many slabs in flight as fit in kTeamBytes (paired: two
  // per team), no more teams than slabs, no team larger than a slab has chunks.
  const int64_t resident = static_cast<int64_t>(per_sm) * sm_count(dev);
  const size_t slab_bytes = static_cast<size_t>(S) * D * Elem<DT>::kBytes;
  const int64_t total_chunks = static_cast<int64_t>(pl.n_slabs) * pl.n_chunks;
  pl.paired = resident >= 4 && total_chunks >= 4 * resident && pl.n_chunks > 1;
  const int64_t role_blocks = pl.paired ? resident / 2 : resident;
  int64_t teams = static_cast<int64_t>(kTeamBytes / ((pl.paired ? 2 : 1) * (slab_bytes ? slab_bytes : 1)));
  teams = std::max<int64_t>(teams, (role_blocks + pl.n_chunks - 1) / pl.n_chunks);
  teams = std::min<int64_t>(std::max<int64_t>(teams, 1), pl.n_slabs);
  pl.teams = static_cast<int>(teams);
  int64_t grid;
  if (pl.paired) {
    grid = 2 * role_blocks;
  } else {
    grid = std::min<int64_t>(resident, teams * pl.n_chunks);
    grid = std::max<int64_t>(grid, teams);
  }
  char* w = static_cast<char*>(wsp);
  const size_t nbh = static_cast<size_t>(B) * H;
  KWorkspace ws;
  ws.status = reinterpret_cast<int*>(w);
  ws.roles = reinterpret_cast<int*>(w + 8);
  ws.sm_slot = reinterpret_cast<int*>(w + 256);
  char* w2 = w + 256 + sizeof(int) * kMaxSmIds;
  ws.a_done = reinterpret_cast<int*>(w2);
  ws.b_done = reinterpret_cast<int*>(w2 + align256(sizeof(int) * nbh));
  ws.amax = reinterpret_cast<unsigned*>(w2 + 2 * align256(sizeof(int) * nbh));
  // status, role and SM counters, per-slab counters and maxima start at zero
  const size_t clear = 256 + sizeof(int) * kMaxSmIds + 2 * align256(sizeof(int) * nbh) +
                       sizeof(unsigned) * nbh * D;
  e = cudaMemsetAsync(wsp, 0, clear, st);
  if (e != cudaSuccess) return static_cast<int>(e);
  // Blocks wait for one another (pass B for pass A's counts): a cooperative
  // launch, so a grid that cannot be resident all at once (SMs held by other
  // work, or planned for more SMs than there are) is refused at launch with
  // cudaErrorCooperativeLaunchTooLarge instead of running into its bounded waits.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, static_cast<const char*>(x), xs[0], xs[1], xs[2], H, S, pl, q,
                         qs[0], qs[1], qs[2], s32, reinterpret_cast<__half*>(s16), ws);
  if (e != cudaSuccess) {
    cudaGetLastError();  // a refused launch leaves no error behind for the caller's next call
    return static_cast<int>(e);
  }
  return HQ_OK;
}

template <int DT, int D>
static int launch_append(const void* k, const void* v, const int64_t* ks, const int64_t* vs,
                         int B, int H, int S_new, int8_t* kq, const int64_t* kqs, int8_t* vq,
                         const int64_t* vqs, float* v32, uint16_t* v16, const int64_t* vss,
                         int* lens, int cap, cudaStream_t st, const void* k_static = nullptr,
                         int k_static_f16 = 0, const int64_t* kss = nullptr) {
  const int64_t z[3] = {0, 0, 0};
  if (!vss) vss = z;
  if (!kss) kss = z;
  append_kernel<DT, D><<<B * H, D, 0, st>>>(
      static_cast<const char*>(k), static_cast<const char*>(v), ks[0], ks[1], ks[2], vs[0], vs[1],
      vs[2], H, S_new, kq, kqs[0], kqs[1], kqs[2], vq, vqs[0], vqs[1], vqs[2], v32,
      reinterpret_cast<__half*>(v16), vss[0], vss[1], vss[2], lens, cap, k_static, k_static_f16,
      kss[0], kss[1], kss[2]);
  return finish_launch();
}

template <int DT, int D>
static int launch_quant_k_static(const void* x, const int64_t* xs, int B, int H, int S,
                                 const void* scale, int scale_dtype, const int64_t* ss, int8_t* q,
                                 const int64_t* qs, cudaStream_t st) {
  constexpr int VPR = D / (16 / Elem<DT>::kBytes);
  constexpr int rows_per_block = (kThreads / VPR) * 4;
  const int n_slabs = B * H;
  // enough row blocks per slab to put ~8 blocks on every SM, at least one
  const int64_t want = std::max<int64_t>(1, 8LL * current_sm_count() / std::max(n_slabs, 1));
  const int64_t need = (S + rows_per_block - 1) / rows_per_block;
  dim3 grid(static_cast<unsigned>(std::min(want, need)), n_slabs < 65535 ? n_slabs : 65535);
  if (scale_dtype == HQ_DTYPE_F16)
    quant_k_static_kernel<DT, D, HQ_DTYPE_F16><<<grid, kThreads, 0, st>>>(
        static_cast<const char*>(x), xs[0], xs[1], xs[2], H, S, n_slabs, scale, ss[0], ss[1], ss[2],
        q, qs[0], qs[1], qs[2]);
  else
    quant_k_static_kernel<DT, D, HQ_DTYPE_F32><<<grid, kThreads, 0, st>>>(
        static_cast<const char*>(x), xs[0], xs[1], xs[2], H, S, n_slabs, scale, ss[0], ss[1], ss[2],
        q, qs[0], qs[1], qs[2]);
  return finish_launch();
}

// ------------------------------------------------------------------ column maxima
// max |x| over the tokens of x [B, H, S, D] per (b, h, d): the input of the K scale
// of a bulk write sharded along the sequence (each rank reduces its own tokens and
// the ranks combine their maxima with one all-reduce, after which the codes come from
// the static-scale kernel with scale = RN(max(amax, 1e-8) / 127), the reference's
// rule).  grid (row chunks of kAbsRows, H, B): a block folds its rows into
// per-column maxima (16-byte vectors; a row slot per D / VE threads), reduces the
// row slots in shared memory and publishes one atomicMax per column (float bits:
// every value is >= 0).  amax is zero-filled by the entry point first.
constexpr int kAbsRows = 512;

template <int DT, int D>
__global__ void __launch_bounds__(kThreads) column_absmax_kernel(
    const char* __restrict__ x, int64_t xsb, int64_t xsh, int64_t xss, int S,
    unsigned* __restrict__ amax) {
  constexpr int EB = Elem<DT>::kBytes, VE = 16 / EB, VPR = D / VE, RS = kThreads / VPR;
  __shared__ float red[RS][D];
  const int tid = threadIdx.x, cg = tid % VPR, rs = tid / VPR;
  const int64_t b = blockIdx.z, h = blockIdx.y;
  const int r0 = static_cast<int>(blockIdx.x) * kAbsRows, r1 = min(S, r0 + kAbsRows);
  const char* base = x + (b * xsb + h * xsh) * EB + cg * 16;
  float m[VE];
#pragma unroll
  for (int e = 0; e < VE; ++e) m[e] = 0.0f;
#pragma unroll 4
  for (int r = r0 + rs; r < r1; r += RS) {
    float f[VE];
    Vec16<DT>::unpack(ldg_stream(base + static_cast<int64_t>(r) * xss * EB), f);
#pragma unroll
    for (int e = 0; e < VE; ++e) m[e] = fmaxf(m[e], fabsf(f[e]));
  }
#pragma unroll
  for (int e = 0; e < VE; ++e) red[rs][cg * VE + e] = m[e];
  __syncthreads();
  if (tid < D) {
    float a = red[0][tid];
#pragma unroll
    for (int w = 1; w < RS; ++w) a = fmaxf(a, red[w][tid]);
    atomicMax(amax + (b * gridDim.y + h) * D + tid, __float_as_uint(a));
  }
}

// the reference's scale of a column maximum: RN(max(amax, 1e-8) / 127)
__global__ void k_scale_from_amax_kernel(const float* __restrict__ amax, int n,
                                         float* __restrict__ s32, __half* __restrict__ s16) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float s = Quantizer::from_amax(amax[i]).scale;
  if (s32) s32[i] = s;
  if (s16) s16[i] = __float2half_rn(s);
}

template <int DT, int D>
static int launch_column_absmax(const void* x, const int64_t* xs, int B, int H, int S,
                                float* amax, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(float) * static_cast<size_t>(B) * H * D, st);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (S == 0) return HQ_OK;
  dim3 grid((S + kAbsRows - 1) / kAbsRows, H, B);
  column_absmax_kernel<DT, D><<<grid, kThreads, 0, st>>>(static_cast<const char*>(x), xs[0], xs[1],
                                                         xs[2], S, reinterpret_cast<unsigned*>(amax));
  return finish_launch();
}

static bool valid_dtype_x(int dt) {
  return dt == HQ_DTYPE_F32 || dt == HQ_DTYPE_BF16 || dt == HQ_DTYPE_F16;
}
static int esize(int dt) { return dt == HQ_DTYPE_F32 ? 4 : dt == HQ_DTYPE_I8 ? 1 : 2; }

// rows of D elements starting at 16-byte boundaries
static bool rows16(const void* p, const int64_t* st, int dt) {
  const int64_t e = esize(dt);
  return aligned(p, 16) && (st[0] * e) % 16 == 0 && (st[1] * e) % 16 == 0 &&
         (st[2] * e) % 16 == 0 && st[3] == 1;
}

}  // namespace hq

using namespace hq;

#define HQ_DISPATCH_D(D, ...)                       \
  switch (D) {                                      \
    case 64: { constexpr int kD = 64; __VA_ARGS__ } \
    case 128: { constexpr int kD = 128; __VA_ARGS__ } \
    case 256: { constexpr int kD = 256; __VA_ARGS__ } \
    default: return HQ_ERR_UNSUPPORTED;             \
  }
#define HQ_DISPATCH_X(DT, ...)                                       \
  switch (DT) {                                                      \
    case HQ_DTYPE_F32: { constexpr int kDT = HQ_DTYPE_F32; __VA_ARGS__ } \
    case HQ_DTYPE_BF16: { constexpr int kDT = HQ_DTYPE_BF16; __VA_ARGS__ } \
    case HQ_DTYPE_F16: { constexpr int kDT = HQ_DTYPE_F16; __VA_ARGS__ } \
    default: return HQ_ERR_UNSUPPORTED;                              \
  }

extern "C" size_t hq_quant_k_workspace_bytes(int B, int H, int D) {
  if (B < 0 || H < 0 || D < 0) return 0;
  const size_t nbh = static_cast<size_t>(B) * H;
  return 256 + sizeof(int) * kMaxSmIds + 2 * align256(sizeof(int) * nbh) +
         align256(sizeof(unsigned) * nbh * D);
}

extern "C" int hq_quant_k_perchannel(const void* x, int x_dtype, const int64_t x_strides[4], int B,
                                     int H, int S, int D, int8_t* q, const int64_t q_strides[4],
                                     float* scale_f32, uint16_t* scale_f16, void* workspace,
                                     size_t workspace_bytes, hq_stream_t stream) {
  if (!x || !q || !x_strides || !q_strides || B < 0 || H < 0 || S < 1) return HQ_ERR_INVALID_ARGUMENT;
  if (!valid_dtype_x(x_dtype)) return HQ_ERR_UNSUPPORTED;
  if (B == 0 || H == 0) return HQ_OK;
  if (!rows16(x, x_strides, x_dtype) || q_strides[3] != 1 || !aligned(q, 8) ||
      q_strides[0] % 8 || q_strides[1] % 8 || q_strides[2] % 8)
    return HQ_ERR_INVALID_ARGUMENT;
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < hq_quant_k_workspace_bytes(B, H, D))
    return HQ_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  HQ_DISPATCH_X(x_dtype, HQ_DISPATCH_D(D, return launch_quant_k<kDT, kD>(
                                              x, x_strides, B, H, S, q, q_strides, scale_f32,
                                              scale_f16, workspace, st);))
}

extern "C" int hq_quant_v_pertoken(const void* x, int x_dtype, const int64_t x_strides[4], int B,
                                   int H, int S, int D, int8_t* q, const int64_t q_strides[4],
                                   float* scale_f32, uint16_t* scale_f16,
                                   const int64_t scale_strides[3], hq_stream_t stream) {
  if (!x || !q || !x_strides || !q_strides || B < 0 || H < 0 || S < 1) return HQ_ERR_INVALID_ARGUMENT;
  if ((scale_f32 || scale_f16) && !scale_strides) return HQ_ERR_INVALID_ARGUMENT;
  if (!valid_dtype_x(x_dtype)) return HQ_ERR_UNSUPPORTED;
  if (B == 0 || H == 0) return HQ_OK;
  if (!rows16(x, x_strides, x_dtype) || q_strides[3] != 1 || !aligned(q, 8) ||
      q_strides[0] % 8 || q_strides[1] % 8 || q_strides[2] % 8)
    return HQ_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  HQ_DISPATCH_X(x_dtype, HQ_DISPATCH_D(D, return launch_quant_v<kDT, kD>(
                                              x, x_strides, B, H, S, q, q_strides, scale_f32,
                                              scale_f16, scale_strides, st);))
}

extern "C" int hq_append_kv(const void* k_new, const void* v_new, int x_dtype,
                            const int64_t k_strides[4], const int64_t v_strides[4], int B, int H,
                            int S_new, int D, int8_t* k_dst, const int64_t kq_strides[4],
                            int8_t* v_dst, const int64_t vq_strides[4], float* v_scale_f32,
                            uint16_t* v_scale_f16, const int64_t vs_strides[3],
                            hq_stream_t stream) {
  if (!k_new || !v_new || !k_dst || !v_dst || !k_strides || !v_strides || !kq_strides ||
      !vq_strides || B < 0 || H < 0 || S_new < 1 || S_new > 64)
    return HQ_ERR_INVALID_ARGUMENT;
  if ((v_scale_f32 || v_scale_f16) && !vs_strides) return HQ_ERR_INVALID_ARGUMENT;
  if (k_strides[3] != 1 || v_strides[3] != 1 || kq_strides[3] != 1 || vq_strides[3] != 1)
    return HQ_ERR_INVALID_ARGUMENT;
  if (!valid_dtype_x(x_dtype)) return HQ_ERR_UNSUPPORTED;
  if (B == 0 || H == 0) return HQ_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  HQ_DISPATCH_X(x_dtype, HQ_DISPATCH_D(D, return launch_append<kDT, kD>(
                                              k_new, v_new, k_strides, v_strides, B, H, S_new,
                                              k_dst, kq_strides, v_dst, vq_strides, v_scale_f32,
                                              v_scale_f16, vs_strides, nullptr, 0, st);))
}

extern "C" int hq_quant_k_static(const void* x, int x_dtype, const int64_t x_strides[4], int B,
                                 int H, int S, int D, const void* k_scale, int scale_dtype,
                                 const int64_t scale_strides[3], int8_t* q,
                                 const int64_t q_strides[4], hq_stream_t stream) {
  if (!x || !q || !k_scale || !x_strides || !q_strides || !scale_strides || B < 0 || H < 0 || S < 1)
    return HQ_ERR_INVALID_ARGUMENT;
  if (!valid_dtype_x(x_dtype) || (scale_dtype != HQ_DTYPE_F32 && scale_dtype != HQ_DTYPE_F16))
    return HQ_ERR_UNSUPPORTED;
  if (B == 0 || H == 0) return HQ_OK;
  if (!rows16(x, x_strides, x_dtype) || q_strides[3] != 1 || !aligned(q, 8) ||
      q_strides[0] % 8 || q_strides[1] % 8 || q_strides[2] % 8)
    return HQ_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  HQ_DISPATCH_X(x_dtype, HQ_DISPATCH_D(D, return launch_quant_k_static<kDT, kD>(
                                              x, x_strides, B, H, S, k_scale, scale_dtype,
                                              scale_strides, q, q_strides, st);))
}

extern "C" int hq_append_kv_static(const void* k_new, const void* v_new, int x_dtype,
                                   const int64_t k_strides[4], const int64_t v_strides[4], int B,
                                   int H, int S_new, int D, const void* k_scale, int scale_dtype,
                                   const int64_t k_scale_strides[3], int8_t* k_dst,
                                   const int64_t kq_strides[4], int8_t* v_dst,
                                   const int64_t vq_strides[4], float* v_scale_f32,
                                   uint16_t* v_scale_f16, const int64_t vs_strides[3],
                                   hq_stream_t stream) {
  if (!k_new || !v_new || !k_dst || !v_dst || !k_strides || !v_strides || !kq_strides ||
      !vq_strides || !k_scale || !k_scale_strides || B < 0 || H < 0 || S_new < 1 || S_new > 64)
    return HQ_ERR_INVALID_ARGUMENT;
  if ((v_scale_f32 || v_scale_f16) && !vs_strides) return HQ_ERR_INVALID_ARGUMENT;
  if (k_strides[3] != 1 || v_strides[3] != 1 || kq_strides[3] != 1 || vq_strides[3] != 1)
    return HQ_ERR_INVALID_ARGUMENT;
  if (!valid_dtype_x(x_dtype) || (scale_dtype != HQ_DTYPE_F32 && scale_dtype != HQ_DTYPE_F16))
    return HQ_ERR_UNSUPPORTED;
  if (B == 0 || H == 0) return HQ_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  HQ_DISPATCH_X(x_dtype, HQ_DISPATCH_D(D, return launch_append<kDT, kD>(
                                              k_new, v_new, k_strides, v_strides, B, H, S_new,
                                              k_dst, kq_strides, v_dst, vq_strides, v_scale_f32,
                                              v_scale_f16, vs_strides, nullptr, 0, st, k_scale,
                                              scale_dtype == HQ_DTYPE_F16 ? 1 : 0,
                                              k_scale_strides);))
}

extern "C" int hq_append_kv_at(const void* k_new, const void* v_new, int x_dtype,
                               const int64_t k_strides[4], const int64_t v_strides[4], int B,
                               int H, int S_new, int D, int8_t* k_cache,
                               const int64_t kq_strides[4], int8_t* v_cache,
                               const int64_t vq_strides[4], float* v_scale_f32,
                               uint16_t* v_scale_f16, const int64_t vs_strides[3], int capacity,
                               int* lens, hq_stream_t stream) {
  if (!k_new || !v_new || !k_cache || !v_cache || !k_strides || !v_strides || !kq_strides ||
      !vq_strides || !lens || !aligned(lens, 4) || B < 0 || H < 0 || S_new < 1 || S_new > 64 ||
      capacity < 0)
    return HQ_ERR_INVALID_ARGUMENT;
  if ((v_scale_f32 || v_scale_f16) && !vs_strides) return HQ_ERR_INVALID_ARGUMENT;
  if (k_strides[3] != 1 || v_strides[3] != 1 || kq_strides[3] != 1 || vq_strides[3] != 1)
    return HQ_ERR_INVALID_ARGUMENT;
  if (!valid_dtype_x(x_dtype)) return HQ_ERR_UNSUPPORTED;
  if (B == 0 || H == 0) return HQ_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  HQ_DISPATCH_X(x_dtype, HQ_DISPATCH_D(D, return launch_append<kDT, kD>(
                                              k_new, v_new, k_strides, v_strides, B, H, S_new,
                                              k_cache, kq_strides, v_cache, vq_strides, v_scale_f32,
                                              v_scale_f16, vs_strides, lens, capacity, st);))
}

extern "C" int hq_dequant(const int8_t* q, const int64_t q_strides[4], int B, int H, int S, int D,
                          const void* scale, int scale_dtype, const int64_t scale_strides[3],
                          int per_channel, void* out, int out_dtype, const int64_t out_strides[4],
                          hq_stream_t stream) {
  if (!q || !scale || !out || !q_strides || !scale_strides || !out_strides || B < 0 || H < 0 ||
      S < 0 || D < 1)
    return HQ_ERR_INVALID_ARGUMENT;
  if (q_strides[3] != 1 || out_strides[3] != 1) return HQ_ERR_INVALID_ARGUMENT;
  if ((scale_dtype != HQ_DTYPE_F32 && scale_dtype != HQ_DTYPE_F16) || !valid_dtype_x(out_dtype))
    return HQ_ERR_UNSUPPORTED;
  const int64_t n = static_cast<int64_t>(B) * H * S * D;
  if (n == 0) return HQ_OK;
  int64_t blocks = (n + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(current_sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define HQ_DQ(SDT, ODT)                                                                        \
  dequant_kernel<SDT, ODT><<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(               \
      q, q_strides[0], q_strides[1], q_strides[2], H, S, D, scale, scale_strides[0],           \
      scale_strides[1], scale_strides[2], per_channel, out, out_strides[0], out_strides[1],    \
      out_strides[2], n);                                                                      \
  return finish_launch();
  if (scale_dtype == HQ_DTYPE_F16) {
    switch (out_dtype) {
      case HQ_DTYPE_BF16: { HQ_DQ(HQ_DTYPE_F16, HQ_DTYPE_BF16) }
      case HQ_DTYPE_F16: { HQ_DQ(HQ_DTYPE_F16, HQ_DTYPE_F16) }
      default: { HQ_DQ(HQ_DTYPE_F16, HQ_DTYPE_F32) }
    }
  } else {
    switch (out_dtype) {
      case HQ_DTYPE_BF16: { HQ_DQ(HQ_DTYPE_F32, HQ_DTYPE_BF16) }
      case HQ_DTYPE_F16: { HQ_DQ(HQ_DTYPE_F32, HQ_DTYPE_F16) }
      default: { HQ_DQ(HQ_DTYPE_F32, HQ_DTYPE_F32) }
    }
  }
#undef HQ_DQ
}

extern "C" int hq_set_plan_sms(int device, int sms) {
  if (device < 0 || device >= 64 || sms < 0) return HQ_ERR_INVALID_ARGUMENT;
  hq::g_plan_sms[device].store(sms, std::memory_order_relaxed);
  return HQ_OK;
}

extern "C" int hq_read_status(const void* workspace, hq_stream_t stream) {
  if (!workspace) return HQ_ERR_INVALID_ARGUMENT;
  int v = 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return static_cast<int>(e);
  return v;
}

extern "C" int hq_column_absmax(const void* x, int x_dtype, const int64_t x_strides[4], int B,
                                int H, int S, int D, float* amax, hq_stream_t stream) {
  if (!x || !x_strides || !amax || B < 0 || H < 0 || S < 0) return HQ_ERR_INVALID_ARGUMENT;
  if (!valid_dtype_x(x_dtype)) return HQ_ERR_UNSUPPORTED;
  if (B > 65535 || H > 65535) return HQ_ERR_UNSUPPORTED;  // grid z / y limits
  if (B == 0 || H == 0) return HQ_OK;
  if (!aligned(amax, 4) || (S > 0 && !rows16(x, x_strides, x_dtype))) return HQ_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  HQ_DISPATCH_X(x_dtype, HQ_DISPATCH_D(D, return launch_column_absmax<kDT, kD>(
                                              x, x_strides, B, H, S, amax, st);))
}

extern "C" int hq_k_scale_from_amax(const float* amax, int n, float* scale_f32,
                                    uint16_t* scale_f16, hq_stream_t stream) {
  if (!amax || n < 0 || (!scale_f32 && !scale_f16)) return HQ_ERR_INVALID_ARGUMENT;
  if (n == 0) return HQ_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  k_scale_from_amax_kernel<<<(n + 255) / 256, 256, 0, st>>>(amax, n, scale_f32,
                                                            reinterpret_cast<__half*>(scale_f16));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}
