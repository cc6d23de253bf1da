// Shared pieces of the split-KV decode kernels (sm_100a): launch parameters,
// the split partial format, the in-launch split merge and the sequence-sharded
// exchange, the tensor-core and TMA helpers of the int8 / 16-bit kernels, and
// the host-side split plan, workspace layout and tensor-map encoders.  Used by
// decode_attn.cu (int8 kernel, dense twins, combine) and decode_kblock.cu
// (block-wise K layout).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstring>

#include "hq_common.cuh"

namespace hq {
int sm_count(int dev);
int current_sm_count();

namespace dec {

constexpr int kD = 128;
constexpr int kMaxPeers = 8;
// Longest wait of one block for the partials of the other ranks (a rank that
// never launches turns into HQ_ERR_DEVICE_TIMEOUT in the status word).
constexpr uint64_t kPeerWaitNs = 2000000000ull;
constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kTile = 64;
constexpr float kLog2e = 1.4426950408889634f;

template <int NREP, bool INT8>
struct Cfg {
  static constexpr int LPT = NREP == 1 ? 2 : (NREP == 2 ? 4 : 8);  // lanes per token
  static constexpr int EB = INT8 ? 1 : 2;                            // K/V element bytes
  static constexpr int CE = 16 / EB;                                 // elements per 16 B chunk
  static constexpr int NC = kD * EB / 16;                            // chunks per token row
  static constexpr int CPL = NC / LPT;                               // chunks per lane
  static constexpr int NG = kThreads / LPT;                          // token groups per block
  static constexpr int GPW = 32 / LPT;                               // groups per warp
  static constexpr int TPG = kTile / NG;                             // tokens per group per tile
  static constexpr int ROW = kD * EB;                                // bytes per token row
  static constexpr int TILE_BYTES = kTile * ROW;
  static constexpr int PAIRS = CPL * CE / 2;                         // f32x2 pairs per lane per head
  // ring depth: about the same bytes in flight per SM for int8 (3 blocks x 4
  // stages x 16 KB) and the dense twin (2 blocks x 3 stages x 32 KB)
  static constexpr int kStages = INT8 ? 4 : 3;
  static constexpr int SMEM_STAGES = kStages * 2 * TILE_BYTES;
  static constexpr int SMEM = SMEM_STAGES + NREP * kD * 4 + 2 * kStages * 8;
  static_assert(TPG >= 1 && NG * TPG == kTile, "tile must cover the token groups");
  static_assert(NG * NREP * kD * 4 <= SMEM_STAGES, "epilogue scratch must fit in the ring");
};

struct Params {
  const void* q;
  int64_t qsb, qsh;
  const char* k;
  const char* v;
  int64_t kvsb, kvsh;  // element strides of batch and head (token stride == kD)
  const void* ksc;
  const void* vsc;
  int64_t kscb, ksch, kscd, vscb, vsch, vscs;
  int Hq, Hkv, S;
  float qk_scale;  // sm_scale * log2(e)
  int q_quant;
  // programmatic dependent launch: K/V codes and scales are not written by the
  // kernel launched before this one, so they are requested before that kernel
  // completes; q, the K scales and every global write wait for it
  int overlap;
  void* out;
  int64_t osb, osh;
  float* partial_out;  // [B*Hq][kD+2] or null
  float* ws_part;      // [B*Hq][n_split][kD+2]
  int* ws_count;       // [B*Hkv] arrival tickets
  int* ws_next;        // [B*Hkv] tile claims of the dynamic schedule
  int dynamic;         // host: use the dynamic tile schedule when the V-scale layout allows
  int* ws_status;
  int n_split;
  int tiles_per_split;
  // device-resident cache length (int8 path only): when set, S above is the
  // capacity the tensor maps cover and the length is *seq_len, read at kernel
  // start; the split count stays fixed and the tiles per split follow the length
  const int* seq_len;
  int S_plan;  // host: the length the split count is planned for
  // host only: zero the workspace's status word and arrival tickets on the
  // stream just before the launch (after every argument check has passed)
  int clear_header;
  // block-wise K layout (decode_kblock.cu): tokens per K-scale block; ksc then points
  // at float32 scales [B, Hkv, n_blocks, kD] with strides (kscb, ksch, kscd = per block)
  int kblock_tokens;
  // fused append (with seq_len): the token at row *seq_len is written by this
  // launch from k_new / v_new [B, Hkv, 1, D] (q's dtype), by one extra block per
  // (b, kv head) - split n_split - 1 - which also contributes the token's
  // softmax partial; the other splits attend over rows [0, *seq_len); the last
  // block of the grid advances *seq_len
  const void* k_new;
  const void* v_new;
  int64_t knb, knh, vnb, vnh;
  // sequence-sharded exchange over peer memory (world == 0: this GPU's output only)
  int world, rank;
  char* peer[kMaxPeers];  // receive buffers of all ranks (this rank's own is local)
};

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

// 16-byte chunk -> CE/2 packed float pairs
template <int KVDT>
__device__ __forceinline__ void chunk_to_f2(const uint4& w, F2* f);
template <>
__device__ __forceinline__ void chunk_to_f2<HQ_DTYPE_I8>(const uint4& w, F2* f) {
  s8x4_to_f2x2(w.x, f[0], f[1]);
  s8x4_to_f2x2(w.y, f[2], f[3]);
  s8x4_to_f2x2(w.z, f[4], f[5]);
  s8x4_to_f2x2(w.w, f[6], f[7]);
}
template <>
__device__ __forceinline__ void chunk_to_f2<HQ_DTYPE_BF16>(const uint4& w, F2* f) {
  f[0] = bf16x2_to_f2(w.x);
  f[1] = bf16x2_to_f2(w.y);
  f[2] = bf16x2_to_f2(w.z);
  f[3] = bf16x2_to_f2(w.w);
}
template <>
__device__ __forceinline__ void chunk_to_f2<HQ_DTYPE_F16>(const uint4& w, F2* f) {
  f[0] = f16x2_to_f2(w.x);
  f[1] = f16x2_to_f2(w.y);
  f[2] = f16x2_to_f2(w.z);
  f[3] = f16x2_to_f2(w.w);
}

template <typename T>
__device__ __forceinline__ T warp_max(T v, int from) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1)
    if (o >= from) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Writes the final normalised row or the (m, l, o) partial of one q head.
template <int QDT>
__device__ __forceinline__ void emit(const Params& p, int b, int hq, int d, float M, float L,
                                     float O) {
  if (p.partial_out) {
    float* dst = p.partial_out + (static_cast<int64_t>(b) * p.Hq + hq) * (kD + 2);
    if (d == 0) {
      dst[0] = M;
      dst[1] = L;
    }
    dst[2 + d] = O;
  } else {
    using QE = Elem<QDT>;
    auto* o = reinterpret_cast<typename QE::T*>(p.out);
    o[b * p.osb + hq * p.osh + d] = QE::from_f32(L > 0.0f ? O / L : 0.0f);
  }
}

// Workspace rows of the split partials: m, l, two pad words, o[kD] (o 16-byte aligned).
constexpr int kPartRow = kD + 4;

// Receive buffer of one rank for the sequence-sharded exchange (in that rank's
// memory, zero-filled once):
//   gen   [B*Hkv]                          u32 launches completed per (b, kv head)
//   part  [2][world][B*Hq][kPartRow]       u64 words written by rank r: m, l, -, -, o[kD]
// Every word carries its value in the low half and the epoch of the launch
// that wrote it (launch count + 1, the same on every rank) in the high half,
// stored and loaded as one 64-bit access, so a receiver that reads the epoch it
// waits for has the value with it: no fence and no separate flag (the
// value-plus-flag words of NCCL's low-latency protocol, at 64-bit width).  The
// two halves alternate with the epoch parity: a rank can write epoch e + 2 into
// a half only after every rank finished epoch e + 1, hence finished reading e.
__host__ __device__ inline size_t peer_part_off(int B, int Hkv) {
  return (sizeof(unsigned) * static_cast<size_t>(B) * Hkv + 255) & ~size_t(255);
}
__host__ __device__ inline size_t peer_bytes(int B, int Hq, int Hkv, int world) {
  return peer_part_off(B, Hkv) +
         sizeof(uint64_t) * 2 * static_cast<size_t>(world) * B * Hq * kPartRow;
}

__device__ __forceinline__ void st_word(uint64_t* a, float v, unsigned epoch) {
  const uint64_t w = (static_cast<uint64_t>(epoch) << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
}

// Bounded wait for the word at `a` to carry `epoch`; t0 is the time of this
// thread's first miss (0 before it), so one thread waits kPeerWaitNs at most.
__device__ __forceinline__ bool wait_word(const uint64_t* a, unsigned epoch, float& v,
                                          uint64_t& t0) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
    if (static_cast<unsigned>(w >> 32) == epoch) {
      v = __uint_as_float(static_cast<unsigned>(w));
      return true;
    }
    if (t0 == 0) {
      t0 = global_ns();
    } else if ((i & 15) == 15 && global_ns() - t0 > kPeerWaitNs) {
      return false;
    }
    __nanosleep(32);
  }
  return false;
}

// This block's launch count for (b, kvh) in a sequence-sharded launch (read at
// the start of the kernel, so its latency hides behind the token loop).
__device__ __forceinline__ unsigned peer_gen(const Params& p, int b, int kvh) {
  return p.world > 1 ? __ldcg(reinterpret_cast<const unsigned*>(p.peer[p.rank]) + b * p.Hkv + kvh)
                     : 0u;
}

// Final (M, L, O) of the NREP q heads of (b, kvh), channel d per thread: the
// output (or partial) of this GPU, or - when the sequence is sharded over
// several ranks - this rank's (m, l, o) words stored into every other rank's
// receive buffer, then the words of ranks 0 .. world-1 merged in rank order as
// they arrive (the same arithmetic, so the same output, on every rank).
// Called by all threads of one block; gen0 = peer_gen(p, b, kvh).
template <int NREP, int QDT>
__device__ __forceinline__ void finish_heads(const Params& p, int b, int kvh, int d,
                                             const float (&M)[NREP], const float (&L)[NREP],
                                             const float (&O)[NREP], unsigned gen0) {
  if (p.world <= 1) {
#pragma unroll
    for (int r = 0; r < NREP; ++r) emit<QDT>(p, b, kvh * NREP + r, d, M[r], L[r], O[r]);
    return;
  }
  const int B = gridDim.z, W = p.world;
  const size_t poff = peer_part_off(B, p.Hkv);
  const unsigned epoch = gen0 + 1u;
  const size_t half = static_cast<size_t>(epoch & 1u) * W;
  const size_t head0 = static_cast<size_t>(b) * p.Hq + kvh * NREP;
  // 1. this rank's words into slot [half][rank] of the other ranks' buffers
  for (int w = 0; w < W; ++w) {
    if (w == p.rank) continue;
    uint64_t* row = reinterpret_cast<uint64_t*>(p.peer[w] + poff) +
                    ((half + p.rank) * B * p.Hq + head0) * kPartRow;
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      if (d == 0) {
        st_word(row + r * kPartRow, M[r], epoch);
        st_word(row + r * kPartRow + 1, L[r], epoch);
      }
      st_word(row + r * kPartRow + 4 + d, O[r], epoch);
    }
  }
  // 2. online merge over ranks 0 .. W-1 (bounded waits for the remote words)
  const uint64_t* base = reinterpret_cast<const uint64_t*>(p.peer[p.rank] + poff) +
                         half * B * p.Hq * kPartRow;
  float Mt[NREP], Lt[NREP], Ot[NREP];
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    Mt[r] = -INFINITY;
    Lt[r] = 0.0f;
    Ot[r] = 0.0f;
  }
  bool ok = true;
  uint64_t t0 = 0;
  for (int w = 0; w < W && ok; ++w) {
    const uint64_t* row = base + (static_cast<size_t>(w) * B * p.Hq + head0) * kPartRow;
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      float m = M[r], l = L[r], o = O[r];
      if (w != p.rank) {
        ok = ok && wait_word(row + r * kPartRow, epoch, m, t0) &&
             wait_word(row + r * kPartRow + 1, epoch, l, t0) &&
             wait_word(row + r * kPartRow + 4 + d, epoch, o, t0);
      }
      const float mn = fmaxf(Mt[r], m);
      const float a = Mt[r] == -INFINITY ? 0.0f : exp2f(Mt[r] - mn);
      const float f = m == -INFINITY ? 0.0f : exp2f(m - mn);
      Lt[r] = Lt[r] * a + l * f;
      Ot[r] = Ot[r] * a + o * f;
      Mt[r] = mn;
    }
  }
  if (__syncthreads_or(!ok)) {  // gave up: status word set, no output
    if (d == 0) report_error(p.ws_status, HQ_ERR_DEVICE_TIMEOUT);
    return;
  }
#pragma unroll
  for (int r = 0; r < NREP; ++r) emit<QDT>(p, b, kvh * NREP + r, d, Mt[r], Lt[r], Ot[r]);
  if (d == 0) reinterpret_cast<unsigned*>(p.peer[p.rank])[b * p.Hkv + kvh] = epoch;
}

// Publishes one split's (m, l, o) for q head hq; thread d writes o[d].
__device__ __forceinline__ void publish_split(const Params& p, int b, int hq, int split, int d,
                                              float M, float L, float O) {
  float* dst = p.ws_part + ((static_cast<int64_t>(b) * p.Hq + hq) * p.n_split + split) * kPartRow;
  if (d == 0) {
    dst[0] = M;
    dst[1] = L;
  }
  dst[4 + d] = O;
}

// Arrival ticket of a split: adds 1 to *ctr and returns the old count, as one
// acquire-release atomic.  Called by one thread after a block barrier: the
// release makes the partial that every thread of the block stored before that
// barrier visible first; the acquire makes the partials of the splits counted
// earlier visible to the whole block after the barrier that follows.
__device__ __forceinline__ int ticket_add(int* ctr) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(ctr) : "memory");
  return old;
}

// Run by the last block of (b, kvh) to arrive: merges the n_split partials of
// its NREP q heads and emits them.  The rows of one head are contiguous, so the
// block copies them into shared memory in one round trip to L2: one bulk copy
// per head completing on the mbarrier `bar` when the kernel provides one (the
// int8 kernel), else 16-byte cp.async.  With at most 64 rows per head (every
// one-wave plan) warp r then reduces head r's row maxima, weights and sum with
// shuffles, and after one block barrier thread d folds channel d of every row.
// Longer merges reduce the row maxima, write one weight per row, and fold the
// rows with warp w taking rows w, w + 4, ... and lane l channels 4 l .. 4 l + 3
// (16-byte shared loads), a last pass adding the 4 warps; rows beyond the
// scratch capacity are merged in further chunks (online rescaling).  scratch:
// 16-byte aligned, scratch_floats floats.
template <int NREP, int QDT>
__device__ __forceinline__ void merge_splits(const Params& p, int b, int kvh, float* scratch,
                                             int scratch_floats, unsigned gen0,
                                             uint64_t* bar = nullptr) {
  constexpr int kRowVec = kPartRow / 4;  // 16-byte pieces per partial row
  __shared__ float s_red[kWarps][NREP];
  __shared__ float s_l[kWarps][NREP];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = p.n_split;
  const float* src = p.ws_part + (static_cast<int64_t>(b) * p.Hq + kvh * NREP) * n * kPartRow;
  float* wsum = scratch;                          // [kWarps][NREP][kD] per-warp sums
  float* rows_base = scratch + kWarps * NREP * kD;
  const int per_chunk = max(1, (scratch_floats - kWarps * NREP * kD) / (NREP * (kPartRow + 1)));
  float M[NREP], L[NREP], O[NREP];
  if (n <= 64 && NREP * (n * kPartRow + 64) <= scratch_floats) {
    // Up to 64 rows per head (every plan with one wave of blocks): all rows in
    // one cp.async round trip, then warp r alone reduces head r's row maxima,
    // weights and sum (two rows per lane, shuffles only), and after one block
    // barrier thread d folds channel d of every row with those weights.
    float* wbuf = scratch + NREP * n * kPartRow;  // [NREP][64] row weights
    if (bar) {
      // one bulk copy per head (its rows are contiguous), completing on `bar`
      // (initialised by the kernel, used once per launch: phase 0)
      if (tid == 0) {
        asm volatile("fence.proxy.async.global;" ::: "memory");  // acquired partials -> async proxy
        mbar_arrive_expect_tx(bar, NREP * n * kPartRow * 4);
#pragma unroll
        for (int r = 0; r < NREP; ++r)
          bulk_g2s(scratch + r * n * kPartRow, src + static_cast<int64_t>(r) * n * kPartRow,
                   n * kPartRow * 4, bar);
      }
      if (__syncthreads_or(!mbar_wait(bar, 0))) {
        if (tid == 0) report_error(p.ws_status, HQ_ERR_DEVICE_TIMEOUT);
        return;
      }
    } else {
#pragma unroll
      for (int r = 0; r < NREP; ++r) {
        float* dst = scratch + r * n * kPartRow;
        const float* from = src + static_cast<int64_t>(r) * n * kPartRow;
        for (int i = tid; i < n * kRowVec; i += kThreads) cp_async16(dst + 4 * i, from + 4 * i);
      }
      cp_async_commit();
      cp_async_wait<0>();
      __syncthreads();
    }
    if (warp < NREP) {
      const float* rows = scratch + warp * n * kPartRow;
      const bool h0 = lane < n, h1 = lane + 32 < n;
      const float m0 = h0 ? rows[lane * kPartRow] : -INFINITY;
      const float m1 = h1 ? rows[(lane + 32) * kPartRow] : -INFINITY;
      const float mx = warp_max(fmaxf(m0, m1), 1);
      const float w0 = m0 == -INFINITY ? 0.0f : exp2f(m0 - mx);
      const float w1 = m1 == -INFINITY ? 0.0f : exp2f(m1 - mx);
      float l = (h0 ? w0 * rows[lane * kPartRow + 1] : 0.0f) +
                (h1 ? w1 * rows[(lane + 32) * kPartRow + 1] : 0.0f);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      wbuf[warp * 64 + lane] = w0;
      wbuf[warp * 64 + lane + 32] = w1;
      if (lane == 0) {
        s_red[0][warp] = mx;
        s_l[0][warp] = l;
      }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      const float* rows = scratch + r * n * kPartRow + 4 + tid;
      const float* w = wbuf + r * 64;
      float o0 = 0.0f, o1 = 0.0f;
      int s = 0;
      for (; s + 1 < n; s += 2) {
        o0 += w[s] * rows[s * kPartRow];
        o1 += w[s + 1] * rows[(s + 1) * kPartRow];
      }
      if (s < n) o0 += w[s] * rows[s * kPartRow];
      M[r] = s_red[0][r];
      L[r] = s_l[0][r];
      O[r] = o0 + o1;
    }
    if (tid == 0) p.ws_count[b * p.Hkv + kvh] = 0;  // ready for the next launch
    finish_heads<NREP, QDT>(p, b, kvh, tid, M, L, O, gen0);
    return;
  }
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    M[r] = -INFINITY;
    L[r] = 0.0f;
    O[r] = 0.0f;
  }
  for (int s0 = 0; s0 < n; s0 += per_chunk) {
    const int cs = min(per_chunk, n - s0);
    float* wbuf = rows_base + NREP * cs * kPartRow;  // [NREP][cs] row weights
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      float* dst = rows_base + r * cs * kPartRow;
      const float* from = src + (static_cast<int64_t>(r) * n + s0) * kPartRow;
      for (int i = tid; i < cs * kRowVec; i += kThreads) cp_async16(dst + 4 * i, from + 4 * i);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    float Mn[NREP];
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      const float* rows = rows_base + r * cs * kPartRow;
      float m = -INFINITY;
      for (int s = tid; s < cs; s += kThreads) m = fmaxf(m, rows[s * kPartRow]);
      m = warp_max(m, 1);
      if (lane == 0) s_red[warp][r] = m;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      float m = s_red[0][r];
#pragma unroll
      for (int w = 1; w < kWarps; ++w) m = fmaxf(m, s_red[w][r]);
      Mn[r] = fmaxf(M[r], m);
      const float* rows = rows_base + r * cs * kPartRow;
      for (int s = tid; s < cs; s += kThreads) {
        const float ms = rows[s * kPartRow];
        wbuf[r * cs + s] = ms == -INFINITY ? 0.0f : exp2f(ms - Mn[r]);
      }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      const float* rows = rows_base + r * cs * kPartRow;
      const float* w = wbuf + r * cs;
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      float l = 0.0f;
      for (int s = warp; s < cs; s += kWarps) {
        const float ws = w[s];
        const float4 v = reinterpret_cast<const float4*>(rows + s * kPartRow + 4)[lane];
        acc.x += ws * v.x;
        acc.y += ws * v.y;
        acc.z += ws * v.z;
        acc.w += ws * v.w;
        l += ws * rows[s * kPartRow + 1];
      }
      reinterpret_cast<float4*>(wsum + (warp * NREP + r) * kD)[lane] = acc;
      if (lane == 0) s_l[warp][r] = l;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      if (Mn[r] == -INFINITY) continue;  // no token seen yet
      float o = 0.0f, l = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        o += wsum[(w * NREP + r) * kD + tid];
        l += s_l[w][r];
      }
      const float a = M[r] == -INFINITY ? 0.0f : exp2f(M[r] - Mn[r]);
      L[r] = L[r] * a + l;
      O[r] = O[r] * a + o;
      M[r] = Mn[r];
    }
    __syncthreads();  // scratch, s_red and s_l are reused by the next chunk
  }
  if (tid == 0) p.ws_count[b * p.Hkv + kvh] = 0;  // ready for the next launch
  finish_heads<NREP, QDT>(p, b, kvh, tid, M, L, O, gen0);
}

namespace mmak {

constexpr int kTileT = 128;                // tokens per tile
constexpr int kTileB = kTileT * kD;        // 16 KB per K or V tile
constexpr int kStagesM = 3;
constexpr int kStatic = kStagesM + 1;      // dynamic schedule: fixed tiles per block before claims
constexpr float kLimbMax = 8355711.0f;     // 127 * (65536 + 256 + 1): largest |x| of 3 int8 digits


__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// K / V tiles are read once per decode step: they go through L2 as evict-first
// so that they do not push out what every launch reuses (code, q, scales,
// split partials).
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y,
                                            int z, int w, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar)),
      "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y,
                                            int z, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// balanced base-256 digits of x in [-kLimbMax, kLimbMax]: x = 65536 a + 256 b + c,
// each digit in [-128, 127] (a in [-127, 127])
__device__ __forceinline__ void limbs24(int x, int& a, int& b, int& c) {
  c = ((x + 128) & 255) - 128;
  const int x1 = (x - c) >> 8;
  b = ((x1 + 128) & 255) - 128;
  a = (x1 - b) >> 8;
}
__device__ __forceinline__ uint32_t limb_byte(int x, int which) {
  int a, b, c;
  limbs24(x, a, b, c);
  return static_cast<uint32_t>(which == 0 ? a : which == 1 ? b : c) & 0xffu;
}
// byte offset of (row, 16-byte chunk) in a 128-byte-row tile stored with 128B swizzle
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}
// logical MMA k index (0..31) of the warp-local token p (0..31) in the PV product
__device__ __forceinline__ int pv_k(int p) {
  const int th = p >> 4, w = p & 15;
  return 16 * th + 4 * ((w & 7) >> 1) + (w & 1) + 2 * (w >> 3);
}

}  // namespace mmak

// ------------------------------------------------------------------ host side
struct Plan {
  int n_split;
  int tiles_per_split;
};

// Upper bound on splits per (batch, kv head), shared by the workspace query
// and the launch: enough to give every SM up to 8 blocks.
inline int max_splits(int units, int tiles, int sms) {
  if (tiles <= 0) return 1;
  int m = (8 * sms + units - 1) / units;
  if (m < 1) m = 1;
  return m < tiles ? m : tiles;
}

// Picks the tile count per split that minimises (waves x tiles per block).
// one_wave: only plans whose grid fits the resident slots (units <= slots).
inline Plan make_plan(int units, int S, int slots, int sms, int tile = kTile,
                      bool one_wave = false) {
  const int tiles = (S + tile - 1) / tile;
  if (tiles <= 0) return {1, 1};
  int cap = max_splits(units, tiles, sms);
  if (one_wave && cap > slots / units) cap = slots / units;
  Plan best{1, tiles};
  double best_cost = 1e30;
  for (int c = 1; c <= tiles; ++c) {
    const int n = (tiles + c - 1) / c;
    if (n > cap) continue;
    if (c > 1 && (tiles + c - 2) / (c - 1) == n) continue;  // same split count, fewer tiles
    const int64_t ctas = static_cast<int64_t>(units) * n;
    const int64_t waves = (ctas + slots - 1) / slots;
    // one extra tile of fixed cost per block (prologue, epilogue, combine share)
    const double cost = static_cast<double>(waves) * (c + 1.0) + (n > 1 ? 0.5 : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = {n, c};
    }
  }
  return best;
}

inline size_t align256(size_t n) { return (n + 255) & ~size_t(255); }
// arrival tickets [B*Hkv] then the dynamic schedule's tile claims [B*Hkv],
// after the 256-byte header
inline size_t tickets_bytes(int B, int Hkv) {
  return align256(2 * sizeof(int) * static_cast<size_t>(B) * Hkv);
}

inline size_t workspace_bytes(int B, int Hq, int Hkv, int S, int sms) {
  const int units = B * Hkv;
  const int tiles = (S + kTile - 1) / kTile;
  const int ms = max_splits(units > 0 ? units : 1, tiles, sms);
  return 256 + tickets_bytes(B, Hkv) +
         sizeof(float) * static_cast<size_t>(B) * Hq * ms * kPartRow;
}

// ---- tensor maps for the int8 kernel (driver entry point, no libcuda link)
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::atomic<void*> cached{nullptr};
  void* f = cached.load(std::memory_order_acquire);
  if (!f) {
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) !=
            cudaSuccess ||
        qr != cudaDriverEntryPointSuccess || !f)
      return nullptr;
    cached.store(f, std::memory_order_release);
  }
  return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
}

// int8 [B, Hkv, S, 128] with byte strides (sb, sh, 128): boxes of 128 tokens x 128 bytes,
// 128-byte swizzle, zero fill past S.
inline int encode_kv_map(CUtensorMap* m, const void* base, int64_t sb, int64_t sh, int S, int Hkv,
                         int B) {
  auto enc = encode_fn();
  if (!enc) return HQ_ERR_UNSUPPORTED;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(S > 0 ? S : 1),
                        static_cast<cuuint64_t>(Hkv), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(sh),
                           static_cast<cuuint64_t>(sb)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(kD), static_cast<cuuint32_t>(mmak::kTileT), 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? HQ_OK : HQ_ERR_INVALID_ARGUMENT;
}

// V scales [B, Hkv, S] with element strides (sb, sh, 1) for the dynamic schedule's
// third tensor map: boxes of 128 tokens, zero fill past S.  Needs a token stride
// of 1, a 16-byte aligned base and head / batch strides of multiples of 16 bytes.
inline bool vs_map_ok(const void* base, int esz, int64_t sb, int64_t sh, int64_t ss) {
  return base && ss == 1 && reinterpret_cast<uintptr_t>(base) % 16 == 0 && (sh * esz) % 16 == 0 &&
         (sb * esz) % 16 == 0;
}
inline int encode_vs_map(CUtensorMap* m, const void* base, int esz, int64_t sb, int64_t sh, int S,
                         int Hkv, int B) {
  auto enc = encode_fn();
  if (!enc) return HQ_ERR_UNSUPPORTED;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(S > 0 ? S : 1), static_cast<cuuint64_t>(Hkv),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(sh * esz), static_cast<cuuint64_t>(sb * esz)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(mmak::kTileT), 1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, esz == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                   3, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? HQ_OK : HQ_ERR_INVALID_ARGUMENT;
}

}  // namespace dec
}  // namespace hq
