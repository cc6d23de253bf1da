// Block-wise per-channel K layout (opt-in) for sm_100a: quantize-on-write and
// split-KV decode attention.
//
// The reference quantizes K per channel over the whole prefill and then keeps
// that first scale for every later append (tests/qwen_kvcache_full.py:54), so a
// decoded token whose |K| exceeds the prefill's column maximum is clipped to
// +-127.  Its roadmap names block-wise per-channel K as the production answer
// (README.md:141).  Here the sequence is cut into blocks of BT tokens (64, 128
// or 256); each (block, channel) gets its own scale by the reference's
// quantizer rule (quantize_int8, reference/page_attention_int8_pytorch.py:23-30:
// RN(max(amax, 1e-8) / 127), codes clamp(rint(x / scale), -127, 127)) applied to
// the block's tokens.  V stays per token (the reference's rule, reduce over D).
//
// The invariant: after any sequence of writes, the codes and scales equal a
// bulk block-wise quantization of every token written so far (the last block
// over the tokens it holds).  To keep it across single-token appends the
// originals of the open (last, incomplete) block are kept in a small tail
// buffer [B, H, BT, D]; when a new token raises a channel's scale, that
// channel's earlier codes in the block are re-coded from the originals.  RN is
// monotone, so max(old scale, RN(max|new| / 127)) is exactly the scale of the
// block's full column maximum: the stored scale is all the state the rule needs.
//
// Decode: a CUDA-core split-KV kernel.  The K scale varies along the contracted
// dimension per block, so it is folded into q per block (q' = q * s_blk *
// sm_scale * log2 e, in shared memory, once per 128-token tile); one lane per
// token forms q' . codes with packed f32x2 FMAs over codes unpacked by byte
// permutes; an fp32 online softmax per warp; one lane per 4 (D = 128) or 2
// (D = 64) channels accumulates p * v_scale * codes; the 4 warps merge in shared
// memory and the splits merge in the last block to finish (arrival ticket).
#include <algorithm>
#include <atomic>
#include <cmath>

#include "hq_common.cuh"

namespace hq {

int current_sm_count();
int kblock_decode_mma(const void* q, int q_dtype, const int64_t q_strides[3],
                      const int8_t* k_cache, const int64_t kq_strides[3], const float* k_scale,
                      const int64_t ks_strides[3], const int8_t* v_cache,
                      const int64_t vq_strides[3], const void* v_scale, int scale_dtype,
                      const int64_t vs_strides[3], int B, int Hq, int Hkv, int S, int D,
                      int block_tokens, float sm_scale, void* out, const int64_t out_strides[3],
                      void* workspace, size_t workspace_bytes, hq_stream_t stream,
                      const int* seq_len = nullptr, int S_plan = 0);
size_t kblock_decode_mma_workspace_bytes(int B, int Hq, int Hkv, int S, int D);

namespace kb {

constexpr int kWriteThreads = 256;
constexpr int kDecThreads = 128;   // 4 warps: one 32-token chunk each per 128-token tile
constexpr int kTile = 128;
constexpr int kMaxSplit = 128;     // splits per (sequence, kv head)

struct WriteParams {
  const void* k;                   // new K rows [B, H, S_new, D] (element strides)
  int64_t ksb, ksh, kss;
  const void* v;                   // new V rows (optional)
  int64_t vsb, vsh, vss;
  int8_t* kq;                      // K codes, row 0 of the [B, H, capacity, D] buffer
  int64_t kqb, kqh, kqs;
  float* ksc;                      // K block scales [B, H, n_blocks, D]
  int64_t kscb, ksch, kscx;
  void* kt;                        // K tail [B, H, BT, D]: originals of the open block
  int64_t ktb, kth, kts;
  int8_t* vq;                      // V codes, row 0
  int64_t vqb, vqh, vqs;
  float* vs32;                     // V scales, row 0 (one of the two, or none)
  __half* vs16;
  int64_t vssb, vssh, vsss;
  int D, BT, pos, S_new, blk0;
  int tail_mode;                   // 0: write the tail here, 1: leave it, 2: only write it
  // device-resident length {length, ticket, status, -} (one-token writes): the token
  // goes to row lens[0], the grid's last block advances it; a full cache (capacity
  // cap) writes nothing and reports HQ_ERR_INVALID_ARGUMENT in lens[2]
  int* lens;
  int cap;
};

template <int DT>
__device__ __forceinline__ void load_pair(const typename Elem<DT>::T* p, float& a, float& b) {
  a = Elem<DT>::to_f32(p[0]);
  b = Elem<DT>::to_f32(p[1]);
}

__device__ __forceinline__ void store_pair(int8_t* dst, int c0, int c1) {
  *reinterpret_cast<uint16_t*>(dst) =
      static_cast<uint16_t>((static_cast<uint32_t>(c0) & 0xffu) | ((static_cast<uint32_t>(c1) & 0xffu) << 8));
}

// Code of a 16-bit input x for the scale s = RN(m / 127) of a 16-bit maximum m >= |x|
// (r = RN(1 / s)): the quotient x * r with one FMA residual correction, rounded half to
// even by adding 1.5 * 2^23 - equal to rint(RN(x / s)) for every bf16 and fp16 such x,
// so no divide and no branch.  float32 inputs keep Quantizer::code.
template <int DT>
__device__ __forceinline__ int code_of(const Quantizer& q, float x) {
  if constexpr (DT == HQ_DTYPE_F32) {
    return q.code(x);
  } else {
    const float q0 = x * q.rcp;
    const float q1 = __fmaf_rn(__fmaf_rn(q0, -q.scale, x), q.rcp, q0);
    return __float_as_int(q1 + 12582912.0f) - 0x4B400000;
  }
}

__device__ __forceinline__ Quantizer quantizer_of_scale(float s) {
  Quantizer q;
  q.scale = s;
  q.rcp = __frcp_rn(s);
  return q;
}

// grid (blocks touched, H, B); thread (pair j, group g) owns channels 2j, 2j+1
// and the block's rows g, g + G, ...
template <int DT, int D>
__global__ void __launch_bounds__(kWriteThreads) kblock_write_kernel(WriteParams p) {
  using E = Elem<DT>;
  using T = typename E::T;
  __shared__ float smax[2 * kWriteThreads];
  __shared__ int s_pos;
  const int tid = threadIdx.x;
  constexpr int P = D / 2, G = kWriteThreads / P;
  const int j = tid % P, g = tid / P;
  const int c0 = 2 * j;
  int pos = p.pos, blk = p.blk0 + blockIdx.x;
  if (p.lens) {
    if (tid == 0) s_pos = __ldcg(p.lens);
    __syncthreads();
    pos = s_pos;
    if (pos < 0 || pos + p.S_new > p.cap) {  // full cache: nothing is written
      if (tid == 0) report_error(p.lens + 2, HQ_ERR_INVALID_ARGUMENT);
      return;
    }
    blk = pos / p.BT + blockIdx.x;
  }
  const int64_t b = blockIdx.z, h = blockIdx.y;
  const int r0 = blk * p.BT;
  const int lo = max(r0, pos), hi = min(r0 + p.BT, pos + p.S_new);  // new rows here
  const int n_old = lo - r0;                                             // rows already held
  const bool keep_tail = hi < r0 + p.BT;   // the block stays open: its originals are kept
  const T* kin = reinterpret_cast<const T*>(p.k) + b * p.ksb + h * p.ksh;
  T* tail = reinterpret_cast<T*>(p.kt) + b * p.ktb + h * p.kth;

  if (p.tail_mode == 2) {
    if (keep_tail)
      for (int r = lo + g; r < hi; r += G) {
        const T* x = kin + static_cast<int64_t>(r - pos) * p.kss + c0;
        T* t = tail + static_cast<int64_t>(r - r0) * p.kts + c0;
        t[0] = x[0];
        t[1] = x[1];
      }
    return;
  }

  // pass 1: column maxima over the new rows
  float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 8
  for (int r = lo + g; r < hi; r += G) {
    float x0, x1;
    load_pair<DT>(kin + static_cast<int64_t>(r - pos) * p.kss + c0, x0, x1);
    a0 = fmaxf(a0, fabsf(x0));
    a1 = fmaxf(a1, fabsf(x1));
  }
  smax[g * D + c0] = a0;
  smax[g * D + c0 + 1] = a1;
  // the block's stored scales, read before the barrier: group 0 overwrites them below
  float* sc = p.ksc + b * p.kscb + h * p.ksch + static_cast<int64_t>(blk) * p.kscx + c0;
  float o0 = 0.0f, o1 = 0.0f;
  if (n_old > 0) {
    o0 = sc[0];
    o1 = sc[1];
  }
  __syncthreads();
  a0 = smax[c0];
  a1 = smax[c0 + 1];
  for (int gg = 1; gg < G; ++gg) {
    a0 = fmaxf(a0, smax[gg * D + c0]);
    a1 = fmaxf(a1, smax[gg * D + c0 + 1]);
  }
  float s0 = Quantizer::from_amax(a0).scale, s1 = Quantizer::from_amax(a1).scale;
  bool grew = false;
  if (n_old > 0) {
    grew = s0 > o0 || s1 > o1;
    s0 = fmaxf(s0, o0);
    s1 = fmaxf(s1, o1);
  }
  const Quantizer q0 = quantizer_of_scale(s0), q1 = quantizer_of_scale(s1);
  int8_t* kq = p.kq + b * p.kqb + h * p.kqh + c0;

  // pass 2: codes of the new rows (and their originals while the block is open)
#pragma unroll 4
  for (int r = lo + g; r < hi; r += G) {
    const T* xp = kin + static_cast<int64_t>(r - pos) * p.kss + c0;
    float x0, x1;
    load_pair<DT>(xp, x0, x1);
    store_pair(kq + static_cast<int64_t>(r) * p.kqs, code_of<DT>(q0, x0), code_of<DT>(q1, x1));
    if (keep_tail && p.tail_mode == 0) {
      T* t = tail + static_cast<int64_t>(r - r0) * p.kts + c0;
      t[0] = xp[0];
      t[1] = xp[1];
    }
  }
  // earlier rows of the block: re-coded from their originals when a scale grew
  // (a channel whose scale did not change gets its stored code again)
  if (grew) {
#pragma unroll 8
    for (int r = r0 + g; r < lo; r += G) {
      float x0, x1;
      load_pair<DT>(tail + static_cast<int64_t>(r - r0) * p.kts + c0, x0, x1);
      store_pair(kq + static_cast<int64_t>(r) * p.kqs, code_of<DT>(q0, x0), code_of<DT>(q1, x1));
    }
  }
  if (g == 0) {
    sc[0] = s0;
    sc[1] = s1;
  }

  // V per token over D: warp w takes rows lo + w, lo + w + 8, ..., four rows per round
  if (p.v) {
    constexpr int kN = D / 32, kR = 4, kWarps = kWriteThreads / 32;
    const int w = tid >> 5, lane = tid & 31;
    const T* vin = reinterpret_cast<const T*>(p.v) + b * p.vsb + h * p.vsh;
    int8_t* vq = p.vq + b * p.vqb + h * p.vqh;
    for (int rb = lo + w; rb < hi; rb += kR * kWarps) {
      float x[kR][kN], m[kR];
#pragma unroll
      for (int u = 0; u < kR; ++u) {
        const int r = rb + u * kWarps;
        m[u] = 0.0f;
#pragma unroll
        for (int i = 0; i < kN; ++i) {
          x[u][i] = r < hi ? E::to_f32(vin[static_cast<int64_t>(r - pos) * p.vss + lane + 32 * i]) : 0.0f;
          m[u] = fmaxf(m[u], fabsf(x[u][i]));
        }
      }
#pragma unroll
      for (int u = 0; u < kR; ++u)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m[u] = fmaxf(m[u], __shfl_xor_sync(0xffffffffu, m[u], off));
#pragma unroll
      for (int u = 0; u < kR; ++u) {
        const int r = rb + u * kWarps;
        if (r >= hi) break;
        const Quantizer qv = DT == HQ_DTYPE_F32 ? Quantizer::from_amax(m[u]) : Quantizer::from_amax16(m[u]);
        int8_t* dst = vq + static_cast<int64_t>(r) * p.vqs;
#pragma unroll
        for (int i = 0; i < kN; ++i) dst[lane + 32 * i] = static_cast<int8_t>(code_of<DT>(qv, x[u][i]));
        if (lane == 0) {
          const int64_t so = b * p.vssb + h * p.vssh + static_cast<int64_t>(r) * p.vsss;
          if (p.vs32) p.vs32[so] = qv.scale;
          if (p.vs16) p.vs16[so] = __float2half_rn(qv.scale);
        }
      }
    }
  }
  if (p.lens) {
    // every block has read lens[0]; the last one to arrive advances it
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      const int total = static_cast<int>(gridDim.x * gridDim.y * gridDim.z);
      if (atomicAdd(p.lens + 1, 1) == total - 1) {
        p.lens[1] = 0;
        p.lens[0] = pos + p.S_new;
      }
    }
  }
}

// ------------------------------------------------------------------ decode
struct DecParams {
  const void* q;                    // [B, Hq, D] of q_dtype, d contiguous
  int64_t qsb, qsh;
  int q_dtype;
  const int8_t* kq;
  int64_t kqb, kqh, kqs;
  const float* ksc;
  int64_t kscb, ksch, kscx;
  const int8_t* vq;
  int64_t vqb, vqh, vqs;
  const void* vs;
  int vs_f16;
  int64_t vssb, vssh, vsss;
  void* out;                        // [B, Hq, D] of q_dtype, d contiguous
  int64_t osb, osh;
  int Hkv, S, BT, tps, n_split;
  float qscale;                     // sm_scale * log2(e)
  float* ws_ml;                     // [B, Hq, n_split, 2] (m, l)
  float* ws_o;                      // [B, Hq, n_split, D]
  int* ws_cnt;                      // [B, Hkv] arrival tickets (zero between launches)
};

__device__ __forceinline__ float load_any(const void* p, int64_t i, int dt) {
  if (dt == HQ_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == HQ_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_any(void* p, int64_t i, int dt, float x) {
  if (dt == HQ_DTYPE_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else if (dt == HQ_DTYPE_F16)
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(x);
  else
    reinterpret_cast<float*>(p)[i] = x;
}

__device__ __forceinline__ float f2_sum(F2 x) {
  float a, b;
  f2_split(x, a, b);
  return a + b;
}

// Dynamic shared memory: a 2-stage ring per warp holding its 32-token chunk of
// K (rows XOR-swizzled by 16-byte chunk so one-lane-per-token reads are
// conflict-free) and V, then q, the double-buffered q' and the merge scratch.
template <int NR, int D>
struct DecLayout {
  static constexpr int kStages = 2;
  static constexpr int kStageB = 2 * 32 * D;                // K + V of one chunk
  static constexpr int kRingB = 4 * kStages * kStageB;
  static constexpr int kQf = NR * D;                         // floats
  static constexpr int kQp = 2 * 2 * NR * D;                 // [buffer][block of tile][NR*D]
  static constexpr int kPv = 4 * 32 * NR;
  static constexpr int kBytes = kRingB + 4 * (kQf + kQp + kPv + 2 * 4 * NR) + 16;
  static_assert(4 * NR * D * 4 <= kRingB && NR * kMaxSplit * 4 <= kRingB,
                "merge scratch aliases the ring");
};

template <int NR, int D>
__global__ void __launch_bounds__(kDecThreads) kblock_decode_kernel(DecParams p) {
  using L = DecLayout<NR, D>;
  constexpr int DPL = D / 32;                         // V channels per lane
  constexpr int NF = DPL / 2;                         // ... as f32x2 pairs
  constexpr int CPR = D / 16;                         // 16-byte chunks per row
  constexpr int kQpPer = (2 * NR * D + kDecThreads - 1) / kDecThreads;
  extern __shared__ __align__(128) char smem[];
  float* qf = reinterpret_cast<float*>(smem + L::kRingB);
  float* qp = qf + L::kQf;
  float* pvb = qp + L::kQp;
  float* wmb = pvb + L::kPv;
  float* wlb = wmb + 4 * NR;
  int* last = reinterpret_cast<int*>(wlb + 4 * NR);
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int hk = blockIdx.x, split = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int Hq = p.Hkv * NR;
  char* ring = smem + w * L::kStages * L::kStageB;
  for (int i = tid; i < NR * D; i += kDecThreads) {
    const int hh = i / D, d = i % D;
    qf[i] = load_any(p.q, b * p.qsb + static_cast<int64_t>(hk * NR + hh) * p.qsh + d, p.q_dtype) *
            p.qscale;
  }
  const int n_tiles = (p.S + kTile - 1) / kTile;
  const int t_begin = split * p.tps, t_end = min(n_tiles, t_begin + p.tps);
  const int8_t* kbase = p.kq + b * p.kqb + hk * p.kqh;
  const int8_t* vbase = p.vq + b * p.vqb + hk * p.vqh;
  const float* sbase = p.ksc + b * p.kscb + hk * p.ksch;
  const int64_t vsbase = b * p.vssb + hk * p.vssh;
  const int nbq = p.BT < kTile ? kTile / p.BT : 1;   // scale blocks per tile
  const int nqp = nbq * NR * D;

  // the K scales of a tile's blocks (into registers) and q' = q * scale (into smem)
  auto load_ks = [&](int tile, float* r) {
    const int blkA = tile * kTile / p.BT;
#pragma unroll
    for (int k = 0; k < kQpPer; ++k) {
      const int i = tid + k * kDecThreads;
      r[k] = 0.0f;
      if (i < nqp) {
        const int bi = i / (NR * D), d = i % D;
        const int blk = blkA + bi;
        if (blk * p.BT < p.S) r[k] = __ldg(sbase + static_cast<int64_t>(blk) * p.kscx + d);
      }
    }
  };
  auto store_qp = [&](int buf, const float* r) {
    float* dst = qp + buf * 2 * NR * D;
#pragma unroll
    for (int k = 0; k < kQpPer; ++k) {
      const int i = tid + k * kDecThreads;
      if (i < nqp) dst[i] = qf[i % (NR * D)] * r[k];
    }
  };
  // this warp's chunk of a tile: K rows swizzled, V rows plain, one cp.async per 16 bytes
  auto issue = [&](int tile, int stage) {
    const int c0 = tile * kTile + 32 * w;
    if (c0 >= p.S) return;
    const int nv = min(32, p.S - c0);
    char* sK = ring + stage * L::kStageB;
    char* sV = sK + 32 * D;
#pragma unroll
    for (int k = 0; k < CPR; ++k) {
      const int idx = k * 32 + lane, row = idx / CPR, ch = idx % CPR;
      if (row < nv) {
        cp_async16(sK + row * D + ((ch ^ (row % CPR)) * 16),
                   kbase + static_cast<int64_t>(c0 + row) * p.kqs + ch * 16);
        cp_async16(sV + row * D + ch * 16, vbase + static_cast<int64_t>(c0 + row) * p.vqs + ch * 16);
      }
    }
  };
  auto load_sv = [&](int tile) {
    const int t = tile * kTile + 32 * w + lane;
    if (t >= p.S) return 0.0f;
    const int64_t o = vsbase + static_cast<int64_t>(t) * p.vsss;
    return p.vs_f16 ? __half2float(reinterpret_cast<const __half*>(p.vs)[o])
                    : reinterpret_cast<const float*>(p.vs)[o];
  };

  float m[NR], l[NR];
  F2 o[NR][NF];
#pragma unroll
  for (int hh = 0; hh < NR; ++hh) {
    m[hh] = -INFINITY;
    l[hh] = 0.0f;
#pragma unroll
    for (int f = 0; f < NF; ++f) o[hh][f].v = 0ull;
  }

  float ksr[kQpPer];
  __syncthreads();   // q (qf) is complete before the first q' is formed from it
  if (t_begin < t_end) {
    issue(t_begin, 0);
    load_ks(t_begin, ksr);
    store_qp(0, ksr);
  }
  cp_async_commit();
  float sv = t_begin < t_end ? load_sv(t_begin) : 0.0f;
  for (int it = 0; t_begin + it < t_end; ++it) {
    const int tile = t_begin + it, cur = it & 1;
    __syncthreads();   // q'[cur] is written; q'[cur ^ 1] is no longer read
    const bool more = tile + 1 < t_end;
    if (more) {
      issue(tile + 1, cur ^ 1);
      load_ks(tile + 1, ksr);
    }
    cp_async_commit();
    const float sv_next = more ? load_sv(tile + 1) : 0.0f;
    cp_async_wait<1>();   // this tile's chunk has landed
    __syncwarp();
    const int tok0 = tile * kTile;
    const int c0 = tok0 + 32 * w;
    if (c0 < p.S) {
      const bool valid = c0 + lane < p.S;
      const int n_valid = min(32, p.S - c0);
      const float* qpw = qp + cur * 2 * NR * D + (c0 / p.BT - tok0 / p.BT) * NR * D;
      const char* sK = ring + cur * L::kStageB;
      const char* sV = sK + 32 * D;
      // scores: q' . codes (lane = token)
      F2 acc[NR], acc2[NR];   // two chains per head (even / odd words)
#pragma unroll
      for (int hh = 0; hh < NR; ++hh) acc[hh].v = acc2[hh].v = 0ull;
#pragma unroll
      for (int i = 0; i < CPR; ++i) {
        const uint4 kv = *reinterpret_cast<const uint4*>(sK + lane * D + ((i ^ (lane % CPR)) * 16));
        const uint32_t wd[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          F2 lo2, hi2;
          s8x4_to_f2x2(wd[e], lo2, hi2);
          const int d = 16 * i + 4 * e;
#pragma unroll
          for (int hh = 0; hh < NR; ++hh) {
            const ulonglong2 qq = *reinterpret_cast<const ulonglong2*>(qpw + hh * D + d);
            F2 qa, qb;
            qa.v = qq.x;
            qb.v = qq.y;
            if (e & 1) {
              acc2[hh] = f2_fma(lo2, qa, acc2[hh]);
              acc2[hh] = f2_fma(hi2, qb, acc2[hh]);
            } else {
              acc[hh] = f2_fma(lo2, qa, acc[hh]);
              acc[hh] = f2_fma(hi2, qb, acc[hh]);
            }
          }
        }
      }
#pragma unroll
      for (int hh = 0; hh < NR; ++hh) acc[hh] = f2_add(acc[hh], acc2[hh]);
      // online softmax (lane 0 of the chunk is always valid, so the maxima are finite)
#pragma unroll
      for (int hh = 0; hh < NR; ++hh) {
        const float sc = valid ? f2_sum(acc[hh]) : -INFINITY;
        float mx = sc;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float mn = fmaxf(m[hh], mx);
        const float alpha = exp2f(m[hh] - mn);
        const float pr = valid ? exp2f(sc - mn) : 0.0f;
        l[hh] = l[hh] * alpha + pr;
        const F2 a2 = f2_make(alpha, alpha);
#pragma unroll
        for (int f = 0; f < NF; ++f) o[hh][f] = f2_mul(o[hh][f], a2);
        m[hh] = mn;
        pvb[(w * 32 + lane) * NR + hh] = pr * sv;
      }
      __syncwarp();
      // V: lane owns channels lane * DPL ..
#pragma unroll 8
      for (int tt = 0; tt < 32; ++tt) {
        if (tt < n_valid) {
          uint32_t word;
          if constexpr (DPL == 4)
            word = *reinterpret_cast<const uint32_t*>(sV + tt * D + lane * 4);
          else
            word = *reinterpret_cast<const uint16_t*>(sV + tt * D + lane * 2);
          F2 c[2];
          s8x4_to_f2x2(word, c[0], c[1]);
#pragma unroll
          for (int hh = 0; hh < NR; ++hh) {
            const float pp = pvb[(w * 32 + tt) * NR + hh];
            const F2 p2 = f2_make(pp, pp);
#pragma unroll
            for (int f = 0; f < NF; ++f) o[hh][f] = f2_fma(c[f], p2, o[hh][f]);
          }
        }
      }
    }
    if (more) store_qp(cur ^ 1, ksr);
    sv = sv_next;
    __syncwarp();   // the stage is refilled only after every lane has read it
  }
  cp_async_wait<0>();
  __syncthreads();   // the ring is free: the merge scratch below aliases it
  float* wo = reinterpret_cast<float*>(smem);   // [4][NR][D]

  // merge the 4 warps
#pragma unroll
  for (int hh = 0; hh < NR; ++hh) {
    float lt = l[hh];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, off);
    if (lane == 0) {
      wmb[w * NR + hh] = m[hh];
      wlb[w * NR + hh] = lt;
    }
#pragma unroll
    for (int f = 0; f < NF; ++f) {
      float a, c;
      f2_split(o[hh][f], a, c);
      wo[(w * NR + hh) * D + lane * DPL + 2 * f] = a;
      wo[(w * NR + hh) * D + lane * DPL + 2 * f + 1] = c;
    }
  }
  __syncthreads();
  for (int i = tid; i < NR * D; i += kDecThreads) {
    const int hh = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int ww = 0; ww < 4; ++ww) M = fmaxf(M, wmb[ww * NR + hh]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int ww = 0; ww < 4; ++ww) {
        if (wmb[ww * NR + hh] == -INFINITY) continue;
        const float e = exp2f(wmb[ww * NR + hh] - M);
        L += wlb[ww * NR + hh] * e;
        O += wo[(ww * NR + hh) * D + d] * e;
      }
    }
    const int64_t hq = hk * NR + hh;
    if (p.n_split == 1) {
      store_any(p.out, b * p.osb + hq * p.osh + d, p.q_dtype, L > 0.0f ? O / L : 0.0f);
    } else {
      const int64_t row = (b * Hq + hq) * p.n_split + split;
      p.ws_o[row * D + d] = O;
      if (d == 0) {
        p.ws_ml[2 * row] = M;
        p.ws_ml[2 * row + 1] = L;
      }
    }
  }
  if (p.n_split == 1) return;
  // the last split block of this (sequence, kv head) to arrive merges the splits
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int ticket = atomicAdd(p.ws_cnt + b * p.Hkv + hk, 1);
    *last = ticket == p.n_split - 1;
  }
  __syncthreads();
  if (!*last) return;
  __threadfence();
  // split weights 2^(m_s - M) / L per head, one warp per head, all splits in parallel
  // (the per-warp buffers are free again: every thread is past the loop above)
  float* wts = wo;   // [NR][kMaxSplit]
  for (int hh = w; hh < NR; hh += 4) {
    const int64_t row0 = (b * Hq + hk * NR + hh) * p.n_split;
    float mv[kMaxSplit / 32], lv[kMaxSplit / 32];
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < kMaxSplit / 32; ++k) {
      const int s = lane + 32 * k;
      mv[k] = s < p.n_split ? __ldcg(p.ws_ml + 2 * (row0 + s)) : -INFINITY;
      lv[k] = s < p.n_split ? __ldcg(p.ws_ml + 2 * (row0 + s) + 1) : 0.0f;
      M = fmaxf(M, mv[k]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float L = 0.0f;
#pragma unroll
    for (int k = 0; k < kMaxSplit / 32; ++k) {
      mv[k] = mv[k] == -INFINITY ? 0.0f : exp2f(mv[k] - M);
      L += lv[k] * mv[k];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
    for (int k = 0; k < kMaxSplit / 32; ++k) {
      const int s = lane + 32 * k;
      if (s < p.n_split) wts[hh * kMaxSplit + s] = mv[k] * inv;
    }
  }
  __syncthreads();
  for (int i = tid; i < NR * D; i += kDecThreads) {
    const int hh = i / D, d = i % D;
    const int64_t hq = hk * NR + hh;
    const float* src = p.ws_o + (b * Hq + hq) * p.n_split * D + d;
    const float* wt = wts + hh * kMaxSplit;
    float O = 0.0f;
    int s = 0;
    for (; s + 8 <= p.n_split; s += 8) {
      float ov[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) ov[u] = __ldcg(src + static_cast<int64_t>(s + u) * D);
#pragma unroll
      for (int u = 0; u < 8; ++u) O += wt[s + u] * ov[u];
    }
    for (; s < p.n_split; ++s) O += wt[s] * __ldcg(src + static_cast<int64_t>(s) * D);
    store_any(p.out, b * p.osb + hq * p.osh + d, p.q_dtype, O);
  }
  if (tid == 0) p.ws_cnt[b * p.Hkv + hk] = 0;
}

// ------------------------------------------------------------------ dequant
__global__ void kblock_dequant_kernel(const int8_t* __restrict__ kq, int64_t kqb, int64_t kqh,
                                      int64_t kqs, const float* __restrict__ ksc, int64_t kscb,
                                      int64_t ksch, int64_t kscx, int H, int S, int D, int BT,
                                      void* __restrict__ out, int odt, int64_t osb, int64_t osh,
                                      int64_t oss, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t d = i % D, r = i / D;
    const int64_t s = r % S, bh = r / S;
    const int64_t h = bh % H, b = bh / H;
    const float c = static_cast<float>(kq[b * kqb + h * kqh + s * kqs + d]);
    const float f = ksc[b * kscb + h * ksch + (s / BT) * kscx + d];
    store_any(out, b * osb + h * osh + s * oss + d, odt, c * f);
  }
}

// ------------------------------------------------------------------ host side
struct Plan {
  int n_split, tps;
};

static Plan plan(int B, int Hkv, int S, int sms, int per_sm) {
  const int n_tiles = (S + kTile - 1) / kTile;
  const int64_t units = static_cast<int64_t>(B) * Hkv;
  // one wave: as many splits as leave every block resident at once
  int want = static_cast<int>(static_cast<int64_t>(per_sm) * sms / units);
  want = std::max(1, std::min(std::min(want, n_tiles), kMaxSplit));
  const int tps = (n_tiles + want - 1) / want;
  return {(n_tiles + tps - 1) / tps, tps};
}

static size_t al256(size_t n) { return (n + 255) & ~size_t(255); }

// Workspace layout, shared with the tensor-core kernel (decode_common.cuh) so that
// either kernel finds the other's arrival tickets zero: a 256-byte header (status
// word), the ticket region [B*Hkv] x 2 ints from byte 256, then the split partials.
static size_t tickets_region(int B, int Hkv) {
  return al256(2 * sizeof(int) * static_cast<size_t>(B) * Hkv);
}
static size_t ws_bytes(int B, int Hq, int Hkv, int S, int D, int sms, int per_sm) {
  const Plan pl = plan(B, Hkv, S, sms, per_sm);
  if (pl.n_split <= 1) return 256;
  const size_t rows = static_cast<size_t>(B) * Hq * pl.n_split;
  return 256 + tickets_region(B, Hkv) + al256(rows * 2 * sizeof(float)) +
         al256(rows * D * sizeof(float));
}

static bool al(const void* ptr, size_t a) { return reinterpret_cast<uintptr_t>(ptr) % a == 0; }

static bool valid_bt(int bt) { return bt == 64 || bt == 128 || bt == 256; }

static int done() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}

template <int DT>
static void launch_write_d(const WriteParams& p, dim3 grid, cudaStream_t st) {
  if (p.D == 64)
    kblock_write_kernel<DT, 64><<<grid, kWriteThreads, 0, st>>>(p);
  else if (p.D == 128)
    kblock_write_kernel<DT, 128><<<grid, kWriteThreads, 0, st>>>(p);
  else
    kblock_write_kernel<DT, 256><<<grid, kWriteThreads, 0, st>>>(p);
}

static int launch_write(const WriteParams& p, int x_dtype, dim3 grid, cudaStream_t st) {
  if (x_dtype == HQ_DTYPE_BF16)
    launch_write_d<HQ_DTYPE_BF16>(p, grid, st);
  else if (x_dtype == HQ_DTYPE_F16)
    launch_write_d<HQ_DTYPE_F16>(p, grid, st);
  else
    launch_write_d<HQ_DTYPE_F32>(p, grid, st);
  return done();
}

// Blocks of the decode kernel resident per SM (its dynamic shared memory opted in
// on first use per device); -1 if the runtime refuses.
template <int NR, int D>
static int per_sm_blocks() {
  constexpr int kSmem = DecLayout<NR, D>::kBytes;
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  int v = cache[dev].load(std::memory_order_acquire);
  if (v > 0) return v;
  if (cudaFuncSetAttribute(kblock_decode_kernel<NR, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kSmem) != cudaSuccess)
    return -1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kblock_decode_kernel<NR, D>, kDecThreads,
                                                    kSmem) != cudaSuccess || n < 1)
    return -1;
  cache[dev].store(n, std::memory_order_release);
  return n;
}

static int per_sm_for(int NR, int D) {
  if (D == 128) {
    switch (NR) {
      case 1: return per_sm_blocks<1, 128>();
      case 2: return per_sm_blocks<2, 128>();
      case 4: return per_sm_blocks<4, 128>();
      default: return per_sm_blocks<8, 128>();
    }
  }
  switch (NR) {
    case 1: return per_sm_blocks<1, 64>();
    case 2: return per_sm_blocks<2, 64>();
    case 4: return per_sm_blocks<4, 64>();
    default: return per_sm_blocks<8, 64>();
  }
}

template <int NR, int D>
static int launch_decode(const DecParams& p, int B, cudaStream_t st) {
  dim3 grid(p.Hkv, p.n_split, B);
  kblock_decode_kernel<NR, D><<<grid, kDecThreads, DecLayout<NR, D>::kBytes, st>>>(p);
  return done();
}

}  // namespace kb
}  // namespace hq

using namespace hq;
using namespace hq::kb;

static int kblock_write_impl(const void* k_new, const void* v_new, int x_dtype,
                             const int64_t k_strides[4], const int64_t v_strides[4], int B,
                             int H, int pos, int S_new, int D, int block_tokens,
                             int8_t* k_cache, const int64_t kq_strides[4], float* k_scale,
                             const int64_t ks_strides[3], void* k_tail,
                             const int64_t kt_strides[4], int8_t* v_cache,
                             const int64_t vq_strides[4], float* v_scale_f32,
                             uint16_t* v_scale_f16, const int64_t vs_strides[3], int capacity,
                             int* lens, hq_stream_t stream) {
  if (!k_new || !k_strides || !k_cache || !kq_strides || !k_scale || !ks_strides || !k_tail ||
      !kt_strides || B < 0 || H < 0 || pos < 0 || S_new < 1 || capacity < 1 ||
      static_cast<int64_t>(pos) + S_new > capacity)
    return HQ_ERR_INVALID_ARGUMENT;
  if (lens && (S_new != 1 || !al(lens, 4))) return HQ_ERR_INVALID_ARGUMENT;
  if (v_new && (!v_strides || !v_cache || !vq_strides || (!v_scale_f32 && !v_scale_f16) ||
                !vs_strides || (v_scale_f32 && v_scale_f16)))
    return HQ_ERR_INVALID_ARGUMENT;
  if (x_dtype != HQ_DTYPE_BF16 && x_dtype != HQ_DTYPE_F16 && x_dtype != HQ_DTYPE_F32)
    return HQ_ERR_UNSUPPORTED;
  if ((D != 64 && D != 128 && D != 256) || !valid_bt(block_tokens)) return HQ_ERR_UNSUPPORTED;
  if (B == 0 || H == 0) return HQ_OK;
  if (B > 65535 || H > 65535) return HQ_ERR_UNSUPPORTED;   // grid z / y limits
  // channel pairs: the last dimension contiguous, rows and pairs 2-element aligned
  if (k_strides[3] != 1 || kq_strides[3] != 1 || ks_strides == nullptr || kt_strides[3] != 1 ||
      !al(k_cache, 2) || kq_strides[0] % 2 || kq_strides[1] % 2 || kq_strides[2] % 2 ||
      !al(k_scale, 8) || ks_strides[0] % 2 || ks_strides[1] % 2 || ks_strides[2] % 2)
    return HQ_ERR_INVALID_ARGUMENT;
  if (v_new && (v_strides[3] != 1 || vq_strides[3] != 1)) return HQ_ERR_INVALID_ARGUMENT;
  WriteParams p{};
  p.k = k_new;
  p.ksb = k_strides[0]; p.ksh = k_strides[1]; p.kss = k_strides[2];
  p.v = v_new;
  if (v_new) {
    p.vsb = v_strides[0]; p.vsh = v_strides[1]; p.vss = v_strides[2];
    p.vq = v_cache;
    p.vqb = vq_strides[0]; p.vqh = vq_strides[1]; p.vqs = vq_strides[2];
    p.vs32 = v_scale_f32;
    p.vs16 = reinterpret_cast<__half*>(v_scale_f16);
    p.vssb = vs_strides[0]; p.vssh = vs_strides[1]; p.vsss = vs_strides[2];
  }
  p.kq = k_cache;
  p.kqb = kq_strides[0]; p.kqh = kq_strides[1]; p.kqs = kq_strides[2];
  p.ksc = k_scale;
  p.kscb = ks_strides[0]; p.ksch = ks_strides[1]; p.kscx = ks_strides[2];
  p.kt = k_tail;
  p.ktb = kt_strides[0]; p.kth = kt_strides[1]; p.kts = kt_strides[2];
  p.D = D;
  p.BT = block_tokens;
  p.pos = pos;
  p.S_new = S_new;
  p.lens = lens;
  p.cap = capacity;
  if (lens) {  // one token: one block, whose index the kernel takes from lens[0]
    p.blk0 = 0;
    p.tail_mode = 0;
    return launch_write(p, x_dtype, dim3(1, H, B), reinterpret_cast<cudaStream_t>(stream));
  }
  const int blk0 = pos / block_tokens, blk1 = (pos + S_new - 1) / block_tokens;
  p.blk0 = blk0;
  // the first block reads the tail (its earlier rows) while the last one would write
  // it: when both happen in different blocks the tail is written by a second launch
  const bool old_rows = pos % block_tokens != 0;
  const bool open_end = (pos + S_new) % block_tokens != 0;
  const bool split_tail = blk1 > blk0 && old_rows && open_end;
  p.tail_mode = split_tail ? 1 : 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc = launch_write(p, x_dtype, dim3(blk1 - blk0 + 1, H, B), st);
  if (rc != HQ_OK || !split_tail) return rc;
  p.tail_mode = 2;
  p.blk0 = blk1;
  p.v = nullptr;
  return launch_write(p, x_dtype, dim3(1, H, B), st);
}

extern "C" int hq_kblock_write(const void* k_new, const void* v_new, int x_dtype,
                               const int64_t k_strides[4], const int64_t v_strides[4], int B,
                               int H, int pos, int S_new, int D, int block_tokens,
                               int8_t* k_cache, const int64_t kq_strides[4], float* k_scale,
                               const int64_t ks_strides[3], void* k_tail,
                               const int64_t kt_strides[4], int8_t* v_cache,
                               const int64_t vq_strides[4], float* v_scale_f32,
                               uint16_t* v_scale_f16, const int64_t vs_strides[3], int capacity,
                               hq_stream_t stream) {
  return kblock_write_impl(k_new, v_new, x_dtype, k_strides, v_strides, B, H, pos, S_new, D,
                           block_tokens, k_cache, kq_strides, k_scale, ks_strides, k_tail,
                           kt_strides, v_cache, vq_strides, v_scale_f32, v_scale_f16, vs_strides,
                           capacity, nullptr, stream);
}

extern "C" int hq_kblock_write_at(const void* k_new, const void* v_new, int x_dtype,
                                  const int64_t k_strides[4], const int64_t v_strides[4], int B,
                                  int H, int D, int block_tokens, int8_t* k_cache,
                                  const int64_t kq_strides[4], float* k_scale,
                                  const int64_t ks_strides[3], void* k_tail,
                                  const int64_t kt_strides[4], int8_t* v_cache,
                                  const int64_t vq_strides[4], float* v_scale_f32,
                                  uint16_t* v_scale_f16, const int64_t vs_strides[3],
                                  int capacity, int* lens, hq_stream_t stream) {
  if (!lens) return HQ_ERR_INVALID_ARGUMENT;
  return kblock_write_impl(k_new, v_new, x_dtype, k_strides, v_strides, B, H, 0, 1, D,
                           block_tokens, k_cache, kq_strides, k_scale, ks_strides, k_tail,
                           kt_strides, v_cache, vq_strides, v_scale_f32, v_scale_f16, vs_strides,
                           capacity, lens, stream);
}

extern "C" size_t hq_kblock_decode_workspace_bytes(int B, int Hq, int Hkv, int S, int D) {
  if (B < 1 || Hkv < 1 || Hq < Hkv || Hq % Hkv || S < 1 || (D != 64 && D != 128)) return 0;
  const int NR = Hq / Hkv;
  if (NR != 1 && NR != 2 && NR != 4 && NR != 8) return 0;
  const int per_sm = per_sm_for(NR, D);
  if (per_sm < 1) return 0;
  // either kernel may serve the call: room for the larger of their layouts
  return std::max(ws_bytes(B, Hq, Hkv, S, D, current_sm_count(), per_sm),
                  kblock_decode_mma_workspace_bytes(B, Hq, Hkv, S, D));
}

extern "C" int hq_kblock_decode(const void* q, int q_dtype, const int64_t q_strides[3],
                                const int8_t* k_cache, const int64_t kq_strides[3],
                                const float* k_scale, const int64_t ks_strides[3],
                                const int8_t* v_cache, const int64_t vq_strides[3],
                                const void* v_scale, int scale_dtype,
                                const int64_t vs_strides[3], int B, int Hq, int Hkv, int S, int D,
                                int block_tokens, float sm_scale, void* out,
                                const int64_t out_strides[3], void* workspace,
                                size_t workspace_bytes, hq_stream_t stream) {
  if (!q || !q_strides || !k_cache || !kq_strides || !k_scale || !ks_strides || !v_cache ||
      !vq_strides || !v_scale || !vs_strides || !out || !out_strides || B < 0 || Hkv < 1 ||
      Hq < Hkv || Hq % Hkv || S < 1)
    return HQ_ERR_INVALID_ARGUMENT;
  if (q_dtype != HQ_DTYPE_BF16 && q_dtype != HQ_DTYPE_F16 && q_dtype != HQ_DTYPE_F32)
    return HQ_ERR_UNSUPPORTED;
  if (scale_dtype != HQ_DTYPE_F32 && scale_dtype != HQ_DTYPE_F16) return HQ_ERR_UNSUPPORTED;
  const int NR = Hq / Hkv;
  if ((D != 64 && D != 128) || !valid_bt(block_tokens) || (NR != 1 && NR != 2 && NR != 4 && NR != 8))
    return HQ_ERR_UNSUPPORTED;
  if (B == 0) return HQ_OK;
  if (B > 65535) return HQ_ERR_UNSUPPORTED;   // grid z limit
  // K rows are read as 16-byte vectors, V by 2 or 4 bytes per lane
  if (q_strides[2] != 1 || out_strides[2] != 1 || !al(k_cache, 16) || kq_strides[0] % 16 ||
      kq_strides[1] % 16 || kq_strides[2] % 16 || !al(v_cache, 16) || vq_strides[0] % 16 ||
      vq_strides[1] % 16 || vq_strides[2] % 16)
    return HQ_ERR_INVALID_ARGUMENT;
  // the tensor-core kernel (decode_kblock.cu) for head_dim 128 and up to 4 q heads per
  // kv head; the CUDA-core kernel below for the rest
  if (B <= 65535) {
    const int rc = kblock_decode_mma(q, q_dtype, q_strides, k_cache, kq_strides, k_scale,
                                     ks_strides, v_cache, vq_strides, v_scale, scale_dtype,
                                     vs_strides, B, Hq, Hkv, S, D, block_tokens, sm_scale, out,
                                     out_strides, workspace, workspace_bytes, stream);
    if (rc != HQ_ERR_UNSUPPORTED) return rc;
  }
  const int sms = current_sm_count();
  const int per_sm = per_sm_for(NR, D);
  if (per_sm < 1) return HQ_ERR_UNSUPPORTED;
  const Plan pl = plan(B, Hkv, S, sms, per_sm);
  DecParams p{};
  p.q = q;
  p.qsb = q_strides[0]; p.qsh = q_strides[1];
  p.q_dtype = q_dtype;
  p.kq = k_cache;
  p.kqb = kq_strides[0]; p.kqh = kq_strides[1]; p.kqs = kq_strides[2];
  p.ksc = k_scale;
  p.kscb = ks_strides[0]; p.ksch = ks_strides[1]; p.kscx = ks_strides[2];
  p.vq = v_cache;
  p.vqb = vq_strides[0]; p.vqh = vq_strides[1]; p.vqs = vq_strides[2];
  p.vs = v_scale;
  p.vs_f16 = scale_dtype == HQ_DTYPE_F16;
  p.vssb = vs_strides[0]; p.vssh = vs_strides[1]; p.vsss = vs_strides[2];
  p.out = out;
  p.osb = out_strides[0]; p.osh = out_strides[1];
  p.Hkv = Hkv;
  p.S = S;
  p.BT = block_tokens;
  p.tps = pl.tps;
  p.n_split = pl.n_split;
  p.qscale = sm_scale * 1.4426950408889634f;
  if (pl.n_split > 1) {
    const size_t need = ws_bytes(B, Hq, Hkv, S, D, sms, per_sm);
    if (!workspace || workspace_bytes < need || !al(workspace, 256)) return HQ_ERR_WORKSPACE;
    char* w = static_cast<char*>(workspace);
    const size_t rows = static_cast<size_t>(B) * Hq * pl.n_split;
    p.ws_cnt = reinterpret_cast<int*>(w + 256);
    w += 256 + tickets_region(B, Hkv);
    p.ws_ml = reinterpret_cast<float*>(w);
    w += al256(rows * 2 * sizeof(float));
    p.ws_o = reinterpret_cast<float*>(w);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define HQ_KB_NR(D_)                                              \
  switch (NR) {                                                   \
    case 1: return launch_decode<1, D_>(p, B, st);                \
    case 2: return launch_decode<2, D_>(p, B, st);                \
    case 4: return launch_decode<4, D_>(p, B, st);                \
    default: return launch_decode<8, D_>(p, B, st);               \
  }
  if (D == 128) {
    HQ_KB_NR(128)
  } else {
    HQ_KB_NR(64)
  }
#undef HQ_KB_NR
}

extern "C" int hq_kblock_decode_len(const void* q, int q_dtype, const int64_t q_strides[3],
                                    const int8_t* k_cache, const int64_t kq_strides[3],
                                    const float* k_scale, const int64_t ks_strides[3],
                                    const int8_t* v_cache, const int64_t vq_strides[3],
                                    const void* v_scale, int scale_dtype,
                                    const int64_t vs_strides[3], int B, int Hq, int Hkv,
                                    int capacity, const int* seq_len, int S_plan, int D,
                                    int block_tokens, float sm_scale, void* out,
                                    const int64_t out_strides[3], void* workspace,
                                    size_t workspace_bytes, hq_stream_t stream) {
  if (!q || !q_strides || !k_cache || !kq_strides || !k_scale || !ks_strides || !v_cache ||
      !vq_strides || !v_scale || !vs_strides || !out || !out_strides || !seq_len ||
      !al(seq_len, 4) || B < 0 || Hkv < 1 || Hq < Hkv || Hq % Hkv || capacity < 1)
    return HQ_ERR_INVALID_ARGUMENT;
  if (q_dtype != HQ_DTYPE_BF16 && q_dtype != HQ_DTYPE_F16 && q_dtype != HQ_DTYPE_F32)
    return HQ_ERR_UNSUPPORTED;
  if ((scale_dtype != HQ_DTYPE_F32 && scale_dtype != HQ_DTYPE_F16) || !valid_bt(block_tokens))
    return HQ_ERR_UNSUPPORTED;
  if (B == 0) return HQ_OK;
  if (B > 65535) return HQ_ERR_UNSUPPORTED;
  if (q_strides[2] != 1 || out_strides[2] != 1 || !al(k_cache, 16) || kq_strides[0] % 16 ||
      kq_strides[1] % 16 || kq_strides[2] % 16 || !al(v_cache, 16) || vq_strides[0] % 16 ||
      vq_strides[1] % 16 || vq_strides[2] % 16)
    return HQ_ERR_INVALID_ARGUMENT;
  if (!workspace || !al(workspace, 256)) return HQ_ERR_WORKSPACE;
  // the tensor-core kernel only (head_dim 128, up to 4 q heads per kv head)
  return kblock_decode_mma(q, q_dtype, q_strides, k_cache, kq_strides, k_scale, ks_strides,
                           v_cache, vq_strides, v_scale, scale_dtype, vs_strides, B, Hq, Hkv,
                           capacity, D, block_tokens, sm_scale, out, out_strides, workspace,
                           workspace_bytes, stream, seq_len, S_plan);
}

extern "C" int hq_kblock_dequant(const int8_t* k_cache, const int64_t kq_strides[3],
                                 const float* k_scale, const int64_t ks_strides[3], int B, int H,
                                 int S, int D, int block_tokens, void* out, int out_dtype,
                                 const int64_t out_strides[4], hq_stream_t stream) {
  if (!k_cache || !kq_strides || !k_scale || !ks_strides || !out || !out_strides || B < 0 ||
      H < 0 || S < 0 || D < 1 || !valid_bt(block_tokens) || out_strides[3] != 1)
    return HQ_ERR_INVALID_ARGUMENT;
  if (out_dtype != HQ_DTYPE_BF16 && out_dtype != HQ_DTYPE_F16 && out_dtype != HQ_DTYPE_F32)
    return HQ_ERR_UNSUPPORTED;
  const int64_t n = static_cast<int64_t>(B) * H * S * D;
  if (n == 0) return HQ_OK;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 8LL * current_sm_count());
  kblock_dequant_kernel<<<static_cast<unsigned>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      k_cache, kq_strides[0], kq_strides[1], kq_strides[2], k_scale, ks_strides[0], ks_strides[1],
      ks_strides[2], H, S, D, block_tokens, out, out_dtype, out_strides[0], out_strides[1],
      out_strides[2], n);
  return done();
}
