// Split-KV decode attention over an int8 KV cache (sm_100a), its dense
// (bf16 / f16) twin and the log-sum-exp combine.
//
// Reference semantics: int8_decode_attn (src/kernels/int8_decode_attn_triton.py:15-63,
// 101-113) - dequantize K per channel and V per token in registers, online
// float32 softmax, one query token - and the decode step of
// quantized_attention_forward (tests/qwen_kvcache_full.py:95-113), including its
// optional per-token fake quantization of q.  The reference launches one
// program per q head (16 programs for the whole GPU).  This kernel:
//
//   * splits the sequence: grid = (split, kv head, batch), split count chosen
//     on the host so that the grid fills every SM (batch 1 included);
//   * serves all n_rep = Hq / Hkv q heads of a kv head from one K/V tile;
//   * streams K/V tiles (64 tokens) through a 4-stage shared-memory ring filled
//     by 1-D bulk copies (cp.async.bulk, completion on mbarriers, no tensor
//     map, no multicast); every barrier wait is bounded;
//   * gives each token to LPT lanes (LPT = 2 * n_rep), each owning D / LPT
//     channels; a lane keeps q * k_scale * sm_scale * log2(e) for its channels
//     in registers, so K dequantization costs nothing per element beyond the
//     int8 -> float conversion (byte permute + packed subtract) and the packed
//     f32x2 FMA; V scales are folded into the softmax weight p;
//   * rotates each lane's chunk order by its token parity so the 16-byte
//     shared-memory reads of a quarter warp hit 8 distinct bank groups;
//   * combines splits in the same launch: each block writes (m, l, o) for its
//     split, and the last block of a (batch, kv head) to arrive - an atomic
//     ticket, no waiting - merges them and resets the ticket.
#include <atomic>
#include <cmath>

#include "hq_common.cuh"

namespace hq {
int sm_count(int dev);
int current_sm_count();

namespace dec {

constexpr int kD = 128;
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
  void* out;
  int64_t osb, osh;
  float* partial_out;  // [B*Hq][kD+2] or null
  float* ws_part;      // [B*Hq][n_split][kD+2]
  int* ws_count;       // [B*Hkv]
  int* ws_status;
  int n_split;
  int tiles_per_split;
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

template <int NREP, int KVDT, int SDT, int QDT>
__global__ void __launch_bounds__(kThreads, 3) decode_kernel(const Params p) {
  constexpr bool kInt8 = KVDT == HQ_DTYPE_I8;
  using C = Cfg<NREP, kInt8>;
  using QE = Elem<QDT>;
  using SE = Elem<SDT>;
  constexpr int kStages = C::kStages;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* ring = smem;
  float* qs = reinterpret_cast<float*>(smem + C::SMEM_STAGES);
  uint64_t* full = reinterpret_cast<uint64_t*>(qs + NREP * kD);
  uint64_t* empty = full + kStages;
  __shared__ float red[kWarps][NREP];
  __shared__ float wl[C::NG][NREP];
  __shared__ float wm[kWarps][NREP];
  __shared__ float cM[NREP], cL[NREP];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int g = tid / C::LPT, j = tid % C::LPT;
  const int rot = g % C::CPL;
  const int s_begin = split * p.tiles_per_split * kTile;
  const int s_end = min(p.S, s_begin + p.tiles_per_split * kTile);
  const int ntok = max(0, s_end - s_begin);
  const int ntiles = (ntok + kTile - 1) / kTile;
  const char* kbase = p.k + (b * p.kvsb + kvh * p.kvsh + static_cast<int64_t>(s_begin) * kD) * C::EB;
  const char* vbase = p.v + (b * p.kvsb + kvh * p.kvsh + static_cast<int64_t>(s_begin) * kD) * C::EB;

  int issued = 0;  // tiles whose copies were started (thread 0 only)
  auto issue = [&](int t) {
    const int st = t % kStages;
    const uint32_t bytes = static_cast<uint32_t>(min(kTile, ntok - t * kTile) * C::ROW);
    unsigned char* dst = ring + st * 2 * C::TILE_BYTES;
    mbar_arrive_expect_tx(&full[st], 2 * bytes);
    bulk_g2s(dst, kbase + static_cast<int64_t>(t) * C::TILE_BYTES, bytes, &full[st]);
    bulk_g2s(dst + C::TILE_BYTES, vbase + static_cast<int64_t>(t) * C::TILE_BYTES, bytes, &full[st]);
    issued = t + 1;
  };

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0)
    for (int t = 0; t < min(kStages, ntiles); ++t) issue(t);

  // ---- q prologue (overlaps the first copies): thread tid owns channel d = tid
  {
    const int d = tid;
    const auto* qp = reinterpret_cast<const typename QE::T*>(p.q);
    float qv[NREP];
#pragma unroll
    for (int r = 0; r < NREP; ++r) qv[r] = QE::to_f32(qp[b * p.qsb + (kvh * NREP + r) * p.qsh + d]);
    if (p.q_quant) {
#pragma unroll
      for (int r = 0; r < NREP; ++r) {
        const float m = warp_max(fabsf(qv[r]), 1);
        if (lane == 0) red[warp][r] = m;
      }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < NREP; ++r) {
        float m = red[0][r];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) m = fmaxf(m, red[w][r]);
        const Quantizer qz = Quantizer::from_amax(m);
        qv[r] = QE::to_f32(QE::from_f32(static_cast<float>(qz.code(qv[r])) * qz.scale));
      }
    }
    float ks = 1.0f;
    if constexpr (kInt8) {
      const auto* kp = reinterpret_cast<const typename SE::T*>(p.ksc);
      ks = SE::to_f32(kp[b * p.kscb + kvh * p.ksch + d * p.kscd]);
    }
#pragma unroll
    for (int r = 0; r < NREP; ++r) qs[r * kD + d] = qv[r] * ks * p.qk_scale;
  }
  __syncthreads();

  // lane-private operands, in this lane's chunk load order
  int off[C::CPL];
  F2 qr[NREP][C::PAIRS];
#pragma unroll
  for (int i = 0; i < C::CPL; ++i) {
    const int c = j + C::LPT * ((i + rot) % C::CPL);
    off[i] = c * 16;
#pragma unroll
    for (int e = 0; e < C::CE / 2; ++e)
#pragma unroll
      for (int r = 0; r < NREP; ++r)
        qr[r][i * (C::CE / 2) + e] = f2_make(qs[r * kD + c * C::CE + 2 * e], qs[r * kD + c * C::CE + 2 * e + 1]);
  }

  F2 oacc[NREP][C::PAIRS];
  float m_run[NREP], l_run[NREP];
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    m_run[r] = -INFINITY;
    l_run[r] = 0.0f;
#pragma unroll
    for (int e = 0; e < C::PAIRS; ++e) oacc[r][e] = f2_make(0.0f, 0.0f);
  }

  const auto* vscp = reinterpret_cast<const typename SE::T*>(p.vsc);
  const int64_t vsc_row = b * p.vscb + kvh * p.vsch;
  bool ok = true;
  int consumed = 0;
  for (int t = 0; t < ntiles; ++t) {
    const int st = t % kStages;
    const uint32_t par = (t / kStages) & 1;
    const int nvalid = min(kTile, ntok - t * kTile);
    float vsf[C::TPG];
#pragma unroll
    for (int tg = 0; tg < C::TPG; ++tg) {
      const int row = tg * C::NG + g;
      vsf[tg] = 1.0f;
      if constexpr (kInt8)
        if (row < nvalid) vsf[tg] = SE::to_f32(vscp[vsc_row + static_cast<int64_t>(s_begin + t * kTile + row) * p.vscs]);
    }
    if (!mbar_wait(&full[st], par)) {
      ok = false;
      break;
    }
    consumed = t + 1;
    const unsigned char* kt = ring + st * 2 * C::TILE_BYTES;
    const unsigned char* vt = kt + C::TILE_BYTES;

    float sc[NREP][C::TPG];
#pragma unroll
    for (int tg = 0; tg < C::TPG; ++tg) {
      const int row = tg * C::NG + g;
      F2 acc[NREP];
#pragma unroll
      for (int r = 0; r < NREP; ++r) acc[r] = f2_make(0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < C::CPL; ++i) {
        const uint4 w = lds128(kt + row * C::ROW + off[i]);
        F2 kf[C::CE / 2];
        chunk_to_f2<KVDT>(w, kf);
#pragma unroll
        for (int e = 0; e < C::CE / 2; ++e)
#pragma unroll
          for (int r = 0; r < NREP; ++r) acc[r] = f2_fma(qr[r][i * (C::CE / 2) + e], kf[e], acc[r]);
      }
#pragma unroll
      for (int r = 0; r < NREP; ++r) {
        float a0, a1;
        f2_split(acc[r], a0, a1);
        float s = a0 + a1;
#pragma unroll
        for (int o = 1; o < C::LPT; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        sc[r][tg] = row < nvalid ? s : -INFINITY;
      }
    }
    // online softmax: the running max is shared by the whole warp
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      float mt = sc[r][0];
#pragma unroll
      for (int tg = 1; tg < C::TPG; ++tg) mt = fmaxf(mt, sc[r][tg]);
      mt = warp_max(mt, C::LPT);
      if (mt > m_run[r]) {
        const float alpha = exp2f(m_run[r] - mt);
        l_run[r] *= alpha;
        const F2 a2 = f2_make(alpha, alpha);
#pragma unroll
        for (int e = 0; e < C::PAIRS; ++e) oacc[r][e] = f2_mul(oacc[r][e], a2);
        m_run[r] = mt;
      }
    }
#pragma unroll
    for (int tg = 0; tg < C::TPG; ++tg) {
      const int row = tg * C::NG + g;
      if (row < nvalid) {
        F2 pp[NREP];
#pragma unroll
        for (int r = 0; r < NREP; ++r) {
          const float pr = exp2f(sc[r][tg] - m_run[r]);
          l_run[r] += pr;
          const float pv = pr * vsf[tg];
          pp[r] = f2_make(pv, pv);
        }
#pragma unroll
        for (int i = 0; i < C::CPL; ++i) {
          const uint4 w = lds128(vt + row * C::ROW + off[i]);
          F2 vf[C::CE / 2];
          chunk_to_f2<KVDT>(w, vf);
#pragma unroll
          for (int e = 0; e < C::CE / 2; ++e)
#pragma unroll
            for (int r = 0; r < NREP; ++r)
              oacc[r][i * (C::CE / 2) + e] = f2_fma(pp[r], vf[e], oacc[r][i * (C::CE / 2) + e]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (tid == 0 && t + kStages < ntiles) {
      if (!mbar_wait(&empty[st], par)) {
        ok = false;
        break;
      }
      issue(t + kStages);
    }
  }
  if (!ok) {
    report_error(p.ws_status, HQ_ERR_DEVICE_TIMEOUT);
    // let this block's own copies land before the block exits (bounded)
    if (tid == 0)
      for (int t = consumed; t < issued; ++t) mbar_wait(&full[t % kStages], (t / kStages) & 1);
  }
  __syncthreads();
  // every block reaches this point; a block that gave up writes nothing
  if (__syncthreads_or(!ok)) return;

  // ---- block epilogue: merge the NG groups (4 warps) of this split
  float* wo = reinterpret_cast<float*>(ring);  // [NG][NREP][kD]
#pragma unroll
  for (int i = 0; i < C::CPL; ++i) {
    const int c = j + C::LPT * ((i + rot) % C::CPL);
#pragma unroll
    for (int e = 0; e < C::CE / 2; ++e)
#pragma unroll
      for (int r = 0; r < NREP; ++r) {
        float a0, a1;
        f2_split(oacc[r][i * (C::CE / 2) + e], a0, a1);
        float* dst = wo + (g * NREP + r) * kD + c * C::CE + 2 * e;
        dst[0] = a0;
        dst[1] = a1;
      }
  }
  if (j == 0)
#pragma unroll
    for (int r = 0; r < NREP; ++r) wl[g][r] = l_run[r];
  if (lane == 0)
#pragma unroll
    for (int r = 0; r < NREP; ++r) wm[warp][r] = m_run[r];
  __syncthreads();

  const int d = tid;
  float Ms[NREP], Ls[NREP], Os[NREP];
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    float M = wm[0][r];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) M = fmaxf(M, wm[w][r]);
    float wf[kWarps];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) wf[w] = wm[w][r] == -INFINITY ? 0.0f : exp2f(wm[w][r] - M);
    float L = 0.0f, O = 0.0f;
#pragma unroll 4
    for (int gg = 0; gg < C::NG; ++gg) {
      const float f = wf[gg / C::GPW];
      L += wl[gg][r] * f;
      O += wo[(gg * NREP + r) * kD + d] * f;
    }
    Ms[r] = M;
    Ls[r] = L;
    Os[r] = O;
  }

  if (p.n_split == 1) {
#pragma unroll
    for (int r = 0; r < NREP; ++r) emit<QDT>(p, b, kvh * NREP + r, d, Ms[r], Ls[r], Os[r]);
    return;
  }

  // ---- publish this split, then the last block of (b, kvh) merges all splits
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    float* dst = p.ws_part + ((static_cast<int64_t>(b) * p.Hq + kvh * NREP + r) * p.n_split + split) * (kD + 2);
    if (d == 0) {
      dst[0] = Ms[r];
      dst[1] = Ls[r];
    }
    dst[2 + d] = Os[r];
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int ticket = atomicAdd(p.ws_count + b * p.Hkv + kvh, 1);
    s_last = ticket == p.n_split - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  float* wsc = reinterpret_cast<float*>(ring);  // [n_split] weights (ring is free now)
  for (int r = 0; r < NREP; ++r) {
    const float* src = p.ws_part + (static_cast<int64_t>(b) * p.Hq + kvh * NREP + r) * p.n_split * (kD + 2);
    float M = -INFINITY;
    for (int s = tid; s < p.n_split; s += kThreads) M = fmaxf(M, __ldcg(src + s * (kD + 2)));
    M = warp_max(M, 1);
    if (lane == 0) red[warp][0] = M;
    __syncthreads();
    M = fmaxf(fmaxf(red[0][0], red[1][0]), fmaxf(red[2][0], red[3][0]));
    float L = 0.0f;
    for (int s = tid; s < p.n_split; s += kThreads) {
      const float ms = __ldcg(src + s * (kD + 2));
      const float w = ms == -INFINITY ? 0.0f : exp2f(ms - M);
      wsc[s] = w;
      L += w * __ldcg(src + s * (kD + 2) + 1);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    __syncthreads();  // red[] reads above are done; wsc[] complete
    if (lane == 0) red[warp][0] = L;
    __syncthreads();
    if (tid == 0) {
      cM[r] = M;
      cL[r] = red[0][0] + red[1][0] + red[2][0] + red[3][0];
    }
    float O = 0.0f;
    for (int s = 0; s < p.n_split; ++s) O += wsc[s] * __ldcg(src + s * (kD + 2) + 2 + d);
    __syncthreads();
    emit<QDT>(p, b, kvh * NREP + r, d, cM[r], cL[r], O);
    __syncthreads();
  }
  if (tid == 0) p.ws_count[b * p.Hkv + kvh] = 0;  // ready for the next launch
}

// ------------------------------------------------------------------ cross-part combine
template <int ODT>
__global__ void __launch_bounds__(kThreads) combine_kernel(const float* __restrict__ parts,
                                                           int n_parts, int64_t part_stride,
                                                           int Hq, void* __restrict__ out,
                                                           int64_t osb, int64_t osh) {
  using OE = Elem<ODT>;
  const int bh = blockIdx.x;
  const int b = bh / Hq, h = bh % Hq;
  const int d = threadIdx.x;
  const float* base = parts + static_cast<int64_t>(bh) * (kD + 2);
  float M = -INFINITY;
  for (int i = 0; i < n_parts; ++i) M = fmaxf(M, base[i * part_stride]);
  float L = 0.0f, O = 0.0f;
  for (int i = 0; i < n_parts; ++i) {
    const float m = base[i * part_stride];
    const float w = m == -INFINITY ? 0.0f : exp2f(m - M);
    L += w * base[i * part_stride + 1];
    O += w * base[i * part_stride + 2 + d];
  }
  auto* o = reinterpret_cast<typename OE::T*>(out);
  o[b * osb + h * osh + d] = OE::from_f32(L > 0.0f ? O / L : 0.0f);
}

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
inline Plan make_plan(int units, int S, int slots, int sms) {
  const int tiles = (S + kTile - 1) / kTile;
  if (tiles <= 0) return {1, 1};
  const int cap = max_splits(units, tiles, sms);
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

inline size_t workspace_bytes(int B, int Hq, int Hkv, int S, int sms) {
  const int units = B * Hkv;
  const int tiles = (S + kTile - 1) / kTile;
  const int ms = max_splits(units > 0 ? units : 1, tiles, sms);
  return 256 + align256(sizeof(int) * static_cast<size_t>(B) * Hkv) +
         sizeof(float) * static_cast<size_t>(B) * Hq * ms * (kD + 2);
}

template <int NREP, int KVDT, int SDT, int QDT>
int launch(Params p, int B, void* ws, size_t ws_bytes, cudaStream_t st) {
  using C = Cfg<NREP, KVDT == HQ_DTYPE_I8>;
  auto kern = decode_kernel<NREP, KVDT, SDT, QDT>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<int> occ[64];
  int per_sm = (dev >= 0 && dev < 64) ? occ[dev].load(std::memory_order_relaxed) : 0;
  if (per_sm <= 0) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return static_cast<int>(e);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, C::SMEM);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (per_sm <= 0) return HQ_ERR_UNSUPPORTED;
    if (dev >= 0 && dev < 64) occ[dev].store(per_sm, std::memory_order_relaxed);
  }
  const int sms = sm_count(dev);
  const Plan pl = make_plan(B * p.Hkv, p.S, per_sm * sms, sms);
  if (ws_bytes < workspace_bytes(B, p.Hq, p.Hkv, p.S, sms)) return HQ_ERR_WORKSPACE;
  char* w = static_cast<char*>(ws);
  p.ws_status = reinterpret_cast<int*>(w);
  p.ws_count = reinterpret_cast<int*>(w + 256);
  p.ws_part = reinterpret_cast<float*>(w + 256 + align256(sizeof(int) * static_cast<size_t>(B) * p.Hkv));
  p.n_split = pl.n_split;
  p.tiles_per_split = pl.tiles_per_split;
  dim3 grid(pl.n_split, p.Hkv, B);
  kern<<<grid, kThreads, C::SMEM, st>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}

template <int KVDT, int SDT, int QDT>
int dispatch_nrep(int nrep, const Params& p, int B, void* ws, size_t wsb, cudaStream_t st) {
  switch (nrep) {
    case 1: return launch<1, KVDT, SDT, QDT>(p, B, ws, wsb, st);
    case 2: return launch<2, KVDT, SDT, QDT>(p, B, ws, wsb, st);
    case 4: return launch<4, KVDT, SDT, QDT>(p, B, ws, wsb, st);
    default: return HQ_ERR_UNSUPPORTED;
  }
}

inline bool aligned(const void* x, size_t a) { return reinterpret_cast<uintptr_t>(x) % a == 0; }

}  // namespace dec
}  // namespace hq

using namespace hq;
using namespace hq::dec;

extern "C" size_t hq_decode_workspace_bytes(int B, int Hq, int Hkv, int S, int D) {
  if (B < 0 || Hq < 0 || Hkv <= 0 || S < 0 || D != kD) return 0;
  return workspace_bytes(B, Hq, Hkv, S, current_sm_count());
}

static int check_common(const int64_t* q_strides, const int64_t* kv_strides,
                        const int64_t* out_strides, const float* partial_out, int B, int Hq,
                        int Hkv, int S, int D, const void* workspace) {
  if (!q_strides || !kv_strides || B < 0 || Hq <= 0 || Hkv <= 0 || S < 0)
    return HQ_ERR_INVALID_ARGUMENT;
  if (!partial_out && !out_strides) return HQ_ERR_INVALID_ARGUMENT;
  if (D != kD || Hq % Hkv) return HQ_ERR_UNSUPPORTED;
  if (q_strides[2] != 1 || kv_strides[2] != D || (out_strides && out_strides[2] != 1))
    return HQ_ERR_INVALID_ARGUMENT;
  if (!workspace || !aligned(workspace, 256)) return HQ_ERR_WORKSPACE;
  return HQ_OK;
}

extern "C" int hq_decode_int8(const void* q, int q_dtype, const int64_t q_strides[3],
                              const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                              const void* k_scale, const void* v_scale, int scale_dtype,
                              const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                              int Hq, int Hkv, int S, int D, float sm_scale, int q_quant,
                              void* out, const int64_t out_strides[3], float* partial_out,
                              void* workspace, size_t workspace_bytes, hq_stream_t stream) {
  int rc = check_common(q_strides, kv_strides, out_strides, partial_out, B, Hq, Hkv, S, D, workspace);
  if (rc != HQ_OK) return rc;
  // an empty cache (S == 0) may come with null K/V/v_scale pointers
  if (!q || !k_scale || !ksc_strides || !vsc_strides || (!out && !partial_out) ||
      (S > 0 && (!k || !v || !v_scale)))
    return HQ_ERR_INVALID_ARGUMENT;
  // token rows are copied in whole 64-token tiles: 16-byte aligned starts
  if (!aligned(k, 16) || !aligned(v, 16) || kv_strides[0] % 16 || kv_strides[1] % 16)
    return HQ_ERR_INVALID_ARGUMENT;
  if (B == 0) return HQ_OK;
  Params p{};
  p.q = q;
  p.qsb = q_strides[0];
  p.qsh = q_strides[1];
  p.k = reinterpret_cast<const char*>(k);
  p.v = reinterpret_cast<const char*>(v);
  p.kvsb = kv_strides[0];
  p.kvsh = kv_strides[1];
  p.ksc = k_scale;
  p.vsc = v_scale;
  p.kscb = ksc_strides[0];
  p.ksch = ksc_strides[1];
  p.kscd = ksc_strides[2];
  p.vscb = vsc_strides[0];
  p.vsch = vsc_strides[1];
  p.vscs = vsc_strides[2];
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.S = S;
  p.qk_scale = sm_scale * kLog2e;
  p.q_quant = q_quant;
  p.out = out;
  p.osb = out_strides ? out_strides[0] : 0;
  p.osh = out_strides ? out_strides[1] : 0;
  p.partial_out = partial_out;
  const int nrep = Hq / Hkv;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define HQ_Q(SDT)                                                                                \
  switch (q_dtype) {                                                                             \
    case HQ_DTYPE_BF16: return dispatch_nrep<HQ_DTYPE_I8, SDT, HQ_DTYPE_BF16>(nrep, p, B, workspace, workspace_bytes, st); \
    case HQ_DTYPE_F16: return dispatch_nrep<HQ_DTYPE_I8, SDT, HQ_DTYPE_F16>(nrep, p, B, workspace, workspace_bytes, st);   \
    case HQ_DTYPE_F32: return dispatch_nrep<HQ_DTYPE_I8, SDT, HQ_DTYPE_F32>(nrep, p, B, workspace, workspace_bytes, st);   \
    default: return HQ_ERR_UNSUPPORTED;                                                          \
  }
  if (scale_dtype == HQ_DTYPE_F16) {
    HQ_Q(HQ_DTYPE_F16)
  } else if (scale_dtype == HQ_DTYPE_F32) {
    HQ_Q(HQ_DTYPE_F32)
  }
#undef HQ_Q
  return HQ_ERR_UNSUPPORTED;
}

extern "C" int hq_decode_dense(const void* q, const int64_t q_strides[3], const void* k,
                               const void* v, int kv_dtype, const int64_t kv_strides[3], int B,
                               int Hq, int Hkv, int S, int D, float sm_scale, int q_quant,
                               void* out, const int64_t out_strides[3], float* partial_out,
                               void* workspace, size_t workspace_bytes, hq_stream_t stream) {
  int rc = check_common(q_strides, kv_strides, out_strides, partial_out, B, Hq, Hkv, S, D, workspace);
  if (rc != HQ_OK) return rc;
  if (!q || (!out && !partial_out) || (S > 0 && (!k || !v))) return HQ_ERR_INVALID_ARGUMENT;
  if (!aligned(k, 16) || !aligned(v, 16) || kv_strides[0] % 8 || kv_strides[1] % 8)
    return HQ_ERR_INVALID_ARGUMENT;
  if (B == 0) return HQ_OK;
  Params p{};
  p.q = q;
  p.qsb = q_strides[0];
  p.qsh = q_strides[1];
  p.k = static_cast<const char*>(k);
  p.v = static_cast<const char*>(v);
  p.kvsb = kv_strides[0];
  p.kvsh = kv_strides[1];
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.S = S;
  p.qk_scale = sm_scale * kLog2e;
  p.q_quant = q_quant;
  p.out = out;
  p.osb = out_strides ? out_strides[0] : 0;
  p.osh = out_strides ? out_strides[1] : 0;
  p.partial_out = partial_out;
  const int nrep = Hq / Hkv;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (kv_dtype) {
    case HQ_DTYPE_BF16:
      return dispatch_nrep<HQ_DTYPE_BF16, HQ_DTYPE_F32, HQ_DTYPE_BF16>(nrep, p, B, workspace, workspace_bytes, st);
    case HQ_DTYPE_F16:
      return dispatch_nrep<HQ_DTYPE_F16, HQ_DTYPE_F32, HQ_DTYPE_F16>(nrep, p, B, workspace, workspace_bytes, st);
    default:
      return HQ_ERR_UNSUPPORTED;
  }
}

extern "C" int hq_decode_combine(const float* parts, int n_parts, int64_t part_stride, int B,
                                 int Hq, int D, void* out, int out_dtype,
                                 const int64_t out_strides[3], hq_stream_t stream) {
  if (!parts || !out || !out_strides || n_parts < 1 || B < 0 || Hq <= 0) return HQ_ERR_INVALID_ARGUMENT;
  if (D != kD) return HQ_ERR_UNSUPPORTED;
  if (out_strides[2] != 1) return HQ_ERR_INVALID_ARGUMENT;
  if (B == 0) return HQ_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned blocks = static_cast<unsigned>(B * Hq);
  switch (out_dtype) {
    case HQ_DTYPE_BF16:
      combine_kernel<HQ_DTYPE_BF16><<<blocks, kThreads, 0, st>>>(parts, n_parts, part_stride, Hq, out, out_strides[0], out_strides[1]);
      break;
    case HQ_DTYPE_F16:
      combine_kernel<HQ_DTYPE_F16><<<blocks, kThreads, 0, st>>>(parts, n_parts, part_stride, Hq, out, out_strides[0], out_strides[1]);
      break;
    case HQ_DTYPE_F32:
      combine_kernel<HQ_DTYPE_F32><<<blocks, kThreads, 0, st>>>(parts, n_parts, part_stride, Hq, out, out_strides[0], out_strides[1]);
      break;
    default:
      return HQ_ERR_UNSUPPORTED;
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}
