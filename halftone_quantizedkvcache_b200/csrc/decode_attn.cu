// Split-KV decode attention over an int8 KV cache (sm_100a), its dense
// (bf16 / f16) twin and the log-sum-exp combine.
//
// Reference semantics: int8_decode_attn (src/kernels/int8_decode_attn_triton.py:15-63,
// 101-113) - dequantize K per channel and V per token, online float32 softmax,
// one query token - and the decode step of quantized_attention_forward
// (tests/qwen_kvcache_full.py:95-113), including its optional per-token fake
// quantization of q.  The reference launches one program per q head (16
// programs for the whole GPU).  Here, common to both kernels:
//
//   * the sequence is split: grid = (split, kv head, batch), split count chosen
//     on the host so that the grid fills every SM (batch 1 included);
//   * all n_rep = Hq / Hkv q heads of a kv head are served from one K/V tile;
//   * K/V tiles stream through a shared-memory ring filled by asynchronous
//     copies completing on mbarriers; every barrier wait is bounded;
//   * splits are combined in the same launch: each block writes (m, l, o) for
//     its split, and the last block of a (batch, kv head) to arrive - an atomic
//     ticket, no waiting - merges them and resets the ticket.
//
// decode_mma_kernel (int8 K/V, the hq_decode_int8 path) runs both dot products
// on the int8 tensor cores; decode_kernel (the dense twin, hq_decode_dense) uses
// CUDA-core packed f32x2 FMAs on 64-token tiles copied with 1-D bulk copies,
// each token owned by LPT = 2 * n_rep lanes.
#include "decode_common.cuh"

namespace hq {
namespace dec {

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
    finish_heads<NREP, QDT>(p, b, kvh, d, Ms, Ls, Os, peer_gen(p, b, kvh));
    return;
  }

  // ---- publish this split, then the last block of (b, kvh) merges all splits
#pragma unroll
  for (int r = 0; r < NREP; ++r) publish_split(p, b, kvh * NREP + r, split, d, Ms[r], Ls[r], Os[r]);
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int ticket = atomicAdd(p.ws_count + b * p.Hkv + kvh, 1);
    s_last = ticket == p.n_split - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  merge_splits<NREP, QDT>(p, b, kvh, reinterpret_cast<float*>(ring), C::SMEM_STAGES / 4,
                          peer_gen(p, b, kvh));
}

// ------------------------------------------------------------------ int8 tensor-core kernel
// The int8 decode kernel proper.  Same grid, split plan, partial format and
// last-block combine as the CUDA-core kernel above (which remains the dense
// bf16/f16 twin), but the two dot products run on the int8 tensor cores with
// exact integer accumulation:
//
//   scores  S[t, c] = sum_d K[t, d] * Qlimb[d, c]        mma.m16n8k32 s8 x s8 -> s32
//   output  O[d, c] = sum_t V[t, d] * Plimb[t, c]        (A = V^T via ldmatrix.trans)
//
// q' = q * k_scale * sm_scale * log2(e) and p' = p * v_scale are real-valued,
// so each is written as three balanced int8 limbs of a 24-bit fixed-point value
// (x24 = 65536 a + 256 b + c, |x24| <= 127 * 65793) with one float scale
// per head; the 8 n-columns of an MMA hold (a, b) and (c, 0) of two q heads.
// Scores are rebuilt exactly as sa * Sa + sb * Sb + sc * Sc in float32.  The
// PV products accumulate in int32 across tiles and are flushed into float32
// only when the running max or the limb scale of a head changes.
//
// K / V tiles of 128 tokens x 128 bytes arrive by tensor-map TMA with 128-byte
// swizzle (16-byte chunk c of row r stored at chunk c ^ (r % 8)), which makes
// every ldmatrix phase conflict-free.  4 warps per block, 32 tokens per warp
// per tile; each warp keeps its own online-softmax state.
namespace mmak {

template <int NREP>
struct MCfg {
  static constexpr int NT = (NREP + 1) / 2;               // n8 tiles, 2 heads each
  static constexpr int RING = kStagesM * 2 * kTileB;      // 96 KB
  static constexpr int LIMB = kWarps * NT * 8 * 32;       // p' limb staging
  static constexpr int QTAB = NT * 256 * 4;                // q' limb B-fragment words
  static constexpr int VSM = kStagesM * kTileT * 4;        // dynamic schedule: V scales per stage
  static_assert(RING % 1024 == 0 && (kTileT * 2) % 128 == 0, "V scale slots on 128-byte boundaries");
  static constexpr int SMEM =
      1024 + RING + NREP * kD * 4 + LIMB + 2 * kStagesM * 8 + QTAB + VSM + 16;
  static_assert(kWarps * NREP * kD * 4 + kWarps * NREP * 8 <= RING, "epilogue scratch");
};

// Fused append: counts this block on the grid ticket (in the workspace, after
// the status word) once all its threads have read the length; the last block of
// the grid advances the length by the appended token (unless the cache is full).
__device__ __forceinline__ void grid_arrive(const Params& p, int S) {
  int* ticket = p.ws_status + 32;
  __threadfence();  // this block's reads of the length come first
  const int total = static_cast<int>(gridDim.x * gridDim.y * gridDim.z);
  if (atomicAdd(ticket, 1) == total - 1) {
    *ticket = 0;
    if (S < p.S) *const_cast<int*>(p.seq_len) = S + 1;
  }
}

// The extra split of a fused append, one block per (b, kv head), thread d owns
// channel d: quantizes the new token exactly as hq_append_kv does (K per channel
// over this one token - its scale is not stored; V per token, scale stored in the
// cache's scale dtype), writes its codes at row S, and publishes the token's
// softmax partial for the NREP q heads - the score q'.K in float32 from the codes
// and the stored K scale, l = 1, o = V dequantized with the stored V scale - then
// takes the split ticket like every other split (and merges if it is last).
template <int NREP, int SDT, int QDT>
__device__ void append_split(const Params& p, int b, int kvh, int S, unsigned char* ring,
                             int scratch_floats, float (&red)[kWarps][NREP], int& s_last,
                             uint64_t* merge_bar) {
  using QE = Elem<QDT>;
  using SE = Elem<SDT>;
  const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
  const bool room = S < p.S;
  const float xk = QE::to_f32(reinterpret_cast<const typename QE::T*>(p.k_new)[b * p.knb + kvh * p.knh + d]);
  const float xv = QE::to_f32(reinterpret_cast<const typename QE::T*>(p.v_new)[b * p.vnb + kvh * p.vnh + d]);
  const float ks = SE::to_f32(reinterpret_cast<const typename SE::T*>(p.ksc)[b * p.kscb + kvh * p.ksch + d * p.kscd]);
  float qv[NREP];
#pragma unroll
  for (int r = 0; r < NREP; ++r)
    qv[r] = QE::to_f32(reinterpret_cast<const typename QE::T*>(p.q)[b * p.qsb + (kvh * NREP + r) * p.qsh + d]);
  // V row maximum and, with q_quant, the q row maxima (one reduction)
  __shared__ float vred[kWarps];
  {
    const float mv = warp_max(fabsf(xv), 1);
    if (lane == 0) vred[warp] = mv;
    if (p.q_quant) {
#pragma unroll
      for (int r = 0; r < NREP; ++r) {
        const float m = warp_max(fabsf(qv[r]), 1);
        if (lane == 0) red[warp][r] = m;
      }
    }
  }
  __syncthreads();
  if (p.seq_len && d == 32) grid_arrive(p, S);
  float mv = vred[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) mv = fmaxf(mv, vred[w]);
  // 16-bit inputs: the scale without a divide (exact for a 16-bit maximum) and the code
  // as the rint of the quotient with one FMA residual correction (exact for |x| <= that
  // maximum) - no divide and no branch on this block's path to the merge
  Quantizer qk, qvz;
  int ck, cv;
  if constexpr (QDT == HQ_DTYPE_F32) {
    qk = Quantizer::from_amax(fabsf(xk));
    qvz = Quantizer::from_amax(mv);
    ck = qk.code(xk);
    cv = qvz.code(xv);
  } else {
    qk = Quantizer::from_amax16(fabsf(xk));
    qvz = Quantizer::from_amax16(mv);
    auto code16 = [](const Quantizer& q, float x) {
      const float q0 = x * q.rcp;
      const float q1 = __fmaf_rn(__fmaf_rn(q0, -q.scale, x), q.rcp, q0);
      return __float_as_int(q1 + 12582912.0f) - 0x4B400000;
    };
    ck = code16(qk, xk);
    cv = code16(qvz, xv);
  }
  const typename SE::T vs_stored = SE::from_f32(qvz.scale);
  if (room) {
    int8_t* kc = const_cast<int8_t*>(reinterpret_cast<const int8_t*>(p.k)) + b * p.kvsb + kvh * p.kvsh +
                 static_cast<int64_t>(S) * kD + d;
    int8_t* vc = const_cast<int8_t*>(reinterpret_cast<const int8_t*>(p.v)) + b * p.kvsb + kvh * p.kvsh +
                 static_cast<int64_t>(S) * kD + d;
    *kc = static_cast<int8_t>(ck);
    *vc = static_cast<int8_t>(cv);
    if (d == 0) {
      auto* vsp = const_cast<typename SE::T*>(reinterpret_cast<const typename SE::T*>(p.vsc));
      vsp[b * p.vscb + kvh * p.vsch + static_cast<int64_t>(S) * p.vscs] = vs_stored;
    }
  } else if (d == 0) {
    report_error(p.ws_status, HQ_ERR_INVALID_ARGUMENT);
  }
  // scores of the new token (base 2), as the main splits define them
  if (p.q_quant) {
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      float m = red[0][r];
#pragma unroll
      for (int w = 1; w < kWarps; ++w) m = fmaxf(m, red[w][r]);
      const Quantizer qz = Quantizer::from_amax(m);
      qv[r] = QE::to_f32(QE::from_f32(static_cast<float>(qz.code(qv[r])) * qz.scale));
    }
  }
  __syncthreads();  // red is reused below
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    float part = qv[r] * ks * p.qk_scale * static_cast<float>(ck);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (lane == 0) red[warp][r] = part;
  }
  __syncthreads();
  float Ms[NREP], Ls[NREP], Os[NREP];
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    float sc = red[0][r];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) sc += red[w][r];
    Ms[r] = room ? sc : -INFINITY;
    Ls[r] = room ? 1.0f : 0.0f;
    Os[r] = room ? static_cast<float>(cv) * SE::to_f32(vs_stored) : 0.0f;
  }
  const int split = p.n_split - 1;
#pragma unroll
  for (int r = 0; r < NREP; ++r) publish_split(p, b, kvh * NREP + r, split, d, Ms[r], Ls[r], Os[r]);
  __syncthreads();
  if (d == 0) s_last = ticket_add(p.ws_count + b * p.Hkv + kvh) == p.n_split - 1;
  __syncthreads();
  if (!s_last) return;
  if (d == 0) p.ws_next[b * p.Hkv + kvh] = 0;  // (dynamic schedule) every split has stopped claiming
  merge_splits<NREP, QDT>(p, b, kvh, reinterpret_cast<float*>(ring), scratch_floats, 0u,
                          merge_bar);
}

// DYN: the dynamic tile schedule.  The ntiles tiles of (b, kvh) are shared out
// among its n_main splits as they go: split j first streams tiles
// j + k * n_main for k < kStatic (no atomics), then claims tile
// kStatic * n_main + c with c = atomicAdd(next, 1) until none are left, so a
// block whose copies were served late simply takes fewer.  Each stage carries
// its tile index (-1: the block's run has ended) and the tile's V scales, copied
// by a third tensor map with the tile.  The split partials then cover timing-
// dependent tile sets: the result is the same attention with float32 sums
// grouped differently from call to call (not bit-reproducible).
template <int NREP, int SDT, int QDT, bool DYN>
__global__ void __launch_bounds__(kThreads, 2) decode_mma_kernel(
    const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
    const __grid_constant__ CUtensorMap tmvs, const Params p) {
  using C = MCfg<NREP>;
  using QE = Elem<QDT>;
  using SE = Elem<SDT>;
  constexpr int NT = C::NT;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* ring = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // V scale slots of the stages (DYN) right after the ring: a tensor copy's
  // destination must start on a 128-byte boundary (each slot is 512 or 256 bytes)
  auto* vsm = reinterpret_cast<typename SE::T*>(ring + C::RING);  // [kStagesM][kTileT]
  float* qs = reinterpret_cast<float*>(ring + C::RING + C::VSM);
  unsigned char* plimb = reinterpret_cast<unsigned char*>(qs + NREP * kD);
  uint64_t* full = reinterpret_cast<uint64_t*>(plimb + C::LIMB);
  uint64_t* empty = full + kStagesM;
  uint32_t* qtab = reinterpret_cast<uint32_t*>(empty + kStagesM);
  int* stile = reinterpret_cast<int*>(qtab + NT * 256);
  __shared__ float red[kWarps][NREP];
  __shared__ float qmax_s[NREP];
  __shared__ int s_last;
  __shared__ __align__(8) uint64_t merge_bar;  // bulk loads of the split partials

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
  if (tid == 0) {
    mbar_init(&merge_bar, 1);
    fence_mbar_init();
  }
  // an overlapped launch after this one may be scheduled now: its blocks take
  // the slots of this grid's blocks as they exit, and wait for this grid's
  // completion before reading q or writing anything
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const unsigned gen0 = peer_gen(p, b, kvh);
  int S = p.S, tps = p.tiles_per_split;
  if (p.seq_len) {
    S = min(max(__ldcg(p.seq_len), 0), p.S);
    const int n_main = p.k_new ? p.n_split - 1 : p.n_split;
    tps = max(1, ((S + kTileT - 1) / kTileT + n_main - 1) / n_main);
  }
  if (p.k_new && split == p.n_split - 1) {
    append_split<NREP, SDT, QDT>(p, b, kvh, S, ring, C::RING / 4, red, s_last, &merge_bar);
    return;
  }
  const int s_begin = split * tps * kTileT;
  const int s_end = min(S, s_begin + tps * kTileT);
  const int ntok = max(0, s_end - s_begin);
  const int ntiles = (ntok + kTileT - 1) / kTileT;

  int issued = 0;
  const uint64_t pol_stream = l2_evict_first();
  // dynamic schedule (tid 0): fixed part, claims, and the tile of iteration k
  const int n_main = p.k_new ? p.n_split - 1 : p.n_split;
  const int ntiles_all = (S + kTileT - 1) / kTileT;
  int* next_ctr = p.ws_next + b * p.Hkv + kvh;
  int claim = -1;  // tid 0 (DYN): the claim made one refill ahead (-1: none)
  auto fixed_tile = [&](int k) {
    const int t = split + k * n_main;
    return t < ntiles_all ? t : -1;
  };
  // requests iteration t's tile into its stage: static - tile t of this split's run;
  // DYN - absolute tile `tabs` (-1: no tile, the stage only carries the end mark)
  auto issue = [&](int t, int tabs = 0) {
    const int st = t % kStagesM;
    unsigned char* dst = ring + st * 2 * kTileB;
    if constexpr (DYN) {
      stile[st] = tabs;
      if (tabs < 0) {
        mbar_arrive(&full[st]);
        return;
      }
      mbar_arrive_expect_tx(&full[st], 2 * kTileB + kTileT * SE::kBytes);
      tma_load_4d(dst, &tmk, 0, tabs * kTileT, kvh, b, &full[st], pol_stream);
      tma_load_4d(dst + kTileB, &tmv, 0, tabs * kTileT, kvh, b, &full[st], pol_stream);
      tma_load_3d(vsm + st * kTileT, &tmvs, tabs * kTileT, kvh, b, &full[st], pol_stream);
    } else {
      mbar_arrive_expect_tx(&full[st], 2 * kTileB);
      tma_load_4d(dst, &tmk, 0, s_begin + t * kTileT, kvh, b, &full[st], pol_stream);
      tma_load_4d(dst + kTileB, &tmv, 0, s_begin + t * kTileT, kvh, b, &full[st], pol_stream);
    }
    issued = t + 1;
  };
  // V scales of this lane's own tokens (row g for even t4, g + 8 for odd t4, of
  // both 16-row blocks), loaded two tiles ahead so their latency stays hidden
  const auto* vscp = reinterpret_cast<const typename SE::T*>(p.vsc);
  const int64_t vsc_row = b * p.vscb + kvh * p.vsch;
  auto load_vs = [&](int t, float (&v)[2]) {
#pragma unroll
    for (int rb = 0; rb < 2; ++rb) {
      const int tok = t * kTileT + warp * 32 + rb * 16 + g + 8 * (t4 & 1);
      v[rb] = tok < ntok ? SE::to_f32(vscp[vsc_row + static_cast<int64_t>(s_begin + tok) * p.vscs]) : 0.0f;
    }
  };
  // The small loads (q, K scales, first V scales) go out before this block's
  // first TMA copy and only one stage is requested until q' is ready: the
  // grid's opening burst of tile copies would otherwise queue ahead of them.
  // Overlapped launches instead request every stage and the V scales while
  // the previous kernel finishes, and load q and the K scales after it.
  const int d = tid;
  typename SE::T ks_raw;
  typename QE::T q_raw[NREP];
  auto load_q = [&] {
    const auto* qp = reinterpret_cast<const typename QE::T*>(p.q);
    const auto* kp = reinterpret_cast<const typename SE::T*>(p.ksc);
    ks_raw = kp[b * p.kscb + kvh * p.ksch + d * p.kscd];
#pragma unroll
    for (int r = 0; r < NREP; ++r) q_raw[r] = qp[b * p.qsb + (kvh * NREP + r) * p.qsh + d];
  };
  if (!p.overlap) load_q();
  float vs_a[2] = {0.0f, 0.0f}, vs_b[2] = {0.0f, 0.0f};
  if constexpr (!DYN) {
    load_vs(0, vs_a);
    load_vs(1, vs_b);
  }
  if (tid == 0) {
    for (int s = 0; s < kStagesM; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    fence_mbar_init();
  }
  // zero the p' staging (columns 3 and 7 stay zero)
  for (int i = tid; i < C::LIMB / 4; i += kThreads) reinterpret_cast<uint32_t*>(plimb)[i] = 0;
  __syncthreads();
  if (tid == 0) {
    if constexpr (DYN) {
      for (int t = 0; t < (p.overlap ? kStagesM : 1); ++t) issue(t, fixed_tile(t));
    } else {
      for (int t = 0; t < min(p.overlap ? kStagesM : 1, ntiles); ++t) issue(t);
    }
  }
  if (p.k_new && tid == 32) grid_arrive(p, S);  // every thread has read the length
  if (p.overlap) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    load_q();
  }

  // ---- q prologue: q' = q_in * k_scale * sm_scale * log2(e), thread owns channel d
  {
    const float ks = SE::to_f32(ks_raw);
    float qv[NREP];
#pragma unroll
    for (int r = 0; r < NREP; ++r) qv[r] = QE::to_f32(q_raw[r]);
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
      __syncthreads();
    }
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      const float v = qv[r] * ks * p.qk_scale;
      qs[r * kD + d] = v;
      const float m = warp_max(fabsf(v), 1);
      if (lane == 0) red[warp][r] = m;
    }
    __syncthreads();
    if (tid < NREP) {
      float m = red[0][tid];
#pragma unroll
      for (int w = 1; w < kWarps; ++w) m = fmaxf(m, red[w][tid]);
      qmax_s[tid] = m;
    }
    __syncthreads();
  }
  if (tid == 0) {
    if constexpr (DYN) {
      if (!p.overlap)
        for (int t = 1; t < kStagesM; ++t) issue(t, fixed_tile(t));
      // the first claim, after any wait for the previous grid (whose merging blocks reset the counters)
      if (fixed_tile(kStatic - 1) >= 0) claim = atomicAdd(next_ctr, 1);
    } else if (!p.overlap) {
      for (int t = 1; t < min(kStagesM, ntiles); ++t) issue(t);
    }
  }

  // q' limb B-fragments, built by the whole block into qtab: word
  // (nt, j, hh, lane g * 4 + t4) packs limb g % 4 of head 2 nt + g / 4 at the four
  // channels 32 j + 16 hh + 4 t4 + e (a compact loop: this code runs once per block)
#pragma unroll 1
  for (int i = tid; i < NT * 256; i += kThreads) {
    const int nt = i >> 8, j = (i >> 6) & 3, hh = (i >> 5) & 1, gg = (i >> 2) & 7, tt = i & 3;
    const int col_head = 2 * nt + (gg >> 2), col_limb = gg & 3;
    uint32_t w = 0;
    if (col_head < NREP && col_limb < 3) {
      const float qm = qmax_s[col_head];
      const float inv = qm > 0.0f ? kLimbMax / qm : 0.0f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int dd = 32 * j + 16 * hh + 4 * tt + e;
        const int x = max(-static_cast<int>(kLimbMax),
                          min(static_cast<int>(kLimbMax), __float2int_rn(qs[col_head * kD + dd] * inv)));
        w |= limb_byte(x, col_limb) << (8 * e);
      }
    }
    qtab[i] = w;
  }
  __syncthreads();
  // per lane: its B-fragments, per n-tile and k-step; score factors
  uint32_t bq[NT][4][2];
  float f0[NT], f1[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) bq[nt][j][hh] = qtab[(nt << 8) | (j << 6) | (hh << 5) | lane];
    const int my_head = 2 * nt + (t4 >> 1);
    const float qsc = my_head < NREP && qmax_s[my_head] > 0.0f ? qmax_s[my_head] / kLimbMax : 0.0f;
    f0[nt] = (t4 & 1) ? qsc : qsc * 65536.0f;
    f1[nt] = (t4 & 1) ? 0.0f : qsc * 256.0f;
  }

  // running state per n-tile (this lane's head 2*nt + t4/2)
  float m_run[NT], l_run[NT], pmax[NT], o_acc[NT][4][2][2];
  int acc[NT][4][2][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_run[nt] = -INFINITY;
    l_run[nt] = 0.0f;
    pmax[nt] = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int pi = 0; pi < 2; ++pi) {
        o_acc[nt][j][pi][0] = o_acc[nt][j][pi][1] = 0.0f;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][j][pi][e] = 0;
      }
  }
  // flush the int32 PV sums of n-tile nt into float (lanes where do_flush)
  auto flush = [&](int nt, bool do_flush) {
    const float ps = pmax[nt] / kLimbMax;
    const float F0 = (t4 & 1) ? ps : ps * 65536.0f;
    const float F1 = (t4 & 1) ? 0.0f : ps * 256.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int pi = 0; pi < 2; ++pi) {
        float lo = F0 * static_cast<float>(acc[nt][j][pi][0]) + F1 * static_cast<float>(acc[nt][j][pi][1]);
        float hi = F0 * static_cast<float>(acc[nt][j][pi][2]) + F1 * static_cast<float>(acc[nt][j][pi][3]);
        lo += __shfl_xor_sync(0xffffffffu, lo, 1);
        hi += __shfl_xor_sync(0xffffffffu, hi, 1);
        if (do_flush) {
          o_acc[nt][j][pi][0] += lo;
          o_acc[nt][j][pi][1] += hi;
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[nt][j][pi][e] = 0;
        }
      }
  };

  unsigned char* my_limb = plimb + warp * NT * 256;
  bool ok = true;
  int consumed = 0;
  // tokens: static - relative to the split's first token; DYN - absolute
  const int tok_limit = DYN ? S : ntok;
  for (int t = 0; DYN || t < ntiles; ++t) {
    const int st = t % kStagesM;
    const uint32_t par = (t / kStagesM) & 1;
    float vsf[2];
    bool own_ok[2];
    int base_tok;
    if constexpr (DYN) {
      if (!mbar_wait(&full[st], par)) {
        ok = false;
        break;
      }
      const int tabs = stile[st];
      if (tabs < 0) break;  // the block's run has ended (the same stage for every warp)
      base_tok = tabs * kTileT + warp * 32;
#pragma unroll
      for (int rb = 0; rb < 2; ++rb) {
        const int i = warp * 32 + rb * 16 + g + 8 * (t4 & 1);  // this lane's own token
        own_ok[rb] = tabs * kTileT + i < S;
        vsf[rb] = SE::to_f32(vsm[st * kTileT + i]);
      }
    } else {
      base_tok = t * kTileT + warp * 32;  // first token of this warp (within split)
#pragma unroll
      for (int rb = 0; rb < 2; ++rb) {
        own_ok[rb] = base_tok + rb * 16 + g + 8 * (t4 & 1) < ntok;
        vsf[rb] = vs_a[rb];
        vs_a[rb] = vs_b[rb];
      }
      load_vs(t + 2, vs_b);
      if (!mbar_wait(&full[st], par)) {
        ok = false;
        break;
      }
    }
    consumed = t + 1;
    const uint32_t kt = smem_u32(ring + st * 2 * kTileB);
    const uint32_t vt = kt + kTileB;

    // ---- scores: 2 row blocks of 16 tokens x 4 k-steps of 32 channels
    float sc[NT][2][2];  // [nt][rb][lo=row g, hi=row g+8]
#pragma unroll
    for (int rb = 0; rb < 2; ++rb) {
      int sacc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sacc[nt][e] = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int mat = lane >> 3;
        const int row = warp * 32 + rb * 16 + (mat & 1) * 8 + (lane & 7);
        uint32_t a[4];
        ldsm_x4(kt + swz(row, 2 * j + (mat >> 1)), a);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_s8(sacc[nt], a, bq[nt][j][0], bq[nt][j][1]);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float lo = f0[nt] * static_cast<float>(sacc[nt][0]) + f1[nt] * static_cast<float>(sacc[nt][1]);
        float hi = f0[nt] * static_cast<float>(sacc[nt][2]) + f1[nt] * static_cast<float>(sacc[nt][3]);
        lo += __shfl_xor_sync(0xffffffffu, lo, 1);
        hi += __shfl_xor_sync(0xffffffffu, hi, 1);
        const int tok = base_tok + rb * 16 + g;
        sc[nt][rb][0] = tok < tok_limit ? lo : -INFINITY;
        sc[nt][rb][1] = tok + 8 < tok_limit ? hi : -INFINITY;
      }
    }
    // ---- online softmax per head; p' limbs of this lane's own two tokens
    __syncwarp();  // the previous tile's limb reads are done
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float mt = fmaxf(fmaxf(sc[nt][0][0], sc[nt][0][1]), fmaxf(sc[nt][1][0], sc[nt][1][1]));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
      const float m_new = fmaxf(m_run[nt], mt);
      float pr[2], pv[2];
      float pm = 0.0f;
#pragma unroll
      for (int rb = 0; rb < 2; ++rb) {
        const float sown = (t4 & 1) ? sc[nt][rb][1] : sc[nt][rb][0];
        pr[rb] = own_ok[rb] ? exp2f(sown - m_new) : 0.0f;
        pv[rb] = pr[rb] * vsf[rb];
        pm = fmaxf(pm, pv[rb]);
      }
      pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 1));
      pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 4));
      pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 8));
      pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 16));
      const bool rescale = m_new > m_run[nt];
      const bool grow = pm > pmax[nt];
      if (__any_sync(0xffffffffu, rescale || grow)) {
        flush(nt, rescale || grow);
        if (rescale) {
          const float alpha = exp2f(m_run[nt] - m_new);  // 0 on the first tile
          l_run[nt] *= alpha;
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int pi = 0; pi < 2; ++pi) {
              o_acc[nt][j][pi][0] *= alpha;
              o_acc[nt][j][pi][1] *= alpha;
            }
        }
        if (grow) pmax[nt] = 2.0f * pm;
      }
      m_run[nt] = m_new;
      l_run[nt] += pr[0] + pr[1];
      const float inv_ps = pmax[nt] > 0.0f ? kLimbMax / pmax[nt] : 0.0f;
      const int hh = t4 >> 1;
      unsigned char* dst = my_limb + nt * 256;
#pragma unroll
      for (int rb = 0; rb < 2; ++rb) {
        const int x = min(__float2int_rn(pv[rb] * inv_ps), static_cast<int>(kLimbMax));
        int la, lb, lc;
        limbs24(x, la, lb, lc);
        const int k = pv_k(rb * 16 + g + 8 * (t4 & 1));
        dst[(4 * hh + 0) * 32 + k] = static_cast<unsigned char>(la);
        dst[(4 * hh + 1) * 32 + k] = static_cast<unsigned char>(lb);
        dst[(4 * hh + 2) * 32 + k] = static_cast<unsigned char>(lc);
      }
    }
    __syncwarp();
    // ---- PV: A = V^T (ldmatrix.trans + byte permute), B = p' limbs
    uint32_t bp[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const unsigned char* src = my_limb + nt * 256 + g * 32;
      bp[nt][0] = *reinterpret_cast<const uint32_t*>(src + 4 * t4);
      bp[nt][1] = *reinterpret_cast<const uint32_t*>(src + 16 + 4 * t4);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t ae[4], ao[4];
#pragma unroll
      for (int th = 0; th < 2; ++th) {
        const int mat = lane >> 3;
        const int row = warp * 32 + th * 16 + (mat & 1) * 8 + (lane & 7);
        uint32_t r[4];
        ldsm_x4_t(vt + swz(row, 2 * j + (mat >> 1)), r);
        ae[2 * th + 0] = prmt(r[0], r[1], 0x6420u);
        ao[2 * th + 0] = prmt(r[0], r[1], 0x7531u);
        ae[2 * th + 1] = prmt(r[2], r[3], 0x6420u);
        ao[2 * th + 1] = prmt(r[2], r[3], 0x7531u);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma_s8(acc[nt][j][0], ae, bp[nt][0], bp[nt][1]);
        mma_s8(acc[nt][j][1], ao, bp[nt][0], bp[nt][1]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if constexpr (DYN) {
      if (tid == 0) {
        if (!mbar_wait(&empty[st], par)) {
          ok = false;
          break;
        }
        // iteration t + kStagesM: its fixed tile, or the claim made one refill ago (then
        // the claim for the next refill goes out, its latency hidden by a tile's time)
        const int k = t + kStagesM;
        int tabs;
        if (k < kStatic) {
          tabs = fixed_tile(k);
        } else {
          tabs = claim >= 0 && kStatic * n_main + claim < ntiles_all ? kStatic * n_main + claim : -1;
        }
        issue(k, tabs);
        if (k >= kStatic) claim = tabs >= 0 ? atomicAdd(next_ctr, 1) : -1;
      }
    } else if (tid == 0 && t + kStagesM < ntiles) {
      if (!mbar_wait(&empty[st], par)) {
        ok = false;
        break;
      }
      issue(t + kStagesM);
    }
  }
  if (!ok) {
    report_error(p.ws_status, HQ_ERR_DEVICE_TIMEOUT);
    if (tid == 0)
      for (int t = consumed; t < issued; ++t) mbar_wait(&full[t % kStagesM], (t / kStagesM) & 1);
  }
  __syncthreads();
  if (__syncthreads_or(!ok)) return;

  // ---- block epilogue: flush, then merge the 4 warps
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) flush(nt, true);
  float* wo = reinterpret_cast<float*>(ring);                 // [kWarps][NREP][kD]
  float* wl = wo + kWarps * NREP * kD;                        // [kWarps][NREP]
  float* wm = wl + kWarps * NREP;                             // [kWarps][NREP]
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int h = 2 * nt + (t4 >> 1);
    float l = l_run[nt];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 4);
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
    if (h < NREP) {
      float* dst = wo + (warp * NREP + h) * kD;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int pi = 0; pi < 2; ++pi) {
          // even lane writes the row-g channel, odd lane the row-g+8 channel
          const int d = 32 * j + 2 * g + pi + 16 * (t4 & 1);
          dst[d] = (t4 & 1) ? o_acc[nt][j][pi][1] : o_acc[nt][j][pi][0];
        }
      if (g == 0 && (t4 & 1) == 0) {
        wl[warp * NREP + h] = l;
        wm[warp * NREP + h] = m_run[nt];
      }
    }
  }
  __syncthreads();
  float Ms[NREP], Ls[NREP], Os[NREP];
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    float M = wm[r];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) M = fmaxf(M, wm[w * NREP + r]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mw = wm[w * NREP + r];
      const float f = mw == -INFINITY ? 0.0f : exp2f(mw - M);
      L += wl[w * NREP + r] * f;
      O += wo[(w * NREP + r) * kD + d] * f;
    }
    Ms[r] = M;
    Ls[r] = L;
    Os[r] = O;
  }
  if (p.n_split == 1) {
    if (DYN && tid == 0) *next_ctr = 0;  // ready for the next launch
    finish_heads<NREP, QDT>(p, b, kvh, d, Ms, Ls, Os, gen0);
    return;
  }
#pragma unroll
  for (int r = 0; r < NREP; ++r) publish_split(p, b, kvh * NREP + r, split, d, Ms[r], Ls[r], Os[r]);
  __syncthreads();
  if (tid == 0) s_last = ticket_add(p.ws_count + b * p.Hkv + kvh) == p.n_split - 1;
  __syncthreads();
  if (!s_last) return;
  if (DYN && tid == 0) *next_ctr = 0;  // every split has stopped claiming
  merge_splits<NREP, QDT>(p, b, kvh, reinterpret_cast<float*>(ring), C::RING / 4, gen0,
                          &merge_bar);
}

}  // namespace mmak

// ------------------------------------------------------------------ dense tensor-core twin
// The bf16 / f16 twin of decode_mma_kernel with the same design: 128-token K/V
// tiles by tensor-map TMA into a 3-stage mbarrier ring (each 256-byte token row
// arrives as two 128-byte-swizzled halves of 64 channels), the same grid, split
// plan, split ticket and merge, 4 warps with 32 tokens each per tile and their
// own online softmax.  Only the element type changes: the two products run on
// the 16-bit tensor cores (mma.sync m16n8k16, float32 accumulation) instead of
// the int8 ones, with no scales:
//
//   scores  S[t, c] = sum_d K[t, d] * Q[d, c]   q in the K/V dtype, exact; column c
//                                               holds q head c % NREP, so every lane
//                                               owns scores of real heads
//   output  O[d, c] = sum_t V[t, d] * P[t, c]   A = V^T by ldmatrix.trans; column
//                                               2h + i holds the high (i = 0) or low
//                                               (i = 1) 16-bit part of head h's
//                                               probabilities (about 16 bits)
//
// Per K/V byte it moves twice what the int8 kernel moves, so with the same
// bytes in flight per SM it runs one block per SM (192 KB of ring).
namespace mmab {

constexpr int kTileT = 128;
constexpr int kHalfB = kTileT * 128;  // 16 KB: 128 tokens x 64 channels x 2 bytes
constexpr int kTileB = 2 * kHalfB;    // 32 KB per K or V tile
constexpr int kStagesB = 3;
constexpr int kPCol = 40;             // P staging column stride (16-bit words): conflict-free reads

template <int NREP>
struct BCfg {
  static constexpr int RING = kStagesB * 2 * kTileB;   // 192 KB
  static constexpr int PST = kWarps * 8 * kPCol * 2;   // per warp [8 columns][kPCol] 16-bit
  static constexpr int QSM = NREP * kD * 2;            // q in the K/V dtype
  static constexpr int SMEM = 1024 + RING + PST + QSM + 2 * kStagesB * 8;
  static_assert(kWarps * NREP * kD * 4 + kWarps * NREP * 8 <= RING, "epilogue scratch");
};

template <int KVDT>
__device__ __forceinline__ void mma_16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                       uint32_t b1) {
  if constexpr (KVDT == HQ_DTYPE_BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

template <int KVDT>
__device__ __forceinline__ uint16_t bits16(float x) {
  using E = Elem<KVDT>;
  const typename E::T v = E::from_f32(x);
  return *reinterpret_cast<const uint16_t*>(&v);
}

template <int NREP, int KVDT>
__global__ void __launch_bounds__(kThreads, 1) decode_dense_mma_kernel(
    const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
    const Params p) {
  using C = BCfg<NREP>;
  using E = Elem<KVDT>;  // q has the K/V dtype
  extern __shared__ unsigned char smem_raw[];
  unsigned char* ring = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint16_t* pst = reinterpret_cast<uint16_t*>(ring + C::RING);
  uint16_t* qsm = pst + kWarps * 8 * kPCol;
  uint64_t* full = reinterpret_cast<uint64_t*>(qsm + NREP * kD);
  uint64_t* empty = full + kStagesB;
  __shared__ float red[kWarps][NREP];
  __shared__ int s_last;
  __shared__ __align__(8) uint64_t merge_bar;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
  const int d = tid;
  const int S = p.S, tps = p.tiles_per_split;
  const int s_begin = split * tps * kTileT;
  const int ntok = max(0, min(S, s_begin + tps * kTileT) - s_begin);
  const int ntiles = (ntok + kTileT - 1) / kTileT;

  const uint64_t pol_stream = mmak::l2_evict_first();
  int issued = 0;
  auto issue = [&](int t) {
    const int st = t % kStagesB;
    unsigned char* dst = ring + st * 2 * kTileB;
    const int y = s_begin + t * kTileT;
    mbar_arrive_expect_tx(&full[st], 2 * kTileB);
    mmak::tma_load_4d(dst, &tmk, 0, y, kvh, b, &full[st], pol_stream);
    mmak::tma_load_4d(dst + kHalfB, &tmk, 64, y, kvh, b, &full[st], pol_stream);
    mmak::tma_load_4d(dst + kTileB, &tmv, 0, y, kvh, b, &full[st], pol_stream);
    mmak::tma_load_4d(dst + kTileB + kHalfB, &tmv, 64, y, kvh, b, &full[st], pol_stream);
    issued = t + 1;
  };
  const auto* qp = reinterpret_cast<const typename E::T*>(p.q);
  float qv[NREP];
#pragma unroll
  for (int r = 0; r < NREP; ++r) qv[r] = E::to_f32(qp[b * p.qsb + (kvh * NREP + r) * p.qsh + d]);
  if (tid == 0) {
    for (int s = 0; s < kStagesB; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    mbar_init(&merge_bar, 1);
    fence_mbar_init();
  }
  for (int i = tid; i < kWarps * 8 * kPCol; i += kThreads) pst[i] = 0;  // padding columns stay 0
  __syncthreads();
  if (tid == 0)
    for (int t = 0; t < min(kStagesB, ntiles); ++t) issue(t);

  // ---- q prologue: the reference's per-token fake quantization (q_quant), q kept
  // in the K/V dtype (exact), staged for the B fragments
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
      qv[r] = static_cast<float>(qz.code(qv[r])) * qz.scale;
    }
  }
#pragma unroll
  for (int r = 0; r < NREP; ++r) qsm[r * kD + d] = bits16<KVDT>(qv[r]);
  __syncthreads();
  // B fragments of q: column g holds head g % NREP; k-step j covers channels 16 j .. 16 j + 15
  uint32_t bq[8][2];
  {
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(qsm + (g % NREP) * kD);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      bq[j][0] = qw[8 * j + t4];
      bq[j][1] = qw[8 * j + 4 + t4];
    }
  }

  float m_run[NREP], l_run[NREP], o_acc[8][4];
#pragma unroll
  for (int h = 0; h < NREP; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.0f;
  }
#pragma unroll
  for (int m = 0; m < 8; ++m)
#pragma unroll
    for (int e = 0; e < 4; ++e) o_acc[m][e] = 0.0f;
  uint16_t* my_p = pst + warp * 8 * kPCol;

  bool ok = true;
  int consumed = 0;
  for (int t = 0; t < ntiles; ++t) {
    const int st = t % kStagesB;
    const uint32_t par = (t / kStagesB) & 1;
    if (!mbar_wait(&full[st], par)) {
      ok = false;
      break;
    }
    consumed = t + 1;
    const uint32_t kt = smem_u32(ring + st * 2 * kTileB);
    const uint32_t vt = kt + kTileB;
    const int base_tok = t * kTileT + warp * 32;  // within the split

    // ---- scores: 2 row blocks of 16 tokens x 8 k-steps of 16 channels
    float sc[2][4];  // [rb]: (token g, column 2 t4), (g, 2 t4 + 1), (g + 8, 2 t4), (g + 8, 2 t4 + 1)
#pragma unroll
    for (int rb = 0; rb < 2; ++rb) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int mat = lane >> 3;
        const int row = warp * 32 + rb * 16 + (mat & 1) * 8 + (lane & 7);
        uint32_t a[4];
        mmak::ldsm_x4(kt + (j >> 2) * kHalfB + mmak::swz(row, (j & 3) * 2 + (mat >> 1)), a);
        mma_16<KVDT>(acc, a, bq[j][0], bq[j][1]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = base_tok + rb * 16 + g + 8 * (e >> 1);
        sc[rb][e] = tok < ntok ? acc[e] * p.qk_scale : -INFINITY;
      }
    }
    // ---- online softmax per head (every lane keeps every head's state)
    float alpha[NREP], m_new[NREP];
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      float mt = -INFINITY;
#pragma unroll
      for (int rb = 0; rb < 2; ++rb)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if ((2 * t4 + (e & 1)) % NREP == h) mt = fmaxf(mt, sc[rb][e]);
      mt = warp_max(mt, 1);
      m_new[h] = fmaxf(m_run[h], mt);
      alpha[h] = m_new[h] == -INFINITY ? 1.0f : exp2f(m_run[h] - m_new[h]);
      m_run[h] = m_new[h];
      l_run[h] *= alpha[h];
    }
    // probabilities of the first replica of each head (column < NREP) into the staging
    __syncwarp();  // the previous tile's P reads are done
#pragma unroll
    for (int rb = 0; rb < 2; ++rb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = 2 * t4 + (e & 1);
        if (col < NREP) {
          float mh = m_new[0];
#pragma unroll
          for (int h = 1; h < NREP; ++h)
            if (col == h) mh = m_new[h];
          const float pr = sc[rb][e] == -INFINITY ? 0.0f : exp2f(sc[rb][e] - mh);
#pragma unroll
          for (int h = 0; h < NREP; ++h)
            if (col == h) l_run[h] += pr;
          const uint16_t hi = bits16<KVDT>(pr);
          typename E::T hv = *reinterpret_cast<const typename E::T*>(&hi);
          const uint16_t lo = bits16<KVDT>(pr - E::to_f32(hv));
          const int tk = rb * 16 + g + 8 * (e >> 1);
          my_p[(2 * col) * kPCol + tk] = hi;
          my_p[(2 * col + 1) * kPCol + tk] = lo;
        }
      }
    // rescale this lane's output columns (head t4, its high and low parts)
    if (t4 < NREP) {
      float a = alpha[0];
#pragma unroll
      for (int h = 1; h < NREP; ++h)
        if (t4 == h) a = alpha[h];
      if (a != 1.0f) {
#pragma unroll
        for (int m = 0; m < 8; ++m)
#pragma unroll
          for (int e = 0; e < 4; ++e) o_acc[m][e] *= a;
      }
    }
    __syncwarp();
    // ---- PV: A = V^T (ldmatrix.trans), B = P parts; 8 channel tiles x 2 token steps
    uint32_t bp[2][2];
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(my_p + g * kPCol + 16 * kk);
      bp[kk][0] = pw[t4];
      bp[kk][1] = pw[4 + t4];
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) {
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const int mat = lane >> 3;
        const int row = warp * 32 + kk * 16 + (mat >> 1) * 8 + (lane & 7);
        uint32_t a[4];
        mmak::ldsm_x4_t(vt + (m >> 2) * kHalfB + mmak::swz(row, (m & 3) * 2 + (mat & 1)), a);
        mma_16<KVDT>(o_acc[m], a, bp[kk][0], bp[kk][1]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (tid == 0 && t + kStagesB < ntiles) {
      if (!mbar_wait(&empty[st], par)) {
        ok = false;
        break;
      }
      issue(t + kStagesB);
    }
  }
  if (!ok) {
    report_error(p.ws_status, HQ_ERR_DEVICE_TIMEOUT);
    if (tid == 0)
      for (int t = consumed; t < issued; ++t) mbar_wait(&full[t % kStagesB], (t / kStagesB) & 1);
  }
  __syncthreads();
  if (__syncthreads_or(!ok)) return;

  // ---- block epilogue: the 4 warps' states into shared memory, merged per channel
  float* wo = reinterpret_cast<float*>(ring);  // [kWarps][NREP][kD]
  float* wl = wo + kWarps * NREP * kD;         // [kWarps][NREP]
  float* wm = wl + kWarps * NREP;              // [kWarps][NREP]
#pragma unroll
  for (int h = 0; h < NREP; ++h) {
    float l = l_run[h];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      wl[warp * NREP + h] = l;
      wm[warp * NREP + h] = m_run[h];
    }
  }
  if (t4 < NREP) {
    float* dst = wo + (warp * NREP + t4) * kD;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      dst[16 * m + g] = o_acc[m][0] + o_acc[m][1];
      dst[16 * m + g + 8] = o_acc[m][2] + o_acc[m][3];
    }
  }
  __syncthreads();
  float Ms[NREP], Ls[NREP], Os[NREP];
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    float M = wm[r];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) M = fmaxf(M, wm[w * NREP + r]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mw = wm[w * NREP + r];
      const float f = mw == -INFINITY ? 0.0f : exp2f(mw - M);
      L += wl[w * NREP + r] * f;
      O += wo[(w * NREP + r) * kD + d] * f;
    }
    Ms[r] = M;
    Ls[r] = L;
    Os[r] = O;
  }
  if (p.n_split == 1) {
    finish_heads<NREP, KVDT>(p, b, kvh, d, Ms, Ls, Os, 0u);
    return;
  }
#pragma unroll
  for (int r = 0; r < NREP; ++r) publish_split(p, b, kvh * NREP + r, split, d, Ms[r], Ls[r], Os[r]);
  __syncthreads();
  if (tid == 0) s_last = ticket_add(p.ws_count + b * p.Hkv + kvh) == p.n_split - 1;
  __syncthreads();
  if (!s_last) return;
  merge_splits<NREP, KVDT>(p, b, kvh, reinterpret_cast<float*>(ring), C::RING / 4, 0u, &merge_bar);
}

}  // namespace mmab

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
  p.ws_next = p.ws_count + static_cast<size_t>(B) * p.Hkv;
  p.ws_part = reinterpret_cast<float*>(w + 256 + tickets_bytes(B, p.Hkv));
  p.n_split = pl.n_split;
  p.tiles_per_split = pl.tiles_per_split;
  dim3 grid(pl.n_split, p.Hkv, B);
  kern<<<grid, kThreads, C::SMEM, st>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}

template <int NREP, int SDT, int QDT>
int launch_mma(Params p, int B, void* ws, size_t ws_bytes, cudaStream_t st) {
  using C = mmak::MCfg<NREP>;
  const bool dyn = p.dynamic && vs_map_ok(p.vsc, Elem<SDT>::kBytes, p.vscb, p.vsch, p.vscs);
  auto kern = dyn ? mmak::decode_mma_kernel<NREP, SDT, QDT, true>
                  : mmak::decode_mma_kernel<NREP, SDT, QDT, false>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<int> occ[64];
  int per_sm = (dev >= 0 && dev < 64) ? occ[dev].load(std::memory_order_relaxed) : 0;
  if (per_sm <= 0) {
    // both schedules: the same shared memory, so the same occupancy
    for (auto k : {mmak::decode_mma_kernel<NREP, SDT, QDT, true>,
                   mmak::decode_mma_kernel<NREP, SDT, QDT, false>}) {
      cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(k),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
      if (e != cudaSuccess) return static_cast<int>(e);
    }
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, C::SMEM);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (per_sm <= 0) return HQ_ERR_UNSUPPORTED;
    if (dev >= 0 && dev < 64) occ[dev].store(per_sm, std::memory_order_relaxed);
  }
  const int sms = sm_count(dev);
  // Sequence-sharded launches wait for the other ranks inside the grid: every
  // block must be resident at once, so that a waiting block never holds the
  // slot of a block another rank is waiting for.
  if (p.world > 0 && B * p.Hkv > per_sm * sms) return HQ_ERR_UNSUPPORTED;
  const int S_plan = p.seq_len ? p.S_plan : p.S;
  // fused append: the appended token's split is one more block per (b, kv head); the
  // main splits are planned for the slots left, so that it runs in the same wave
  // rather than waiting for a slot while every merge waits for it
  const int slots = per_sm * sms;
  const int plan_slots = (p.k_new && slots >= 2 * B * p.Hkv) ? slots - B * p.Hkv : slots;
  const Plan pl = make_plan(B * p.Hkv, S_plan, plan_slots, sms, mmak::kTileT, p.world > 0);
  if (ws_bytes < workspace_bytes(B, p.Hq, p.Hkv, S_plan, sms)) return HQ_ERR_WORKSPACE;
  // fused append: one more partial row per head (the appended token's split)
  const int n_rows = pl.n_split + (p.k_new ? 1 : 0);
  if (p.k_new && ws_bytes < 256 + tickets_bytes(B, p.Hkv) +
                                sizeof(float) * static_cast<size_t>(B) * p.Hq * n_rows * kPartRow)
    return HQ_ERR_WORKSPACE;
  CUtensorMap tmk, tmv, tmvs;
  int rc = encode_kv_map(&tmk, p.k, p.kvsb, p.kvsh, p.S, p.Hkv, B);
  if (rc == HQ_OK) rc = encode_kv_map(&tmv, p.v, p.kvsb, p.kvsh, p.S, p.Hkv, B);
  if (rc == HQ_OK && dyn)
    rc = encode_vs_map(&tmvs, p.vsc, Elem<SDT>::kBytes, p.vscb, p.vsch, p.S, p.Hkv, B);
  if (rc != HQ_OK) return rc;
  if (!dyn) tmvs = tmv;  // unused by the static schedule
  char* w = static_cast<char*>(ws);
  p.ws_status = reinterpret_cast<int*>(w);
  p.ws_count = reinterpret_cast<int*>(w + 256);
  p.ws_next = p.ws_count + static_cast<size_t>(B) * p.Hkv;
  p.ws_part = reinterpret_cast<float*>(w + 256 + tickets_bytes(B, p.Hkv));
  p.n_split = n_rows;
  p.tiles_per_split = pl.tiles_per_split;
  if (p.clear_header) {
    const cudaError_t e =
        cudaMemsetAsync(ws, 0, 256 + tickets_bytes(B, p.Hkv), st);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  // kv head fastest: the blocks dispatched last are the last splits, which hold
  // the remainder tiles (the shortest runs)
  dim3 grid(p.Hkv, n_rows, B);
  if (p.overlap || p.world > 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (p.world > 0) {
      // the sequence-sharded exchange waits inside the grid: a cooperative
      // launch, refused (cudaErrorCooperativeLaunchTooLarge) when its blocks
      // cannot all be resident at once
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
    } else {
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tmk, tmv, tmvs, p);
    if (e != cudaSuccess) cudaGetLastError();  // leave no error behind for the caller's next call
    return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
  }
  kern<<<grid, kThreads, C::SMEM, st>>>(tmk, tmv, tmvs, p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}

// 16-bit [B, Hkv, S, 128] with element strides (sb, sh, 128): boxes of 128 tokens x 64
// channels (128 bytes), 128-byte swizzle, zero fill past S; two boxes per token row.
inline int encode_kv_map16(CUtensorMap* m, const void* base, int64_t sb, int64_t sh, int S,
                           int Hkv, int B) {
  auto enc = encode_fn();
  if (!enc) return HQ_ERR_UNSUPPORTED;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(S > 0 ? S : 1),
                        static_cast<cuuint64_t>(Hkv), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(kD * 2), static_cast<cuuint64_t>(sh * 2),
                           static_cast<cuuint64_t>(sb * 2)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(mmab::kTileT), 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<void*>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? HQ_OK : HQ_ERR_INVALID_ARGUMENT;
}

template <int NREP, int KVDT>
int launch_dense_mma(Params p, int B, void* ws, size_t ws_bytes, cudaStream_t st) {
  using C = mmab::BCfg<NREP>;
  auto kern = mmab::decode_dense_mma_kernel<NREP, KVDT>;
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
  // one block per SM: a second wave would leave the SMs of finished blocks idle while
  // it starts, so plans fit in one wave when the work allows
  const Plan pl = make_plan(B * p.Hkv, p.S, per_sm * sms, sms, mmab::kTileT,
                            per_sm == 1 && B * p.Hkv <= sms);
  if (ws_bytes < workspace_bytes(B, p.Hq, p.Hkv, p.S, sms)) return HQ_ERR_WORKSPACE;
  CUtensorMap tmk, tmv;
  int rc = encode_kv_map16(&tmk, p.k, p.kvsb, p.kvsh, p.S, p.Hkv, B);
  if (rc == HQ_OK) rc = encode_kv_map16(&tmv, p.v, p.kvsb, p.kvsh, p.S, p.Hkv, B);
  if (rc != HQ_OK) return rc;
  char* w = static_cast<char*>(ws);
  p.ws_status = reinterpret_cast<int*>(w);
  p.ws_count = reinterpret_cast<int*>(w + 256);
  p.ws_next = p.ws_count + static_cast<size_t>(B) * p.Hkv;
  p.ws_part = reinterpret_cast<float*>(w + 256 + tickets_bytes(B, p.Hkv));
  p.n_split = pl.n_split;
  p.tiles_per_split = pl.tiles_per_split;
  dim3 grid(p.Hkv, pl.n_split, B);
  kern<<<grid, kThreads, C::SMEM, st>>>(tmk, tmv, p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}

template <int KVDT>
int dispatch_dense_mma(int nrep, const Params& p, int B, void* ws, size_t wsb, cudaStream_t st) {
  switch (nrep) {
    case 1: return launch_dense_mma<1, KVDT>(p, B, ws, wsb, st);
    case 2: return launch_dense_mma<2, KVDT>(p, B, ws, wsb, st);
    case 4: return launch_dense_mma<4, KVDT>(p, B, ws, wsb, st);
    default: return HQ_ERR_UNSUPPORTED;
  }
}

template <int SDT, int QDT>
int dispatch_mma(int nrep, const Params& p, int B, void* ws, size_t wsb, cudaStream_t st) {
  switch (nrep) {
    case 1: return launch_mma<1, SDT, QDT>(p, B, ws, wsb, st);
    case 2: return launch_mma<2, SDT, QDT>(p, B, ws, wsb, st);
    case 4: return launch_mma<4, SDT, QDT>(p, B, ws, wsb, st);
    default: return HQ_ERR_UNSUPPORTED;
  }
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

static int decode_int8_impl(const void* q, int q_dtype, const int64_t q_strides[3],
                              const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                              const void* k_scale, const void* v_scale, int scale_dtype,
                              const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                              int Hq, int Hkv, int S, int D, float sm_scale, int q_quant,
                              void* out, const int64_t out_strides[3], float* partial_out,
                              void* workspace, size_t workspace_bytes, hq_stream_t stream,
                              void* const* peer_bufs, int world, int rank,
                              const int* seq_len = nullptr, int S_plan = 0, int overlap = 0,
                              const void* k_new = nullptr, const void* v_new = nullptr,
                              const int64_t* kn_strides = nullptr,
                              const int64_t* vn_strides = nullptr, int clear_header = 0,
                              int dynamic = 0) {
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
  p.world = world;
  p.rank = rank;
  for (int w = 0; w < world; ++w) p.peer[w] = static_cast<char*>(peer_bufs[w]);
  p.seq_len = seq_len;
  p.S_plan = S_plan < 0 ? 0 : (S_plan > S ? S : S_plan);
  p.overlap = overlap;
  p.clear_header = clear_header;
  p.dynamic = dynamic;
  p.k_new = k_new;
  p.v_new = v_new;
  if (k_new) {
    p.knb = kn_strides[0];
    p.knh = kn_strides[1];
    p.vnb = vn_strides[0];
    p.vnh = vn_strides[1];
  }
  const int nrep = Hq / Hkv;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define HQ_Q(SDT)                                                                                \
  switch (q_dtype) {                                                                             \
    case HQ_DTYPE_BF16: return dispatch_mma<SDT, HQ_DTYPE_BF16>(nrep, p, B, workspace, workspace_bytes, st); \
    case HQ_DTYPE_F16: return dispatch_mma<SDT, HQ_DTYPE_F16>(nrep, p, B, workspace, workspace_bytes, st);   \
    case HQ_DTYPE_F32: return dispatch_mma<SDT, HQ_DTYPE_F32>(nrep, p, B, workspace, workspace_bytes, st);   \
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

extern "C" int hq_decode_int8(const void* q, int q_dtype, const int64_t q_strides[3],
                              const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                              const void* k_scale, const void* v_scale, int scale_dtype,
                              const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                              int Hq, int Hkv, int S, int D, float sm_scale, int q_quant,
                              void* out, const int64_t out_strides[3], float* partial_out,
                              void* workspace, size_t workspace_bytes, hq_stream_t stream) {
  return decode_int8_impl(q, q_dtype, q_strides, k, v, kv_strides, k_scale, v_scale, scale_dtype,
                          ksc_strides, vsc_strides, B, Hq, Hkv, S, D, sm_scale, q_quant, out,
                          out_strides, partial_out, workspace, workspace_bytes, stream, nullptr, 0, 0);
}

namespace hq {
// hq_decode_int8 whose workspace header (status word, arrival tickets) is
// zeroed on the stream right before the launch, once every argument check has
// passed: for a shared scratch that may still hold the state of a call that
// gave up.  Library-internal (not exported).
int decode_int8_clear_first(const void* q, int q_dtype, const int64_t q_strides[3],
                            const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                            const void* k_scale, const void* v_scale, int scale_dtype,
                            const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                            int Hq, int Hkv, int S, int D, float sm_scale, int q_quant, void* out,
                            const int64_t out_strides[3], float* partial_out, void* workspace,
                            size_t workspace_bytes, hq_stream_t stream) {
  return decode_int8_impl(q, q_dtype, q_strides, k, v, kv_strides, k_scale, v_scale, scale_dtype,
                          ksc_strides, vsc_strides, B, Hq, Hkv, S, D, sm_scale, q_quant, out,
                          out_strides, partial_out, workspace, workspace_bytes, stream, nullptr, 0,
                          0, nullptr, 0, 0, nullptr, nullptr, nullptr, nullptr, 1);
}
}  // namespace hq

extern "C" int hq_decode_int8_ex(const void* q, int q_dtype, const int64_t q_strides[3],
                                 const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                                 const void* k_scale, const void* v_scale, int scale_dtype,
                                 const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                                 int Hq, int Hkv, int S, int D, float sm_scale, int q_quant,
                                 void* out, const int64_t out_strides[3], float* partial_out,
                                 void* workspace, size_t workspace_bytes, unsigned flags,
                                 hq_stream_t stream) {
  if (flags & ~static_cast<unsigned>(HQ_DECODE_OVERLAP_PREVIOUS | HQ_DECODE_DYNAMIC_TILES))
    return HQ_ERR_INVALID_ARGUMENT;
  return decode_int8_impl(q, q_dtype, q_strides, k, v, kv_strides, k_scale, v_scale, scale_dtype,
                          ksc_strides, vsc_strides, B, Hq, Hkv, S, D, sm_scale, q_quant, out,
                          out_strides, partial_out, workspace, workspace_bytes, stream, nullptr, 0,
                          0, nullptr, 0, (flags & HQ_DECODE_OVERLAP_PREVIOUS) ? 1 : 0, nullptr,
                          nullptr, nullptr, nullptr, 0, (flags & HQ_DECODE_DYNAMIC_TILES) ? 1 : 0);
}

// ---------------------------------------------------------------- device-resident length
extern "C" int hq_decode_int8_len(const void* q, int q_dtype, const int64_t q_strides[3],
                                  const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                                  const void* k_scale, const void* v_scale, int scale_dtype,
                                  const int64_t ksc_strides[3], const int64_t vsc_strides[3],
                                  int B, int Hq, int Hkv, int S_max, const int* seq_len,
                                  int S_plan, int D, float sm_scale, int q_quant, void* out,
                                  const int64_t out_strides[3], void* workspace,
                                  size_t workspace_bytes, hq_stream_t stream) {
  if (!seq_len || !aligned(seq_len, 4)) return HQ_ERR_INVALID_ARGUMENT;
  if (S_max > 0 && (!k || !v || !v_scale)) return HQ_ERR_INVALID_ARGUMENT;
  return decode_int8_impl(q, q_dtype, q_strides, k, v, kv_strides, k_scale, v_scale, scale_dtype,
                          ksc_strides, vsc_strides, B, Hq, Hkv, S_max, D, sm_scale, q_quant, out,
                          out_strides, nullptr, workspace, workspace_bytes, stream, nullptr, 0, 0,
                          seq_len, S_plan);
}

extern "C" int hq_decode_append_int8_len(
    const void* q, int q_dtype, const int64_t q_strides[3], const void* k_new, const void* v_new,
    const int64_t kn_strides[3], const int64_t vn_strides[3], int8_t* k, int8_t* v,
    const int64_t kv_strides[3], const void* k_scale, void* v_scale, int scale_dtype,
    const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B, int Hq, int Hkv, int S_max,
    int* seq_len, int S_plan, int D, float sm_scale, int q_quant, void* out,
    const int64_t out_strides[3], void* workspace, size_t workspace_bytes, hq_stream_t stream) {
  if (!seq_len || !aligned(seq_len, 4) || !k_new || !v_new || !kn_strides || !vn_strides ||
      S_max < 1 || !k || !v || !v_scale)
    return HQ_ERR_INVALID_ARGUMENT;
  if (!aligned(workspace, 256)) return HQ_ERR_WORKSPACE;
  return decode_int8_impl(q, q_dtype, q_strides, k, v, kv_strides, k_scale, v_scale, scale_dtype,
                          ksc_strides, vsc_strides, B, Hq, Hkv, S_max, D, sm_scale, q_quant, out,
                          out_strides, nullptr, workspace, workspace_bytes, stream, nullptr, 0, 0,
                          seq_len, S_plan, 0, k_new, v_new, kn_strides, vn_strides);
}

// ---------------------------------------------------------------- sequence sharding over peer memory
extern "C" size_t hq_peer_buffer_bytes(int world, int B, int Hq, int Hkv) {
  if (world < 1 || world > kMaxPeers || B < 1 || Hq < 1 || Hkv < 1) return 0;
  return peer_bytes(B, Hq, Hkv, world);
}

extern "C" int hq_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return HQ_ERR_INVALID_ARGUMENT;
  void* d = nullptr;
  cudaError_t e = cudaMalloc(&d, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemset(d, 0, bytes);  // generation counters, flags and slots start at zero
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), d);
  if (e != cudaSuccess) {
    cudaFree(d);
    return static_cast<int>(e);
  }
  *ptr = d;
  return HQ_OK;
}

extern "C" int hq_peer_open(const void* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) return HQ_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}

extern "C" int hq_peer_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}

extern "C" int hq_peer_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? HQ_OK : static_cast<int>(e);
}

extern "C" int hq_decode_int8_peer(const void* q, int q_dtype, const int64_t q_strides[3],
                                   const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                                   const void* k_scale, const void* v_scale, int scale_dtype,
                                   const int64_t ksc_strides[3], const int64_t vsc_strides[3],
                                   int B, int Hq, int Hkv, int S, int D, float sm_scale,
                                   int q_quant, void* out, const int64_t out_strides[3],
                                   void* workspace, size_t workspace_bytes,
                                   void* const* peer_bufs, int world, int rank,
                                   hq_stream_t stream) {
  if (!peer_bufs || world < 1 || world > kMaxPeers || rank < 0 || rank >= world || !out)
    return HQ_ERR_INVALID_ARGUMENT;
  for (int w = 0; w < world; ++w)
    if (!peer_bufs[w] || !aligned(peer_bufs[w], 256)) return HQ_ERR_INVALID_ARGUMENT;
  return decode_int8_impl(q, q_dtype, q_strides, k, v, kv_strides, k_scale, v_scale, scale_dtype,
                          ksc_strides, vsc_strides, B, Hq, Hkv, S, D, sm_scale, q_quant, out,
                          out_strides, nullptr, workspace, workspace_bytes, stream, peer_bufs,
                          world, rank);
}

static int decode_dense_impl(const void* q, const int64_t q_strides[3], const void* k,
                             const void* v, int kv_dtype, const int64_t kv_strides[3], int B,
                             int Hq, int Hkv, int S, int D, float sm_scale, int q_quant,
                             void* out, const int64_t out_strides[3], float* partial_out,
                             void* workspace, size_t workspace_bytes, hq_stream_t stream,
                             bool tensor_cores) {
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
  if (tensor_cores) {
    switch (kv_dtype) {
      case HQ_DTYPE_BF16: return dispatch_dense_mma<HQ_DTYPE_BF16>(nrep, p, B, workspace, workspace_bytes, st);
      case HQ_DTYPE_F16: return dispatch_dense_mma<HQ_DTYPE_F16>(nrep, p, B, workspace, workspace_bytes, st);
      default: return HQ_ERR_UNSUPPORTED;
    }
  }
  switch (kv_dtype) {
    case HQ_DTYPE_BF16:
      return dispatch_nrep<HQ_DTYPE_BF16, HQ_DTYPE_F32, HQ_DTYPE_BF16>(nrep, p, B, workspace, workspace_bytes, st);
    case HQ_DTYPE_F16:
      return dispatch_nrep<HQ_DTYPE_F16, HQ_DTYPE_F32, HQ_DTYPE_F16>(nrep, p, B, workspace, workspace_bytes, st);
    default:
      return HQ_ERR_UNSUPPORTED;
  }
}

extern "C" int hq_decode_dense(const void* q, const int64_t q_strides[3], const void* k,
                               const void* v, int kv_dtype, const int64_t kv_strides[3], int B,
                               int Hq, int Hkv, int S, int D, float sm_scale, int q_quant,
                               void* out, const int64_t out_strides[3], float* partial_out,
                               void* workspace, size_t workspace_bytes, hq_stream_t stream) {
  return decode_dense_impl(q, q_strides, k, v, kv_dtype, kv_strides, B, Hq, Hkv, S, D, sm_scale,
                           q_quant, out, out_strides, partial_out, workspace, workspace_bytes,
                           stream, true);
}

extern "C" int hq_decode_dense_fma(const void* q, const int64_t q_strides[3], const void* k,
                                   const void* v, int kv_dtype, const int64_t kv_strides[3], int B,
                                   int Hq, int Hkv, int S, int D, float sm_scale, int q_quant,
                                   void* out, const int64_t out_strides[3], float* partial_out,
                                   void* workspace, size_t workspace_bytes, hq_stream_t stream) {
  return decode_dense_impl(q, q_strides, k, v, kv_dtype, kv_strides, B, Hq, Hkv, S, D, sm_scale,
                           q_quant, out, out_strides, partial_out, workspace, workspace_bytes,
                           stream, false);
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
