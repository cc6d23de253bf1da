// Block-wise per-channel K layout: decode attention on the int8 tensor cores (sm_100a).
//
// The block-wise layout (kblock.cu) scales K per (block of BT tokens, channel);
// everything else - int8 codes, per-token V scales - is the default layout's.
// This kernel is decode_mma_kernel (decode_attn.cu) with one change: the K
// scale varies along the contracted dimension from block to block, so q' =
// q * k_scale[block] * sm_scale * log2(e) is rebuilt whenever a warp's tokens
// enter a new block.  BT >= 64 and every warp reads 32 consecutive tokens of a
// 128-token tile, so each warp's tokens lie in one block: warp w of tile t uses
// block (token of its first row) / BT.
//
//   * fixed point: q' is written as three balanced int8 limbs of a 24-bit value
//     relative to one per-head range for the whole split - the largest |q'|
//     over the split's blocks, max_d |q_d| * max_blocks k_scale[block][d] *
//     sm_scale * log2(e), found in the prologue - so the score factors stay
//     constant across the split's tiles and the scores are exact integer sums
//     rescaled once, as in the default kernel;
//   * per warp, a table of q' limb B-fragments (the default kernel's qtab, one per
//     warp here): lane l converts channels 4 l .. 4 l + 3 of every head from its
//     block's K scales (loaded two tiles ahead as one float4), writes the three
//     limb words of each head, and the warp reads its B-fragments back after a
//     __syncwarp - no block barrier inside the tile loop;
//   * K / V tiles by tensor-map TMA into the 3-stage ring, per-token V scales two
//     tiles ahead, p' limbs, int32 PV sums, the split ticket and the merge: the
//     default kernel's code paths.
// Reference semantics: the block-wise decode of kblock.cu's CUDA-core kernel
// (same attention, K dequantized with its block's scale); the reference itself
// keeps one K scale per channel (tests/qwen_kvcache_full.py:54) and names the
// block-wise layout as its roadmap's fix (README.md:141).
#include "decode_common.cuh"

namespace hq {
namespace dec {
namespace kbm {

using mmak::kLimbMax;
using mmak::kStagesM;
using mmak::kTileB;
using mmak::kTileT;

template <int NREP>
struct KCfg {
  static constexpr int NT = (NREP + 1) / 2;               // n8 tiles, 2 heads each
  static constexpr int RING = kStagesM * 2 * kTileB;      // 96 KB
  static constexpr int LIMB = kWarps * NT * 8 * 32;       // p' limb staging
  static constexpr int QTAB = kWarps * NT * 256 * 4;      // per-warp q' limb B-fragment words
  static constexpr int SMEM = 1024 + RING + NREP * kD * 4 + LIMB + 2 * kStagesM * 8 + QTAB;
  static_assert(kWarps * NREP * kD * 4 + kWarps * NREP * 8 <= RING, "epilogue scratch");
};

template <int NREP, int SDT, int QDT>
__global__ void __launch_bounds__(kThreads, 2) kblock_mma_kernel(
    const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
    const Params p) {
  using C = KCfg<NREP>;
  using QE = Elem<QDT>;
  using SE = Elem<SDT>;
  constexpr int NT = C::NT;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* ring = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* qs = reinterpret_cast<float*>(ring + C::RING);  // q * sm_scale * log2(e) * kLimbMax / qmax
  unsigned char* plimb = reinterpret_cast<unsigned char*>(qs + NREP * kD);
  uint64_t* full = reinterpret_cast<uint64_t*>(plimb + C::LIMB);
  uint64_t* empty = full + kStagesM;
  uint32_t* qtab_all = reinterpret_cast<uint32_t*>(empty + kStagesM);
  __shared__ float red[kWarps][NREP];
  __shared__ float qmax_s[NREP];
  __shared__ int s_last;
  __shared__ __align__(8) uint64_t merge_bar;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
  const int d = tid;
  const int BT = p.kblock_tokens;
  int S = p.S, tps = p.tiles_per_split;
  if (p.seq_len) {
    // device-resident length: the split count is the host's plan, the tiles per
    // split follow the length read here (the tensor maps cover the capacity p.S)
    S = min(max(__ldcg(p.seq_len), 0), p.S);
    tps = max(1, ((S + kTileT - 1) / kTileT + p.n_split - 1) / p.n_split);
  }
  const int s_begin = split * tps * kTileT;
  const int s_end = min(S, s_begin + tps * kTileT);
  const int ntok = max(0, s_end - s_begin);
  const int ntiles = (ntok + kTileT - 1) / kTileT;
  uint32_t* qtab = qtab_all + warp * NT * 256;

  int issued = 0;
  const uint64_t pol_stream = mmak::l2_evict_first();
  auto issue = [&](int t) {
    const int st = t % kStagesM;
    unsigned char* dst = ring + st * 2 * kTileB;
    mbar_arrive_expect_tx(&full[st], 2 * kTileB);
    mmak::tma_load_4d(dst, &tmk, 0, s_begin + t * kTileT, kvh, b, &full[st], pol_stream);
    mmak::tma_load_4d(dst + kTileB, &tmv, 0, s_begin + t * kTileT, kvh, b, &full[st], pol_stream);
    issued = t + 1;
  };
  const auto* vscp = reinterpret_cast<const typename SE::T*>(p.vsc);
  const int64_t vsc_row = b * p.vscb + kvh * p.vsch;
  auto load_vs = [&](int t, float (&v)[2]) {
#pragma unroll
    for (int rb = 0; rb < 2; ++rb) {
      const int tok = t * kTileT + warp * 32 + rb * 16 + g + 8 * (t4 & 1);
      v[rb] = tok < ntok ? SE::to_f32(vscp[vsc_row + static_cast<int64_t>(s_begin + tok) * p.vscs]) : 0.0f;
    }
  };
  // K block scales: this warp's block for tile t, and lane l's channels 4 l .. 4 l + 3 of it
  const float* ksp = reinterpret_cast<const float*>(p.ksc) + b * p.kscb + kvh * p.ksch;
  // (a warp whose 32 tokens all lie past the split's end has no block: its scores are masked)
  auto warp_tok = [&](int t) { return s_begin + t * kTileT + warp * 32; };
  auto load_ks = [&](int t) {
    if (t >= ntiles || warp_tok(t) >= s_end) return make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    return *reinterpret_cast<const float4*>(ksp + static_cast<int64_t>(warp_tok(t) / BT) * p.kscd +
                                            4 * lane);
  };

  // q and the split's per-channel K-scale maximum (thread d = channel d)
  const auto* qp = reinterpret_cast<const typename QE::T*>(p.q);
  float qv[NREP];
#pragma unroll
  for (int r = 0; r < NREP; ++r) qv[r] = QE::to_f32(qp[b * p.qsb + (kvh * NREP + r) * p.qsh + d]) * p.qk_scale;
  float vs_a[2], vs_b[2];
  load_vs(0, vs_a);
  load_vs(1, vs_b);
  float4 ks_a = load_ks(0), ks_b = load_ks(1);
  if (tid == 0) {
    for (int s = 0; s < kStagesM; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    mbar_init(&merge_bar, 1);
    fence_mbar_init();
  }
  // zero the p' staging (columns 3 and 7 stay zero) and the q' tables (limb 3 and
  // absent heads stay zero)
  for (int i = tid; i < C::LIMB / 4; i += kThreads) reinterpret_cast<uint32_t*>(plimb)[i] = 0;
  for (int i = tid; i < kWarps * NT * 256; i += kThreads) qtab_all[i] = 0;
  __syncthreads();
  // every stage requested before the K-scale maximum below: its loads (one per block
  // of the split) would otherwise hold back the first tile copies
  if (tid == 0)
    for (int t = 0; t < min(kStagesM, ntiles); ++t) issue(t);
  float ksmax = 0.0f;
  if (ntok > 0) {
    const int blk_lo = s_begin / BT, blk_hi = (s_end + BT - 1) / BT;
#pragma unroll 8
    for (int blk = blk_lo; blk < blk_hi; ++blk)
      ksmax = fmaxf(ksmax, __ldg(ksp + static_cast<int64_t>(blk) * p.kscd + d));
  }

  // per-head fixed-point range of the split: max_d |q'_d| * max over its blocks
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    const float m = warp_max(fabsf(qv[r]) * ksmax, 1);
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
  // q' limbs are rint(q * k_scale * inv): the factor folded into the staged q once
#pragma unroll
  for (int r = 0; r < NREP; ++r)
    qs[r * kD + d] = qv[r] * (qmax_s[r] > 0.0f ? kLimbMax / qmax_s[r] : 0.0f);
  __syncthreads();
  float f0[NT], f1[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int my_head = 2 * nt + (t4 >> 1);
    const float qsc = my_head < NREP && qmax_s[my_head] > 0.0f ? qmax_s[my_head] / kLimbMax : 0.0f;
    f0[nt] = (t4 & 1) ? qsc : qsc * 65536.0f;
    f1[nt] = (t4 & 1) ? 0.0f : qsc * 256.0f;
  }
  // this warp's q' limb B-fragments for a block with K scales ks (lane's 4 channels)
  uint32_t bq[NT][4][2];
  auto build = [&](const float4& ks) {
    const float k4[4] = {ks.x, ks.y, ks.z, ks.w};
    const int jj = lane >> 3, hh = (lane >> 2) & 1, tt = lane & 3;
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int x = max(-static_cast<int>(kLimbMax),
                          min(static_cast<int>(kLimbMax),
                              __float2int_rn(qs[r * kD + 4 * lane + e] * k4[e])));
        int la, lb, lc;
        mmak::limbs24(x, la, lb, lc);
        w0 |= (static_cast<uint32_t>(la) & 0xffu) << (8 * e);
        w1 |= (static_cast<uint32_t>(lb) & 0xffu) << (8 * e);
        w2 |= (static_cast<uint32_t>(lc) & 0xffu) << (8 * e);
      }
      const int base = ((r >> 1) << 8) | (jj << 6) | (hh << 5) | tt;
      const int gg = (r & 1) * 4;
      qtab[base | ((gg + 0) << 2)] = w0;
      qtab[base | ((gg + 1) << 2)] = w1;
      qtab[base | ((gg + 2) << 2)] = w2;
    }
    __syncwarp();
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) bq[nt][j][h2] = qtab[(nt << 8) | (j << 6) | (h2 << 5) | lane];
    __syncwarp();  // the table is rewritten by the next build
  };

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
  int cur_blk = -1;
  for (int t = 0; t < ntiles; ++t) {
    const int st = t % kStagesM;
    const uint32_t par = (t / kStagesM) & 1;
    const int base_tok = t * kTileT + warp * 32;
    float vsf[2];
    bool own_ok[2];
#pragma unroll
    for (int rb = 0; rb < 2; ++rb) {
      own_ok[rb] = base_tok + rb * 16 + g + 8 * (t4 & 1) < ntok;
      vsf[rb] = vs_a[rb];
      vs_a[rb] = vs_b[rb];
    }
    load_vs(t + 2, vs_b);
    // q' of this warp's block (rebuilt when the block changes; a block's 32-token
    // chunks never straddle two blocks)
    const float4 ks_cur = ks_a;
    ks_a = ks_b;
    ks_b = load_ks(t + 2);
    if (warp_tok(t) < s_end && warp_tok(t) / BT != cur_blk) {
      build(ks_cur);
      cur_blk = warp_tok(t) / BT;
    }
    if (!mbar_wait(&full[st], par)) {
      ok = false;
      break;
    }
    consumed = t + 1;
    const uint32_t kt = smem_u32(ring + st * 2 * kTileB);
    const uint32_t vt = kt + kTileB;

    float sc[NT][2][2];
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
        mmak::ldsm_x4(kt + mmak::swz(row, 2 * j + (mat >> 1)), a);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mmak::mma_s8(sacc[nt], a, bq[nt][j][0], bq[nt][j][1]);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float lo = f0[nt] * static_cast<float>(sacc[nt][0]) + f1[nt] * static_cast<float>(sacc[nt][1]);
        float hi = f0[nt] * static_cast<float>(sacc[nt][2]) + f1[nt] * static_cast<float>(sacc[nt][3]);
        lo += __shfl_xor_sync(0xffffffffu, lo, 1);
        hi += __shfl_xor_sync(0xffffffffu, hi, 1);
        const int tok = base_tok + rb * 16 + g;
        sc[nt][rb][0] = tok < ntok ? lo : -INFINITY;
        sc[nt][rb][1] = tok + 8 < ntok ? hi : -INFINITY;
      }
    }
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
          const float alpha = exp2f(m_run[nt] - m_new);
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
        mmak::limbs24(x, la, lb, lc);
        const int k = mmak::pv_k(rb * 16 + g + 8 * (t4 & 1));
        dst[(4 * hh + 0) * 32 + k] = static_cast<unsigned char>(la);
        dst[(4 * hh + 1) * 32 + k] = static_cast<unsigned char>(lb);
        dst[(4 * hh + 2) * 32 + k] = static_cast<unsigned char>(lc);
      }
    }
    __syncwarp();
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
        mmak::ldsm_x4_t(vt + mmak::swz(row, 2 * j + (mat >> 1)), r);
        ae[2 * th + 0] = prmt(r[0], r[1], 0x6420u);
        ao[2 * th + 0] = prmt(r[0], r[1], 0x7531u);
        ae[2 * th + 1] = prmt(r[2], r[3], 0x6420u);
        ao[2 * th + 1] = prmt(r[2], r[3], 0x7531u);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mmak::mma_s8(acc[nt][j][0], ae, bp[nt][0], bp[nt][1]);
        mmak::mma_s8(acc[nt][j][1], ao, bp[nt][0], bp[nt][1]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (tid == 0 && t + kStagesM < ntiles) {
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

  // ---- block epilogue: flush, merge the 4 warps, publish or finish
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) flush(nt, true);
  float* wo = reinterpret_cast<float*>(ring);
  float* wl = wo + kWarps * NREP * kD;
  float* wm = wl + kWarps * NREP;
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
          const int dd = 32 * j + 2 * g + pi + 16 * (t4 & 1);
          dst[dd] = (t4 & 1) ? o_acc[nt][j][pi][1] : o_acc[nt][j][pi][0];
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
    finish_heads<NREP, QDT>(p, b, kvh, d, Ms, Ls, Os, 0u);
    return;
  }
#pragma unroll
  for (int r = 0; r < NREP; ++r) publish_split(p, b, kvh * NREP + r, split, d, Ms[r], Ls[r], Os[r]);
  __syncthreads();
  if (tid == 0) s_last = ticket_add(p.ws_count + b * p.Hkv + kvh) == p.n_split - 1;
  __syncthreads();
  if (!s_last) return;
  merge_splits<NREP, QDT>(p, b, kvh, reinterpret_cast<float*>(ring), C::RING / 4, 0u, &merge_bar);
}

template <int NREP, int SDT, int QDT>
int launch(Params p, int B, void* ws, size_t ws_bytes, cudaStream_t st) {
  using C = KCfg<NREP>;
  auto kern = kblock_mma_kernel<NREP, SDT, QDT>;
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
  const int S_plan = p.seq_len ? p.S_plan : p.S;
  const Plan pl = make_plan(B * p.Hkv, S_plan, per_sm * sms, sms, kTileT);
  if (ws_bytes < workspace_bytes(B, p.Hq, p.Hkv, S_plan, sms)) return HQ_ERR_WORKSPACE;
  CUtensorMap tmk, tmv;
  int rc = encode_kv_map(&tmk, p.k, p.kvsb, p.kvsh, p.S, p.Hkv, B);
  if (rc == HQ_OK) rc = encode_kv_map(&tmv, p.v, p.kvsb, p.kvsh, p.S, p.Hkv, B);
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

template <int SDT, int QDT>
int dispatch(int nrep, const Params& p, int B, void* ws, size_t wsb, cudaStream_t st) {
  switch (nrep) {
    case 1: return launch<1, SDT, QDT>(p, B, ws, wsb, st);
    case 2: return launch<2, SDT, QDT>(p, B, ws, wsb, st);
    case 4: return launch<4, SDT, QDT>(p, B, ws, wsb, st);
    default: return HQ_ERR_UNSUPPORTED;
  }
}

}  // namespace kbm
}  // namespace dec

// The block-wise decode on the tensor cores, or HQ_ERR_UNSUPPORTED (nothing
// launched) for what it does not serve: head_dim other than 128, 8 q heads per kv
// head, K and V with different strides, K block scales not addressable as float4
// rows.  Arguments as hq_kblock_decode (already checked there); with seq_len the
// length is read on the device (S is then the capacity, S_plan the length the
// split count is planned for).
int kblock_decode_mma(const void* q, int q_dtype, const int64_t q_strides[3],
                      const int8_t* k_cache, const int64_t kq_strides[3], const float* k_scale,
                      const int64_t ks_strides[3], const int8_t* v_cache,
                      const int64_t vq_strides[3], const void* v_scale, int scale_dtype,
                      const int64_t vs_strides[3], int B, int Hq, int Hkv, int S, int D,
                      int block_tokens, float sm_scale, void* out, const int64_t out_strides[3],
                      void* workspace, size_t workspace_bytes, hq_stream_t stream,
                      const int* seq_len, int S_plan) {
  using namespace dec;
  const int nrep = Hq / Hkv;
  if (D != kD || (nrep != 1 && nrep != 2 && nrep != 4)) return HQ_ERR_UNSUPPORTED;
  if (kq_strides[0] != vq_strides[0] || kq_strides[1] != vq_strides[1] || kq_strides[2] != kD ||
      vq_strides[2] != kD)
    return HQ_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(k_scale) % 16 || ks_strides[0] % 4 || ks_strides[1] % 4 ||
      ks_strides[2] % 4)
    return HQ_ERR_UNSUPPORTED;
  // no (aligned) workspace: the CUDA-core kernel, which needs none for a single split
  if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256) return HQ_ERR_UNSUPPORTED;
  Params p{};
  p.q = q;
  p.qsb = q_strides[0];
  p.qsh = q_strides[1];
  p.k = reinterpret_cast<const char*>(k_cache);
  p.v = reinterpret_cast<const char*>(v_cache);
  p.kvsb = kq_strides[0];
  p.kvsh = kq_strides[1];
  p.ksc = k_scale;
  p.kscb = ks_strides[0];
  p.ksch = ks_strides[1];
  p.kscd = ks_strides[2];
  p.kblock_tokens = block_tokens;
  p.vsc = v_scale;
  p.vscb = vs_strides[0];
  p.vsch = vs_strides[1];
  p.vscs = vs_strides[2];
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.S = S;
  p.seq_len = seq_len;
  p.S_plan = S_plan < 0 ? 0 : (S_plan > S ? S : S_plan);
  p.qk_scale = sm_scale * kLog2e;
  p.out = out;
  p.osb = out_strides[0];
  p.osh = out_strides[1];
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define HQ_KBQ(SDT)                                                                          \
  switch (q_dtype) {                                                                         \
    case HQ_DTYPE_BF16: return kbm::dispatch<SDT, HQ_DTYPE_BF16>(nrep, p, B, workspace, workspace_bytes, st); \
    case HQ_DTYPE_F16: return kbm::dispatch<SDT, HQ_DTYPE_F16>(nrep, p, B, workspace, workspace_bytes, st);   \
    case HQ_DTYPE_F32: return kbm::dispatch<SDT, HQ_DTYPE_F32>(nrep, p, B, workspace, workspace_bytes, st);   \
    default: return HQ_ERR_UNSUPPORTED;                                                      \
  }
  if (scale_dtype == HQ_DTYPE_F16) {
    HQ_KBQ(HQ_DTYPE_F16)
  } else if (scale_dtype == HQ_DTYPE_F32) {
    HQ_KBQ(HQ_DTYPE_F32)
  }
#undef HQ_KBQ
  return HQ_ERR_UNSUPPORTED;
}

// Workspace bytes of kblock_decode_mma for this shape (0 when it does not serve it).
size_t kblock_decode_mma_workspace_bytes(int B, int Hq, int Hkv, int S, int D) {
  using namespace dec;
  if (B < 1 || Hkv < 1 || Hq % Hkv || D != kD) return 0;
  const int nrep = Hq / Hkv;
  if (nrep != 1 && nrep != 2 && nrep != 4) return 0;
  return workspace_bytes(B, Hq, Hkv, S, current_sm_count());
}

}  // namespace hq
