// Quantize-on-write kernels (sm_100a): symmetric int8, K per channel, V per token.
//
// Reference semantics: quantize_int8 (reference/page_attention_int8_pytorch.py:23-30)
// with reduce dim 2 (K) / 3 (V) of [B, H, S, D], as used by QuantizedKVCache.update
// (tests/qwen_kvcache_full.py:41-47).  The reference's fused Triton kernels
// (src/kernels/quant_kv_triton.py:16-87) run one program per column / row and,
// for K, read each column twice with a 256-byte stride.  Here:
//
//   * V per token: each row of D elements is read once with 16-byte vector
//     loads by D*esize/16 lanes, reduced with warp shuffles, and written as
//     packed int8 (8 codes per 16-byte input vector).
//   * K per channel: a cooperative persistent grid.  A (b, h) slab of S x D is
//     cut into 32 KB chunks of whole rows; each block loads its chunk once
//     into registers (row-contiguous, coalesced), reduces its column maxima,
//     publishes them with atomicMax, waits (bounded) until every chunk of the
//     slab has published, then quantizes the chunk still held in registers.
//     HBM traffic is the algorithmic minimum: 1 read + 1 int8 write per element.
//   * Append: one block per (b, h) quantizes the few new tokens of K (per
//     channel over the new tokens; scale not stored) and V (per token; scale
//     stored), exactly as the reference's update() does on a non-empty layer.
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
  static constexpr int kLanesPerRow = kVecPerRow < 32 ? kVecPerRow : 32;
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

template <int DT, int D>
__global__ void __launch_bounds__(kThreads) quant_v_kernel(
    const char* __restrict__ x, int64_t xsb, int64_t xsh, int64_t xss, int H, int S,
    int64_t n_rows, int8_t* __restrict__ q, int64_t qsb, int64_t qsh, int64_t qss,
    float* __restrict__ sc32, __half* __restrict__ sc16, int64_t ssb, int64_t ssh, int64_t sss) {
  using Sh = VShape<DT, D>;
  constexpr int EB = Elem<DT>::kBytes;
  const int lane = threadIdx.x & 31;
  const int sub = lane % Sh::kLanesPerRow;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
  for (int64_t w = warp0; w * Sh::kRowsPerWarp < n_rows; w += nwarps) {
    const int64_t r = w * Sh::kRowsPerWarp + lane / Sh::kLanesPerRow;
    const bool valid = r < n_rows;
    int64_t s = 0, h = 0, b = 0;
    if (valid) {
      s = r % S;
      const int64_t bh = r / S;
      h = bh % H;
      b = bh / H;
    }
    uint4 vec[Sh::kVecPerLane];
    float amax = 0.0f;
    const char* row = x + (b * xsb + h * xsh + s * xss) * EB;
#pragma unroll
    for (int i = 0; i < Sh::kVecPerLane; ++i) {
      vec[i] = valid ? ldg_stream(row + (sub + i * Sh::kLanesPerRow) * 16) : make_uint4(0, 0, 0, 0);
      float f[Vec16<DT>::N];
      Vec16<DT>::unpack(vec[i], f);
#pragma unroll
      for (int e = 0; e < Vec16<DT>::N; ++e) amax = fmaxf(amax, fabsf(f[e]));
    }
#pragma unroll
    for (int off = Sh::kLanesPerRow / 2; off > 0; off >>= 1)
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if (!valid) continue;
    const Quantizer qz = Quantizer::from_amax(amax);
    int8_t* qrow = q + b * qsb + h * qsh + s * qss;
#pragma unroll
    for (int i = 0; i < Sh::kVecPerLane; ++i) {
      float f[Vec16<DT>::N];
      Vec16<DT>::unpack(vec[i], f);
      int c[Vec16<DT>::N];
#pragma unroll
      for (int e = 0; e < Vec16<DT>::N; ++e) c[e] = qz.code(f[e]);
      store_codes<Vec16<DT>::N>(qrow + (sub + i * Sh::kLanesPerRow) * Sh::kVecElems, c);
    }
    if (sub == 0) {
      const int64_t so = b * ssb + h * ssh + s * sss;
      if (sc32) sc32[so] = qz.scale;
      if (sc16) sc16[so] = __float2half_rn(qz.scale);
    }
  }
}

// ------------------------------------------------------------------ K per channel
// Chunk = kPasses x (kThreads / kVecPerRow) rows; every thread keeps kPasses
// 16-byte vectors of one fixed column group in registers.
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
};

struct KWorkspace {
  int* status;        // [1]
  int* count;         // [B*H] chunks that published their maxima
  unsigned* amax;     // [B*H*D] column absmax as float bits (all >= 0)
};

__host__ __device__ inline size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// mode 0: fused (publish maxima, wait for the slab, write codes; cooperative launch)
// mode 1: publish maxima only          mode 2: write codes from published maxima
template <int DT, int D>
__global__ void __launch_bounds__(kThreads, 3) quant_k_kernel(
    const char* __restrict__ x, int64_t xsb, int64_t xsh, int64_t xss, int H, int S,
    int n_chunks, int64_t n_tasks, int8_t* __restrict__ q, int64_t qsb, int64_t qsh, int64_t qss,
    float* __restrict__ sc32, __half* __restrict__ sc16, KWorkspace ws, int mode) {
  using Sh = KShape<DT, D>;
  constexpr int EB = Elem<DT>::kBytes;
  constexpr int VE = Sh::kVecElems;
  __shared__ float red[Sh::kRedRows][D];
  __shared__ int s_ok;
  const int tid = threadIdx.x;
  const int cg = tid % Sh::kVecPerRow;      // column group: columns cg*VE .. +VE
  const int rs = tid / Sh::kVecPerRow;      // row slot
  const int warp = tid >> 5;
  const int red_row = Sh::kVecPerRow <= 32 ? warp : rs;
  const bool red_writer = Sh::kVecPerRow <= 32 ? (tid & 31) < Sh::kVecPerRow : true;

  for (int64_t task = blockIdx.x; task < n_tasks; task += gridDim.x) {
    const int64_t slab = task / n_chunks;
    const int chunk = static_cast<int>(task % n_chunks);
    const int64_t h = slab % H, b = slab / H;
    const int row0 = chunk * Sh::kRowsPerChunk;
    const char* base = x + (b * xsb + h * xsh) * EB + cg * 16;

    uint4 data[Sh::kPasses];
#pragma unroll
    for (int p = 0; p < Sh::kPasses; ++p) {
      const int s = row0 + p * Sh::kRowSlots + rs;
      data[p] = s < S ? ldg_stream(base + static_cast<int64_t>(s) * xss * EB)
                      : make_uint4(0, 0, 0, 0);
    }
    if (mode != 2) {
      float cmax[VE];
#pragma unroll
      for (int e = 0; e < VE; ++e) cmax[e] = 0.0f;
#pragma unroll
      for (int p = 0; p < Sh::kPasses; ++p) {
        float f[VE];
        Vec16<DT>::unpack(data[p], f);
#pragma unroll
        for (int e = 0; e < VE; ++e) cmax[e] = fmaxf(cmax[e], fabsf(f[e]));
      }
      // lanes of one warp that share a column group differ in bits >= log2(kVecPerRow)
#pragma unroll
      for (int off = Sh::kVecPerRow; off < 32; off <<= 1)
#pragma unroll
        for (int e = 0; e < VE; ++e)
          cmax[e] = fmaxf(cmax[e], __shfl_xor_sync(0xffffffffu, cmax[e], off));
      if (red_writer) {
#pragma unroll
        for (int e = 0; e < VE; ++e) red[red_row][cg * VE + e] = cmax[e];
      }
      __syncthreads();
      for (int c = tid; c < D; c += kThreads) {
        float m = red[0][c];
#pragma unroll
        for (int w = 1; w < Sh::kRedRows; ++w) m = fmaxf(m, red[w][c]);
        if (n_chunks == 1 && mode == 0)
          red[0][c] = m;  // whole slab in this block: the block maximum is final
        else
          atomicMax(ws.amax + slab * D + c, __float_as_uint(m));
      }
      __syncthreads();
      if (mode == 1) continue;
    }
    if (mode == 0 && n_chunks > 1) {
      if (tid == 0) {
        __threadfence();
        atomicAdd(ws.count + slab, 1);
        int ok = 0;
        for (uint32_t it = 0; it < kSpinLimit; ++it) {
          if (*reinterpret_cast<volatile int*>(ws.count + slab) >= n_chunks) {
            ok = 1;
            break;
          }
          __nanosleep(128);
        }
        __threadfence();
        if (!ok) report_error(ws.status, HQ_ERR_DEVICE_TIMEOUT);
        s_ok = ok;
      }
      __syncthreads();
      if (!s_ok) continue;  // status word set; codes of this chunk are left unwritten
    }
    if (mode == 2 || n_chunks > 1) {
      for (int c = tid; c < D; c += kThreads) red[0][c] = __uint_as_float(__ldcg(ws.amax + slab * D + c));
      __syncthreads();
    }
    Quantizer qz[VE];
#pragma unroll
    for (int e = 0; e < VE; ++e) qz[e] = Quantizer::from_amax(red[0][cg * VE + e]);
    if (chunk == 0 && rs == 0) {
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        const int64_t so = slab * D + cg * VE + e;
        if (sc32) sc32[so] = qz[e].scale;
        if (sc16) sc16[so] = __float2half_rn(qz[e].scale);
      }
    }
    int8_t* qbase = q + b * qsb + h * qsh + cg * VE;
#pragma unroll
    for (int p = 0; p < Sh::kPasses; ++p) {
      const int s = row0 + p * Sh::kRowSlots + rs;
      if (s < S) {
        float f[VE];
        Vec16<DT>::unpack(data[p], f);
        int c[VE];
#pragma unroll
        for (int e = 0; e < VE; ++e) c[e] = qz[e].code(f[e]);
        store_codes<VE>(qbase + static_cast<int64_t>(s) * qss, c);
      }
    }
    __syncthreads();  // red[] is reused by the next task
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
    int64_t vsss) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int kW = D / 32;
  __shared__ float wmax[kW];
  const int d = threadIdx.x;
  const int64_t b = blockIdx.x / H, h = blockIdx.x % H;
  const T* kp = reinterpret_cast<const T*>(k) + b * ksb + h * ksh + d;
  const T* vp = reinterpret_cast<const T*>(v) + b * vsb + h * vsh + d;
  // K: per-channel over the S_new new tokens
  float amax = 0.0f;
  for (int s = 0; s < S_new; ++s) amax = fmaxf(amax, fabsf(E::to_f32(kp[s * kss])));
  const Quantizer qk = Quantizer::from_amax(amax);
  for (int s = 0; s < S_new; ++s)
    kq[b * kqb + h * kqh + s * kqs + d] = static_cast<int8_t>(qk.code(E::to_f32(kp[s * kss])));
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
int sm_count(int dev) {
  static std::atomic<int> cache[64];
  if (dev < 0 || dev >= 64) return 148;
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
  const int64_t n_rows = static_cast<int64_t>(B) * H * S;
  const int64_t warps = (n_rows + Sh::kRowsPerWarp - 1) / Sh::kRowsPerWarp;
  int64_t blocks = (warps + kThreads / 32 - 1) / (kThreads / 32);
  const int64_t cap = static_cast<int64_t>(current_sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  const int64_t z[3] = {0, 0, 0};
  if (!ss) ss = z;
  quant_v_kernel<DT, D><<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(
      static_cast<const char*>(x), xs[0], xs[1], xs[2], H, S, n_rows, q, qs[0], qs[1], qs[2], s32,
      reinterpret_cast<__half*>(s16), ss[0], ss[1], ss[2]);
  return finish_launch();
}

template <int DT, int D>
static int launch_quant_k(const void* x, const int64_t* xs, int B, int H, int S, int8_t* q,
                          const int64_t* qs, float* s32, uint16_t* s16, void* wsp,
                          cudaStream_t st) {
  using Sh = KShape<DT, D>;
  const int n_chunks = (S + Sh::kRowsPerChunk - 1) / Sh::kRowsPerChunk;
  const int64_t n_tasks = static_cast<int64_t>(B) * H * n_chunks;
  char* w = static_cast<char*>(wsp);
  KWorkspace ws;
  ws.status = reinterpret_cast<int*>(w);
  ws.count = reinterpret_cast<int*>(w + 256);
  ws.amax = reinterpret_cast<unsigned*>(w + 256 + align256(sizeof(int) * B * H));
  const size_t clear = 256 + align256(sizeof(int) * B * H) + sizeof(unsigned) * B * H * D;
  cudaError_t e = cudaMemsetAsync(wsp, 0, clear, st);
  if (e != cudaSuccess) return static_cast<int>(e);
  auto kern = quant_k_kernel<DT, D>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<int> occ_cache[64];
  int per_sm = (dev >= 0 && dev < 64) ? occ_cache[dev].load(std::memory_order_relaxed) : 0;
  if (per_sm <= 0) {
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, 0);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (per_sm <= 0) return HQ_ERR_UNSUPPORTED;
    if (dev >= 0 && dev < 64) occ_cache[dev].store(per_sm, std::memory_order_relaxed);
  }
  const int64_t resident = static_cast<int64_t>(per_sm) * sm_count(dev);
  int64_t grid = resident < n_tasks ? resident : n_tasks;
  const char* xp = static_cast<const char*>(x);
  int64_t xsb = xs[0], xsh = xs[1], xss = xs[2];
  int64_t qsb = qs[0], qsh = qs[1], qss = qs[2];
  __half* s16h = reinterpret_cast<__half*>(s16);
  if (n_chunks <= resident) {
    // every chunk of a slab can be resident at once: fused single pass
    int mode = 0;
    void* args[] = {&xp, &xsb, &xsh, &xss, &H, &S, (void*)&n_chunks, (void*)&n_tasks, &q, &qsb,
                    &qsh, &qss, &s32, &s16h, &ws, &mode};
    e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kern),
                                    dim3(static_cast<unsigned>(grid)), dim3(kThreads), args, 0,
                                    st);
    if (e != cudaSuccess) return static_cast<int>(e);
    return finish_launch();
  }
  // a slab larger than the resident grid: maxima pass, then code pass
  for (int mode = 1; mode <= 2; ++mode) {
    kern<<<static_cast<unsigned>(grid), kThreads, 0, st>>>(xp, xsb, xsh, xss, H, S, n_chunks,
                                                            n_tasks, q, qsb, qsh, qss, s32, s16h,
                                                            ws, mode);
    const int r = finish_launch();
    if (r != HQ_OK) return r;
  }
  return HQ_OK;
}

template <int DT, int D>
static int launch_append(const void* k, const void* v, const int64_t* ks, const int64_t* vs,
                         int B, int H, int S_new, int8_t* kq, const int64_t* kqs, int8_t* vq,
                         const int64_t* vqs, float* v32, uint16_t* v16, const int64_t* vss,
                         cudaStream_t st) {
  const int64_t z[3] = {0, 0, 0};
  if (!vss) vss = z;
  append_kernel<DT, D><<<B * H, D, 0, st>>>(
      static_cast<const char*>(k), static_cast<const char*>(v), ks[0], ks[1], ks[2], vs[0], vs[1],
      vs[2], H, S_new, kq, kqs[0], kqs[1], kqs[2], vq, vqs[0], vqs[1], vqs[2], v32,
      reinterpret_cast<__half*>(v16), vss[0], vss[1], vss[2]);
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
  return 256 + align256(sizeof(int) * B * H) + align256(sizeof(unsigned) * B * H * D);
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
                                              v_scale_f16, vs_strides, st);))
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

extern "C" int hq_read_status(const void* workspace, hq_stream_t stream) {
  if (!workspace) return HQ_ERR_INVALID_ARGUMENT;
  int v = 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return static_cast<int>(e);
  return v;
}
