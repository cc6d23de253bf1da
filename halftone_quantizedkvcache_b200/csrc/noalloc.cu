// Int8 decode attention for callers that cannot allocate device memory.
//
// Some callers of this library own no device allocator: a host runtime that
// hands the library only the tensors it already holds (for example a plugin
// inside another engine's decode loop, or a binding from a language whose
// runtime manages all device memory itself) cannot call cudaMalloc or
// allocate a workspace per call.  hq_decode_int8_noalloc serves them: it runs
// the same split-KV kernel as hq_decode_int8, with its scratch (split partials,
// arrival tickets, status word) in the file-scope array below instead of a
// caller workspace.
//
// The array is kNoallocScratchBytes (8 MiB) on every GPU that loads the
// library, held until the process exits.  All calls share it: calls that
// overlap on the GPU (different streams, or different host threads without
// ordering) race on it and must be serialised by the caller.  Once a call's
// arguments have passed every check, it clears the tickets and the status word
// on its stream right before its launch, so a call that follows one that gave
// up still starts clean; a call that is refused enqueues nothing.  The array's
// device address is looked up once per device and kept: calls must not cross a
// cudaDeviceReset of that device.
#include <atomic>

#include <cuda_runtime.h>

#include "../../include/halftone_b200.h"

namespace {

constexpr size_t kNoallocScratchBytes = size_t(8) << 20;

__device__ __align__(256) unsigned char g_decode_scratch[kNoallocScratchBytes];

// Device address of g_decode_scratch on the current device.  The array's host
// name is only a stand-in; its device address comes from cudaGetSymbolAddress,
// looked up once per device with that device current.
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::atomic<void*> cache[64];
  if (dev >= 0 && dev < 64) {
    void* p = cache[dev].load(std::memory_order_acquire);
    if (p) {
      *out = p;
      return cudaSuccess;
    }
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_decode_scratch);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64) cache[dev].store(p, std::memory_order_release);
  *out = p;
  return cudaSuccess;
}

}  // namespace

namespace hq {
int decode_int8_clear_first(const void* q, int q_dtype, const int64_t q_strides[3],
                            const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                            const void* k_scale, const void* v_scale, int scale_dtype,
                            const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                            int Hq, int Hkv, int S, int D, float sm_scale, int q_quant, void* out,
                            const int64_t out_strides[3], float* partial_out, void* workspace,
                            size_t workspace_bytes, hq_stream_t stream);
}  // namespace hq

extern "C" int hq_decode_int8_noalloc(const void* q, int q_dtype, const int64_t q_strides[3],
                                      const int8_t* k, const int8_t* v,
                                      const int64_t kv_strides[3], const void* k_scale,
                                      const void* v_scale, int scale_dtype,
                                      const int64_t ksc_strides[3], const int64_t vsc_strides[3],
                                      int B, int Hq, int Hkv, int S, int D, float sm_scale,
                                      int q_quant, void* out, const int64_t out_strides[3],
                                      float* partial_out, hq_stream_t stream) {
  if (B < 0 || Hq <= 0 || Hkv <= 0 || S < 0) return HQ_ERR_INVALID_ARGUMENT;
  const size_t need = hq_decode_workspace_bytes(B, Hq, Hkv, S, D);
  if (need == 0) return HQ_ERR_UNSUPPORTED;                   // head_dim other than 128
  if (need > kNoallocScratchBytes) return HQ_ERR_WORKSPACE;  // beyond the static scratch
  void* ws = nullptr;
  const cudaError_t e = scratch_address(&ws);
  if (e != cudaSuccess) return static_cast<int>(e);
  // the status word and arrival tickets are zeroed on `stream` just before the
  // launch, after the remaining argument checks
  return hq::decode_int8_clear_first(q, q_dtype, q_strides, k, v, kv_strides, k_scale, v_scale,
                                     scale_dtype, ksc_strides, vsc_strides, B, Hq, Hkv, S, D,
                                     sm_scale, q_quant, out, out_strides, partial_out, ws,
                                     kNoallocScratchBytes, stream);
}
