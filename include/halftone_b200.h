/*
 * halftone_b200.h — C ABI of the B200 (sm_100a) int8 KV-cache kernels.
 *
 * The hot paths of the Halftone int8 KV cache, as plain C entry points:
 *   1. quantize-on-write: symmetric int8, K per channel (absmax over tokens),
 *      V per token (absmax over head_dim), round half to even; the fused
 *      append of new tokens; static calibrated K scales;
 *   2. split-KV (flash-decoding) decode attention over int8 K/V with a float32
 *      online softmax, plus a same-design dense (bf16/f16) twin, the
 *      log-sum-exp combine of partial results, a device-resident-length
 *      variant (graph replay) and a sequence-sharded variant over peer memory;
 *   3. causal prefill attention over the int8 cache.
 *
 * Conventions (every entry point):
 *   - Pointers are device pointers; sizes and strides are in ELEMENTS of the
 *     pointed-to type.  The innermost (head_dim) stride is always 1.
 *   - Tensors are 4-D [B, H, S, D] (batch, head, token, head_dim) unless noted.
 *   - Nothing allocates, except hq_peer_alloc (the receive buffer of the
 *     sequence-sharded exchange, by design).  Kernels that need scratch take a
 *     caller-owned `workspace`; its size comes from the matching
 *     *_workspace_bytes query (hq_decode_int8_noalloc uses a static array of
 *     the library instead).
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default)
 *     without any host synchronisation.
 *   - The return value is HQ_OK (0), a negative hq_status for argument errors
 *     (nothing is launched), or a positive cudaError_t from the launch.
 *   - No C++ exception crosses this boundary; entry points are reentrant and
 *     keep no global mutable state besides per-device caches of the SM count,
 *     kernel occupancy and kernel attributes (set once per device).  The one
 *     exception is hq_decode_int8_noalloc: its calls share one static scratch
 *     array per device, so calls that overlap on the GPU race (see its comment).
 */
#ifndef HALFTONE_B200_H_
#define HALFTONE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define HQ_API __attribute__((visibility("default")))
#else
#define HQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* hq_stream_t; /* == cudaStream_t */

/* Element types. */
enum {
  HQ_DTYPE_F32 = 0,
  HQ_DTYPE_BF16 = 1,
  HQ_DTYPE_F16 = 2,
  HQ_DTYPE_I8 = 3
};

/* Negative status codes (positive values are cudaError_t). */
enum {
  HQ_OK = 0,
  HQ_ERR_INVALID_ARGUMENT = -1, /* null pointer, bad shape, stride or alignment */
  HQ_ERR_UNSUPPORTED = -2,      /* dtype / head_dim / group size not compiled in */
  HQ_ERR_WORKSPACE = -3,        /* workspace missing, too small or misaligned */
  HQ_ERR_DEVICE_TIMEOUT = -4    /* a bounded device-side wait gave up (see hq_read_status) */
};

/* Human-readable text for any return value of this library (static storage). */
HQ_API const char* hq_status_string(int status);
/* Library version, "major.minor.patch". */
HQ_API const char* hq_version(void);

/* ------------------------------------------------------------------------
 * Quantize-on-write, K per channel.
 * Replaces quant_k_perchannel_triton (src/kernels/quant_kv_triton.py:90-102,
 * kernel :16-50) and the K half of QuantizedKVCache.update
 * (tests/qwen_kvcache_full.py:41-43); math of quantize_int8(x, (2,))
 * (reference/page_attention_int8_pytorch.py:23-30).
 *
 * x        [B, H, S, D] of x_dtype (F32/BF16/F16), strides x_strides[4].
 * q        [B, H, S, D] int8 codes, strides q_strides[4].
 * scale_f32, scale_f16 : optional (may be NULL) per-channel scales [B, H, D]
 *          contiguous, float32 and float16 (round to nearest even).
 * Requires S >= 1, D in {64, 128, 256}, 16-byte aligned rows.
 * workspace: >= hq_quant_k_workspace_bytes(B, H, D) bytes, 256-byte aligned;
 *          cleared by this call on `stream`.  The kernel is a persistent
 *          grid working through an ordered queue of chunks; blocks exchange
 *          per-channel maxima and per-group counts through the workspace; a
 *          bounded wait reports HQ_ERR_DEVICE_TIMEOUT in the workspace status
 *          word (hq_read_status) instead of hanging.  The grid is a
 *          cooperative launch: if its blocks cannot all be resident at once
 *          the call returns cudaErrorCooperativeLaunchTooLarge and writes
 *          nothing (see hq_set_plan_sms).
 */
HQ_API size_t hq_quant_k_workspace_bytes(int B, int H, int D);
HQ_API int hq_quant_k_perchannel(const void* x, int x_dtype, const int64_t x_strides[4], int B, int H,
                          int S, int D, int8_t* q, const int64_t q_strides[4], float* scale_f32,
                          uint16_t* scale_f16, void* workspace, size_t workspace_bytes,
                          hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Quantize-on-write, V per token.
 * Replaces quant_v_pertoken_triton (src/kernels/quant_kv_triton.py:105-117,
 * kernel :55-87) and the V half of QuantizedKVCache.update
 * (tests/qwen_kvcache_full.py:45-47); math of quantize_int8(x, (3,)).
 *
 * scale_f32 / scale_f16: optional [B, H, S] per-token scales with strides
 * scale_strides[3] (shared by both outputs).  No workspace.
 */
HQ_API int hq_quant_v_pertoken(const void* x, int x_dtype, const int64_t x_strides[4], int B, int H,
                        int S, int D, int8_t* q, const int64_t q_strides[4], float* scale_f32,
                        uint16_t* scale_f16, const int64_t scale_strides[3], hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused append of S_new tokens to an int8 cache, following the reference
 * storage rule of QuantizedKVCache.update on a non-empty layer
 * (tests/qwen_kvcache_full.py:38-54): the new K codes use the per-channel
 * scale of THESE S_new tokens, which is not stored (the cache keeps its first
 * K scale, line 54); the new V codes use per-token scales, which are stored.
 *
 * k_new, v_new  [B, H, S_new, D] of x_dtype with strides k_strides / v_strides.
 * k_dst, v_dst  int8 cache rows for the new tokens ([B, H, S_new, D] views at
 *               the append position) with strides kq_strides / vq_strides.
 * v_scale_f32 / v_scale_f16: optional [B, H, S_new] views, strides vs_strides[3].
 * Requires 1 <= S_new <= 64, D in {64, 128, 256}.  One launch, no workspace.
 */
HQ_API int hq_append_kv(const void* k_new, const void* v_new, int x_dtype, const int64_t k_strides[4],
                 const int64_t v_strides[4], int B, int H, int S_new, int D, int8_t* k_dst,
                 const int64_t kq_strides[4], int8_t* v_dst, const int64_t vq_strides[4],
                 float* v_scale_f32, uint16_t* v_scale_f16, const int64_t vs_strides[3],
                 hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Quantize-on-write with static (calibrated) K scales: the reference's
 * roadmap item "static quantization from calibration distributions - drop the
 * per-step findmax" (README.md:140); the reference itself has no such path.
 * Codes are the rule of quantize_int8 (reference/page_attention_int8_pytorch.py:23-30)
 * with the scale given instead of found: q = clamp(rint(x / k_scale[d]), -127, 127)
 * (IEEE division, round half to even; values past the calibrated range clamp;
 * NaN inputs give an unspecified code).  One streaming pass, no workspace.
 *
 * hq_quant_k_static: x [B, H, S, D] (F32/BF16/F16) -> q [B, H, S, D] int8.
 *   k_scale [B, H, D] of scale_dtype (F32/F16) addressed by scale_strides[3]
 *   = (b, h, d); a stride of 0 broadcasts (one calibrated scale per head and
 *   channel for every sequence).  Scales must be positive and finite.
 * hq_append_kv_static: hq_append_kv with the K codes of the new tokens made
 *   with the static scale (k_scale, scale_dtype, k_scale_strides as above)
 *   instead of their own per-call maximum; V as in hq_append_kv.
 */
HQ_API int hq_quant_k_static(const void* x, int x_dtype, const int64_t x_strides[4], int B, int H,
                             int S, int D, const void* k_scale, int scale_dtype,
                             const int64_t scale_strides[3], int8_t* q, const int64_t q_strides[4],
                             hq_stream_t stream);
HQ_API int hq_append_kv_static(const void* k_new, const void* v_new, int x_dtype,
                               const int64_t k_strides[4], const int64_t v_strides[4], int B,
                               int H, int S_new, int D, const void* k_scale, int scale_dtype,
                               const int64_t k_scale_strides[3], int8_t* k_dst,
                               const int64_t kq_strides[4], int8_t* v_dst,
                               const int64_t vq_strides[4], float* v_scale_f32,
                               uint16_t* v_scale_f16, const int64_t vs_strides[3],
                               hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Bulk K write sharded along the sequence: each rank holds tokens s0 .. s1 of
 * every sequence but the per-channel scale is that of the whole sequence,
 * scale = RN(max(amax, 1e-8) / 127) with amax over every rank's tokens - the
 * rule of quantize_int8 (reference/page_attention_int8_pytorch.py:23-30)
 * applied per channel as quant_k_perchannel_triton does
 * (src/kernels/quant_kv_triton.py:16-50, 90-103).  The reference runs on one
 * device; its multi-GPU form is this library's.
 *
 * hq_column_absmax: amax[b, h, d] = max |x[b, h, s, d]| over the S tokens of x
 *   [B, H, S, D] (x_dtype F32/BF16/F16, rows 16-byte aligned, D in {64, 128,
 *   256}); amax float32 [B, H, D] contiguous, zero-filled by the call first, so
 *   S = 0 (an empty shard) gives zeros.  Ranks combine the maxima with an
 *   all-reduce (MAX) of the float words.
 * hq_k_scale_from_amax: scale[i] = RN(max(amax[i], 1e-8) / 127) for n values,
 *   into scale_f32 and / or scale_f16 (rounded to half).  hq_quant_k_static with
 *   that scale then gives every rank the codes an unsharded
 *   hq_quant_k_perchannel gives those tokens, bit for bit.
 */
HQ_API int hq_column_absmax(const void* x, int x_dtype, const int64_t x_strides[4], int B, int H,
                            int S, int D, float* amax, hq_stream_t stream);
HQ_API int hq_k_scale_from_amax(const float* amax, int n, float* scale_f32, uint16_t* scale_f16,
                                hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Dequantize an int8 cache tensor: out = dtype(float(code) * float(scale)).
 * Replaces the read path of QuantizedKVCache.update
 * (tests/qwen_kvcache_full.py:64-65) and dequantize_int8
 * (reference/page_attention_int8_pytorch.py:33-34).
 *
 * per_channel != 0: scale is [B, H, D] (K); else [B, H, S] (V).
 * scale_strides[3] are the scale's (b, h, d-or-s) strides; scale_dtype F32 or F16.
 */
HQ_API int hq_dequant(const int8_t* q, const int64_t q_strides[4], int B, int H, int S, int D,
               const void* scale, int scale_dtype, const int64_t scale_strides[3],
               int per_channel, void* out, int out_dtype, const int64_t out_strides[4],
               hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Split-KV int8 decode attention (one query token per sequence).
 * Replaces int8_decode_attn (src/kernels/int8_decode_attn_triton.py:101-113,
 * kernel :15-63) and the decode step of quantized_attention_forward
 * (tests/qwen_kvcache_full.py:95-113): out[b, h] = softmax(q K^T * sm_scale) V
 * over the dequantized cache, GQA q head h reading kv head h / (Hq / Hkv).
 *
 * q        [B, Hq, D] of q_dtype (F32/BF16/F16), strides q_strides[3].
 * k, v     int8 [B, Hkv, S, D], strides kv_strides[3] = (b, h, s) shared by K
 *          and V (token rows contiguous: kv_strides[2] == D).
 * k_scale  per-channel [B, Hkv, D], strides ksc_strides[3]; v_scale per-token
 *          [B, Hkv, S], strides vsc_strides[3]; scale_dtype F32 or F16.
 * q_quant  0: use q as given; 1: per-token symmetric int8 fake quantization
 *          of q first, rounded back to q_dtype (tests/qwen_kvcache_full.py:19-23,103).
 * out      [B, Hq, D] of q_dtype, strides out_strides[3]; or, when
 *          partial_out != NULL, out is ignored and the unnormalised partial
 *          (m, l, o[D]) per (b, h) is written as float32 to
 *          partial_out[(b * Hq + h) * (D + 2)], with m the base-2 running max
 *          of s * sm_scale * log2(e), l = sum 2^(s-m), o = sum 2^(s-m) v.
 * Requires D == 128, Hq / Hkv in {1, 2, 4}, S >= 0 (S == 0 gives zeros).
 * workspace: >= hq_decode_workspace_bytes(B, Hq, Hkv, S, D) bytes, 256-byte
 *          aligned, zero-filled once when allocated; the kernel leaves its
 *          arrival counters (bytes 256 .. 256 + 8 * B * Hkv, rounded up to 256)
 *          zero again.  The split partials follow them, so a workspace serves
 *          calls of one B * Hkv: a call of a larger B * Hkv could find an earlier
 *          call's partials where its counters live - zero the workspace (or use
 *          another) when the shape changes.  The decode kernels of this library
 *          (int8, dense twins, block-wise) share this layout.
 */
HQ_API size_t hq_decode_workspace_bytes(int B, int Hq, int Hkv, int S, int D);
HQ_API int hq_decode_int8(const void* q, int q_dtype, const int64_t q_strides[3], const int8_t* k,
                   const int8_t* v, const int64_t kv_strides[3], const void* k_scale,
                   const void* v_scale, int scale_dtype, const int64_t ksc_strides[3],
                   const int64_t vsc_strides[3], int B, int Hq, int Hkv, int S, int D,
                   float sm_scale, int q_quant, void* out, const int64_t out_strides[3],
                   float* partial_out, void* workspace, size_t workspace_bytes,
                   hq_stream_t stream);

/* ------------------------------------------------------------------------
 * hq_decode_int8 with launch options (no counterpart in the reference).
 * flags: 0, or HQ_DECODE_OVERLAP_PREVIOUS - the K/V codes and the V scales
 *   read by this call are not written by the kernel enqueued just before it on
 *   `stream`.  The launch then uses programmatic dependent launch: its blocks
 *   may start, and request their K/V tiles and V scales, while that kernel is
 *   still finishing; q, the K scales and every write of this call wait for its
 *   completion (and for all memory it wrote).  Typical use: decode launches of
 *   consecutive layers, or a decode whose cache was appended to earlier.
 *   With flags == 0 this is hq_decode_int8.
 */
enum { HQ_DECODE_OVERLAP_PREVIOUS = 1, HQ_DECODE_DYNAMIC_TILES = 2 };
HQ_API int hq_decode_int8_ex(const void* q, int q_dtype, const int64_t q_strides[3],
                             const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                             const void* k_scale, const void* v_scale, int scale_dtype,
                             const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                             int Hq, int Hkv, int S, int D, float sm_scale, int q_quant,
                             void* out, const int64_t out_strides[3], float* partial_out,
                             void* workspace, size_t workspace_bytes, unsigned flags,
                             hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Causal prefill attention over an int8 cache (Sq >= 1 new queries).
 * Replaces the prefill branch of quantized_attention_forward
 * (tests/qwen_kvcache_full.py:95-113) over the dequantized cache that
 * QuantizedKVCache.update returns (:64-65): K/V dequantized to q_dtype as the
 * reference does, q per-token fake quantization when q_quant, float32 softmax
 * of q K^T * sm_scale with query i attending keys 0 .. S - Sq + i.
 *
 * q        [B, Hq, Sq, D] of q_dtype (BF16 or F16), strides q_strides[4].
 * k, v     int8 [B, Hkv, S, D] with strides kv_strides[3] = (b, h, s); the
 *          last Sq cached tokens are the queries' own.
 * k_scale  [B, Hkv, D] (ksc_strides[3]); v_scale [B, Hkv, S] (vsc_strides[3]);
 *          scale_dtype F32 or F16.
 * out      logical [B, Hq, Sq, D] of q_dtype addressed by out_strides[4]
 *          (the reference's [B, Sq, Hq, D] output is strides
 *          (Sq*Hq*D, D, Hq*D, 1)).
 * status   optional int32 device word: a block whose bounded wait for a code
 *          tile gave up sets HQ_ERR_DEVICE_TIMEOUT there (first error sticks;
 *          the rows it served are then incomplete).  May be NULL.
 * Requires D == 128, Hq % Hkv == 0, S >= Sq, 16-byte aligned q rows, code
 * rows of at least 128 bytes with a 16-byte aligned base and strides (the code
 * tiles, and q for even group sizes, are read by TMA).  No workspace: the key
 * tiles of a q tile are split over the blocks of a thread-block cluster, which
 * merge their softmax states through distributed shared memory.  Even group
 * sizes run on tcgen05 with S and O in tensor memory (256 columns per block).
 */
HQ_API int hq_prefill_int8(const void* q, int q_dtype, const int64_t q_strides[4],
                           const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                           const void* k_scale, const void* v_scale, int scale_dtype,
                           const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                           int Hq, int Hkv, int Sq, int S, int D, float sm_scale, int q_quant,
                           void* out, const int64_t out_strides[4], int* status,
                           hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Same-design dense twin: the int8 kernel's design (128-token tensor-map tiles,
 * 3-stage ring, split plan, split ticket and merge) over bf16/f16 K/V
 * (kv_dtype), no scales, both products on the 16-bit tensor cores with float32
 * accumulation.  Replaces fp16_decode_attn (src/kernels/int8_decode_attn_triton.py:116-127,
 * kernel :67-97).  Arguments as hq_decode_int8; q_dtype must equal kv_dtype;
 * K/V rows 16-byte aligned, strides multiples of 8 elements.
 * hq_decode_dense_fma: the same attention on CUDA-core float32 FMAs over
 * 64-token tiles (1-D bulk copies), kept as a second comparison point.
 */
HQ_API int hq_decode_dense(const void* q, const int64_t q_strides[3], const void* k, const void* v,
                    int kv_dtype, const int64_t kv_strides[3], int B, int Hq, int Hkv, int S,
                    int D, float sm_scale, int q_quant, void* out, const int64_t out_strides[3],
                    float* partial_out, void* workspace, size_t workspace_bytes,
                    hq_stream_t stream);
HQ_API int hq_decode_dense_fma(const void* q, const int64_t q_strides[3], const void* k, const void* v,
                    int kv_dtype, const int64_t kv_strides[3], int B, int Hq, int Hkv, int S,
                    int D, float sm_scale, int q_quant, void* out, const int64_t out_strides[3],
                    float* partial_out, void* workspace, size_t workspace_bytes,
                    hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Log-sum-exp combine of n_parts partials in the hq_decode_int8 partial
 * format (e.g. one per GPU of a sequence-sharded cache, gathered into one
 * buffer): parts[p * part_stride + (b * Hq + h) * (D + 2) + {0: m, 1: l, 2..: o}].
 * out [B, Hq, D] of out_dtype with strides out_strides[3].
 * No counterpart in the reference (it has no split); the combine restates the
 * flash-decoding rule  out = sum_p 2^(m_p - M) o_p / sum_p 2^(m_p - M) l_p.
 */
HQ_API int hq_decode_combine(const float* parts, int n_parts, int64_t part_stride, int B, int Hq,
                      int D, void* out, int out_dtype, const int64_t out_strides[3],
                      hq_stream_t stream);

/* ------------------------------------------------------------------------
 * hq_decode_int8 for callers that cannot allocate device memory (no
 * counterpart in the reference).  A runtime that owns all device memory - a
 * plugin inside another engine's decode loop, a binding whose language
 * runtime manages the GPU heap - can hand over its tensors but cannot call
 * cudaMalloc for a workspace.  This entry point takes the same arguments as
 * hq_decode_int8 minus the workspace and keeps its scratch in a static
 * 8 MiB (8,388,608-byte) device array of the library, present on every GPU
 * that loads it until the process exits.  Returns HQ_ERR_WORKSPACE without
 * launching when hq_decode_workspace_bytes(B, Hq, Hkv, S, D) exceeds 8 MiB.
 * It allocates nothing; its first call on a device looks up the array's
 * device address and keeps it (make that first call before any stream
 * capture; calls must not cross a cudaDeviceReset of that device).  All calls
 * share the array: calls that overlap on the GPU race and must be ordered by
 * the caller.  A call whose arguments pass every check clears the array's
 * tickets and status word on `stream` right before its launch; a refused call
 * (invalid counts: HQ_ERR_INVALID_ARGUMENT) enqueues nothing.
 */
HQ_API int hq_decode_int8_noalloc(const void* q, int q_dtype, const int64_t q_strides[3],
                                  const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                                  const void* k_scale, const void* v_scale, int scale_dtype,
                                  const int64_t ksc_strides[3], const int64_t vsc_strides[3],
                                  int B, int Hq, int Hkv, int S, int D, float sm_scale,
                                  int q_quant, void* out, const int64_t out_strides[3],
                                  float* partial_out, hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Device-resident cache length, for a decode step captured once as a CUDA
 * graph and replayed for every later token.  The reference keeps the length
 * as host state (QuantizedKVCache._lens, tests/qwen_kvcache_full.py:36,56-62)
 * and grows the cache with torch.cat (:51-53), so its step cannot be replayed;
 * these two entry points replace the append of update() and the decode call
 * of quantized_attention_forward (:95-113) with launches whose arguments do
 * not change from one token to the next.
 *
 * lens     int32[4] in device memory: {length, ticket, status, unused}; the
 *          caller sets length and zeroes the rest once.
 *
 * hq_append_kv_at: hq_append_kv with k_cache / v_cache / v_scale_* addressing
 *   row 0 of capacity buffers ([B, H, capacity, D] codes, [B, H, capacity]
 *   scales): the S_new new rows go to lens[0] .. lens[0] + S_new - 1 and the
 *   launch advances lens[0] by S_new (its last block to finish, through the
 *   ticket lens[1]).  If lens[0] + S_new > capacity nothing is written,
 *   lens[0] stays, and lens[2] is set to HQ_ERR_INVALID_ARGUMENT
 *   (hq_read_status(lens + 2, stream) reads it).
 *
 * hq_decode_int8_len: hq_decode_int8 (no partial output) over the first
 *   *seq_len tokens of K/V/v_scale buffers that hold S_max tokens (the
 *   capacity); *seq_len is read by the kernel, clamped to [0, S_max].  The
 *   split count is planned on the host for S_plan tokens (the length expected
 *   when the graph replays; 0 <= S_plan <= S_max) and stays fixed; the tokens
 *   per split follow the device length.  workspace: at least
 *   hq_decode_workspace_bytes(B, Hq, Hkv, S_plan, D) bytes, as hq_decode_int8.
 */
HQ_API int hq_append_kv_at(const void* k_new, const void* v_new, int x_dtype,
                           const int64_t k_strides[4], const int64_t v_strides[4], int B, int H,
                           int S_new, int D, int8_t* k_cache, const int64_t kq_strides[4],
                           int8_t* v_cache, const int64_t vq_strides[4], float* v_scale_f32,
                           uint16_t* v_scale_f16, const int64_t vs_strides[3], int capacity,
                           int* lens, hq_stream_t stream);
/* hq_decode_append_int8_len: hq_append_kv_at (one token) and hq_decode_int8_len
 *   in one launch.  k_new / v_new [B, Hkv, 1, D] of q_dtype (strides kn_strides /
 *   vn_strides, (b, h, s)) are quantized by the reference's update rule (K with
 *   this token's own per-channel scale, which is not stored; V per token, scale
 *   stored in scale_dtype) and written at row lens[0] of k / v / v_scale by one
 *   extra block per (sequence, kv head), which also contributes the token's
 *   softmax partial; the other blocks attend over rows [0, lens[0]); the launch
 *   advances lens[0] by one.  The output equals the two-launch sequence to float
 *   round-off.  A full cache (lens[0] == S_max) writes nothing, attends over the
 *   cached rows and sets HQ_ERR_INVALID_ARGUMENT in the workspace status word.
 *   workspace: hq_decode_workspace_bytes(B, Hq, Hkv, S_plan + 128, D) bytes.
 */
HQ_API int hq_decode_append_int8_len(const void* q, int q_dtype, const int64_t q_strides[3],
                                     const void* k_new, const void* v_new,
                                     const int64_t kn_strides[3], const int64_t vn_strides[3],
                                     int8_t* k, int8_t* v, const int64_t kv_strides[3],
                                     const void* k_scale, void* v_scale, int scale_dtype,
                                     const int64_t ksc_strides[3], const int64_t vsc_strides[3],
                                     int B, int Hq, int Hkv, int S_max, int* seq_len, int S_plan,
                                     int D, float sm_scale, int q_quant, void* out,
                                     const int64_t out_strides[3], void* workspace,
                                     size_t workspace_bytes, hq_stream_t stream);
HQ_API int hq_decode_int8_len(const void* q, int q_dtype, const int64_t q_strides[3],
                              const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                              const void* k_scale, const void* v_scale, int scale_dtype,
                              const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                              int Hq, int Hkv, int S_max, const int* seq_len, int S_plan, int D,
                              float sm_scale, int q_quant, void* out,
                              const int64_t out_strides[3], void* workspace,
                              size_t workspace_bytes, hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Sequence-sharded decode over peer memory (no counterpart in the reference,
 * whose cache lives on one device).  Each of `world` GPUs (one process per
 * GPU) holds a contiguous range of the cached tokens of every sequence; one
 * launch of hq_decode_int8_peer per rank computes the rank's partial softmax
 * state (m, l, o), stores it straight into the other ranks' receive buffers
 * over NVLink as 64-bit words that carry the value and the launch's epoch
 * together (no fence, no separate flag), waits (bounded) for the other ranks'
 * words and writes the merged attention output - the result of
 * hq_decode_int8 over the whole sequence - on every rank.  The ranks merge in
 * rank order with the same arithmetic, so their outputs are identical.  The
 * exchange is inside the decode kernel: no collective library call, no extra
 * launch.
 *
 * Receive buffers: each rank allocates hq_peer_buffer_bytes(world, B, Hq, Hkv)
 * bytes with hq_peer_alloc (zero-filled, plus a 64-byte CUDA IPC handle),
 * sends the handle to the other ranks, and opens theirs with hq_peer_open.
 * peer_bufs[w] is rank w's buffer as mapped in this process (its own buffer
 * at w == rank).  Layout: gen [B*Hkv] u32 (launches completed per sequence and
 * kv head, padded to 256 bytes), then part [2][world][B*Hq][D+4] u64 words
 * (m, l, two unused, o[D]; value bits low, epoch high; the halves alternate
 * with the epoch parity).  A buffer serves one (world, B, Hq, Hkv) for its
 * lifetime; the ranks' launches pair up in issue order (also under CUDA graph
 * replay): every rank must make the same sequence of calls on the same buffers.
 *
 * hq_decode_int8_peer: arguments as hq_decode_int8 (S = this rank's tokens,
 * may be 0; no partial output), plus the buffers, world (1..8) and rank.
 * Requires B * Hkv <= resident decode blocks of the GPU (HQ_ERR_UNSUPPORTED
 * otherwise): all blocks run at once, as a cooperative launch (a grid that
 * cannot be resident at once is refused with cudaErrorCooperativeLaunchTooLarge
 * and writes nothing).  A rank whose peers do not arrive
 * within 2 s stops waiting, writes no output and sets HQ_ERR_DEVICE_TIMEOUT in
 * the workspace status word (hq_read_status); the buffers of all ranks must
 * then be freed and allocated again.
 */
HQ_API size_t hq_peer_buffer_bytes(int world, int B, int Hq, int Hkv);
HQ_API int hq_peer_alloc(size_t bytes, void** ptr, void* ipc_handle64);
HQ_API int hq_peer_open(const void* ipc_handle64, void** ptr);
HQ_API int hq_peer_close(void* ptr);
HQ_API int hq_peer_free(void* ptr);
HQ_API int hq_decode_int8_peer(const void* q, int q_dtype, const int64_t q_strides[3],
                               const int8_t* k, const int8_t* v, const int64_t kv_strides[3],
                               const void* k_scale, const void* v_scale, int scale_dtype,
                               const int64_t ksc_strides[3], const int64_t vsc_strides[3], int B,
                               int Hq, int Hkv, int S, int D, float sm_scale, int q_quant,
                               void* out, const int64_t out_strides[3], void* workspace,
                               size_t workspace_bytes, void* const* peer_bufs, int world,
                               int rank, hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Block-wise per-channel K layout (opt-in; the reference's roadmap item
 * "block-wise per-channel K", README.md:141).  No reference interface is
 * replaced: these sit beside hq_append_kv / hq_decode_int8 for a cache that
 * opts in, and remove the retained-first-scale behaviour of
 * QuantizedKVCache.update (tests/qwen_kvcache_full.py:54).
 *
 * Layout (block_tokens BT = 64, 128 or 256):
 *   k_cache  int8 [B, H, capacity, D]        (row r = token r)
 *   k_scale  f32  [B, H, ceil(capacity/BT), D] (scale of block r / BT, channel d)
 *   k_tail   x_dtype [B, H, BT, D]            originals of the open (last,
 *            incomplete) block, row r % BT; the library's own state
 *   v_cache / v_scale: as hq_quant_v_pertoken (per token).
 * Each (block, channel) scale is the reference's rule (quantize_int8,
 * reference/page_attention_int8_pytorch.py:23-30) over the block's tokens, so
 * after any sequence of writes the codes and scales equal a bulk block-wise
 * quantization of every token written so far.
 *
 * hq_kblock_write: writes tokens pos .. pos + S_new - 1 (k_new / v_new
 *   [B, H, S_new, D] of x_dtype, last dim contiguous; v_new may be NULL).  An
 *   append into an open block re-codes the block's earlier rows of the channels
 *   whose scale grew, from k_tail.  Writes must be in order (pos = the current
 *   length).  pos + S_new > capacity -> HQ_ERR_INVALID_ARGUMENT.
 * hq_kblock_decode: decode attention for q [B, Hq, D] over the first S tokens
 *   (D = 64 or 128, Hq / Hkv in {1, 2, 4, 8}); kq_strides / vq_strides are the
 *   (b, h, s) strides of k_cache / v_cache (s a multiple of 16 bytes for K),
 *   ks_strides the (b, h, block) strides of k_scale, vs_strides the (b, h, s)
 *   strides of v_scale (scale_dtype F32 or F16).  out [B, Hq, D] of q_dtype.
 *   workspace: hq_kblock_decode_workspace_bytes(B, Hq, Hkv, S, D) bytes, zero
 *   when first used (the launch leaves it zero), 256-byte aligned.  D = 128
 *   with up to 4 q heads per kv head runs on the int8 tensor cores (the
 *   default layout's kernel with q' rebuilt per block), when K and V share
 *   strides and k_scale rows are 16-byte aligned; the rest on CUDA cores.
 * hq_kblock_write_at / hq_kblock_decode_len (no counterpart in the reference):
 *   the same with the cache length on the device, lens = int32[4] {length,
 *   ticket, status, -} (as hq_append_kv_at), so a decode step replays as a CUDA
 *   graph.  hq_kblock_write_at writes ONE token at row lens[0] (the grid's last
 *   block advances it; a full cache writes nothing and sets lens[2]);
 *   hq_kblock_decode_len attends over the first lens[0] tokens of buffers of
 *   `capacity` tokens with a split count planned for S_plan (tensor-core path
 *   only: D = 128, Hq / Hkv in {1, 2, 4}; otherwise HQ_ERR_UNSUPPORTED).
 * hq_kblock_dequant: out[b, h, s, d] = code * k_scale[b, h, s / BT, d] for
 *   s < S (the read path of a block-wise K cache).
 */
HQ_API int hq_kblock_write(const void* k_new, const void* v_new, int x_dtype,
                           const int64_t k_strides[4], const int64_t v_strides[4], int B, int H,
                           int pos, int S_new, int D, int block_tokens, int8_t* k_cache,
                           const int64_t kq_strides[4], float* k_scale,
                           const int64_t ks_strides[3], void* k_tail,
                           const int64_t kt_strides[4], int8_t* v_cache,
                           const int64_t vq_strides[4], float* v_scale_f32,
                           uint16_t* v_scale_f16, const int64_t vs_strides[3], int capacity,
                           hq_stream_t stream);
HQ_API size_t hq_kblock_decode_workspace_bytes(int B, int Hq, int Hkv, int S, int D);
HQ_API int hq_kblock_decode(const void* q, int q_dtype, const int64_t q_strides[3],
                            const int8_t* k_cache, const int64_t kq_strides[3],
                            const float* k_scale, const int64_t ks_strides[3],
                            const int8_t* v_cache, const int64_t vq_strides[3],
                            const void* v_scale, int scale_dtype, const int64_t vs_strides[3],
                            int B, int Hq, int Hkv, int S, int D, int block_tokens,
                            float sm_scale, void* out, const int64_t out_strides[3],
                            void* workspace, size_t workspace_bytes, hq_stream_t stream);
HQ_API int hq_kblock_write_at(const void* k_new, const void* v_new, int x_dtype,
                              const int64_t k_strides[4], const int64_t v_strides[4], int B,
                              int H, int D, int block_tokens, int8_t* k_cache,
                              const int64_t kq_strides[4], float* k_scale,
                              const int64_t ks_strides[3], void* k_tail,
                              const int64_t kt_strides[4], int8_t* v_cache,
                              const int64_t vq_strides[4], float* v_scale_f32,
                              uint16_t* v_scale_f16, const int64_t vs_strides[3], int capacity,
                              int* lens, hq_stream_t stream);
HQ_API int hq_kblock_decode_len(const void* q, int q_dtype, const int64_t q_strides[3],
                                const int8_t* k_cache, const int64_t kq_strides[3],
                                const float* k_scale, const int64_t ks_strides[3],
                                const int8_t* v_cache, const int64_t vq_strides[3],
                                const void* v_scale, int scale_dtype,
                                const int64_t vs_strides[3], int B, int Hq, int Hkv,
                                int capacity, const int* seq_len, int S_plan, int D,
                                int block_tokens, float sm_scale, void* out,
                                const int64_t out_strides[3], void* workspace,
                                size_t workspace_bytes, hq_stream_t stream);
HQ_API int hq_kblock_dequant(const int8_t* k_cache, const int64_t kq_strides[3],
                             const float* k_scale, const int64_t ks_strides[3], int B, int H,
                             int S, int D, int block_tokens, void* out, int out_dtype,
                             const int64_t out_strides[4], hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Reads (and synchronises `stream` for) the device status word at the start
 * of a quantize-K or decode workspace: HQ_OK, or HQ_ERR_DEVICE_TIMEOUT if a
 * bounded device wait gave up during an earlier call on that workspace.
 */
HQ_API int hq_read_status(const void* workspace, hq_stream_t stream);

/* ------------------------------------------------------------------------
 * Grid planning for a shared GPU (no counterpart in the reference).
 * Every grid of this library is planned for the SMs of the current device;
 * hq_set_plan_sms makes the calls on `device` plan for `sms` SMs instead (0
 * restores the device's own count), for a caller that leaves part of the GPU
 * to other work (another stream's kernels, an MPS partition).  The kernels
 * whose blocks wait for one another - the K quantizer (hq_quant_k_perchannel)
 * and the sequence-sharded decode (hq_decode_int8_peer) - are cooperative
 * launches: a grid that cannot be resident all at once, for whatever reason,
 * is refused at launch with cudaErrorCooperativeLaunchTooLarge (720) and
 * writes nothing, instead of reaching its bounded waits.  Workspace sizes
 * depend on the planned count: query them after changing it.  Not thread-safe
 * against concurrent calls on the same device.
 */
HQ_API int hq_set_plan_sms(int device, int sms);

#ifdef __cplusplus
}
#endif

#endif /* HALFTONE_B200_H_ */
