"""torch-facing ops over the C ABI (device memory and streams from PyTorch).

Mirrors the reference's kernel API (src/kernels/quant_kv_triton.py:90-117,
src/kernels/int8_decode_attn_triton.py:101-127) with the same names minus the
``_triton`` suffix, the same argument meaning and the same output shapes and
dtypes:

* ``quant_k_perchannel(x)`` -> (int8 ``[B,H,S,D]``, fp16 scale ``[B,H,1,D]``)
* ``quant_v_pertoken(x)``   -> (int8 ``[B,H,S,D]``, fp16 scale ``[B,H,S,1]``)
* ``int8_decode_attn(q, k_i8, k_sc, v_i8, v_sc, n_rep)`` -> ``[H_q,1,D]`` (or batched)
* ``fp16_decode_attn(q, k, v, n_rep)`` -> the dense twin (fp16 or bf16 K/V)

plus what the cache and the sharded decode need (``append_kv``, ``dequant``,
``decode_partials``, ``decode_combine``).  Every op runs on the current CUDA
stream of the input's device and raises on bad input; there is no CPU path.
"""
from __future__ import annotations

import math
import threading

import torch

from . import _lib
from ._lib import DTYPE_BF16, DTYPE_F16, DTYPE_F32, check

_DT = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}


def _dtype_code(t: torch.Tensor, what: str) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"{what}: unsupported dtype {t.dtype} (float32, bfloat16, float16)") from None


def _cuda(t: torch.Tensor, what: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{what}: expected a CUDA tensor (there is no CPU path)")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(dev: torch.device) -> int:
    """Handle of the current CUDA stream of ``dev``."""
    if _raw_stream is not None:
        return _raw_stream(dev.index if dev.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(dev).cuda_stream


def _status_ptr(word: torch.Tensor | None, dev: torch.device) -> int | None:
    """Device address of an int32 status word on ``dev`` (None: no word)."""
    if word is None:
        return None
    if word.dtype != torch.int32 or word.device != dev or word.numel() < 1:
        raise ValueError("status word: an int32 tensor on the call's device expected")
    return word.data_ptr()


def _rows_ok(t: torch.Tensor) -> bool:
    """[..., D] with unit inner stride and 16-byte aligned rows."""
    es = t.element_size()
    return (t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and
            all((s * es) % 16 == 0 for s in t.stride()[:-1]))


def _rowmajor(t: torch.Tensor) -> torch.Tensor:
    return t if _rows_ok(t) else t.contiguous()


# ---------------------------------------------------------------- workspaces
class _Workspaces:
    """Per (device, stream, kind) scratch buffers, grown on demand.

    Decode workspaces must be zero when first used (arrival tickets); the
    kernel leaves them zero again, so they are zero-filled only when allocated.
    The ticket region's size follows B * Hkv, so a call of another shape could
    find the split partials of an earlier call where its tickets live: decode
    kinds carry B * Hkv (``"decode/8"``), one buffer per shape class.
    """

    def __init__(self):
        self._bufs: dict = {}
        self._lock = threading.Lock()

    def get(self, dev: torch.device, kind: str, nbytes: int) -> torch.Tensor:
        key = (dev.index, _stream(dev), kind)
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                if torch.cuda.is_current_stream_capturing():
                    # memory made during a capture belongs to the graph's pool
                    raise RuntimeError(
                        f"{kind} workspace of {nbytes} bytes needed during CUDA graph capture: "
                        "run the same call once on this stream before capturing it")
                old = buf
                buf = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=dev)
                if old is not None:
                    buf[:4].copy_(old[:4])  # the status word (first error) outlives the growth
                self._bufs[key] = buf
            return buf

    def matching(self, dev: torch.device, prefix: str) -> list:
        """This stream's buffers whose kind starts with ``prefix``."""
        st = _stream(dev)
        with self._lock:
            return [b for (d, s, k), b in self._bufs.items()
                    if d == dev.index and s == st and k.split("/")[0] == prefix]


WORKSPACES = _Workspaces()


# ---------------------------------------------------------------- quantize-on-write
def _check_bhsd(x: torch.Tensor, what: str) -> None:
    _cuda(x, what)
    if x.dim() != 4:
        raise ValueError(f"{what}: expected [B, H, S, D], got {tuple(x.shape)}")
    if x.shape[2] < 1:
        raise ValueError(f"{what}: S must be >= 1 (the reference's amax over an empty axis raises)")


def quant_k_perchannel(x: torch.Tensor, *, out: torch.Tensor | None = None,
                       scale_dtype: torch.dtype | None = torch.float16,
                       scale_out: torch.Tensor | None = None,
                       scale_f32_out: torch.Tensor | None = None,
                       status_into: torch.Tensor | None = None):
    """K per channel: absmax over S of ``x [B,H,S,D]`` -> (int8 codes, scale ``[B,H,1,D]``).

    Same contract as ``quant_k_perchannel_triton`` (src/kernels/quant_kv_triton.py:90-102):
    scale returned as float16 by default; ``scale_dtype=torch.float32`` returns
    the float32 scale of ``quantize_int8`` (reference/page_attention_int8_pytorch.py:23-30);
    ``scale_dtype=None`` writes no scale.  ``out`` / ``scale_out`` /
    ``scale_f32_out`` write into caller buffers (``out`` may be a strided view).
    ``status_into`` (int32 CUDA tensor, first element): the call's device status
    word (0, or ``HQ_ERR_DEVICE_TIMEOUT`` if a bounded wait gave up) is folded
    into it on the stream (the minimum keeps the first error), without a sync.
    """
    _check_bhsd(x, "quant_k_perchannel")
    B, H, S, D = x.shape
    x = _rowmajor(x)
    q = out if out is not None else torch.empty((B, H, S, D), dtype=torch.int8, device=x.device)
    if q.shape != x.shape or q.dtype != torch.int8 or q.device != x.device:
        raise ValueError("quant_k_perchannel: out must be int8 with x's shape and device")
    s16 = scale_out
    s32 = scale_f32_out
    if s16 is None and scale_dtype == torch.float16:
        s16 = torch.empty((B, H, 1, D), dtype=torch.float16, device=x.device)
    if s32 is None and scale_dtype == torch.float32:
        s32 = torch.empty((B, H, 1, D), dtype=torch.float32, device=x.device)
    for t, dt in ((s16, torch.float16), (s32, torch.float32)):
        if t is not None and (t.dtype != dt or not t.is_contiguous() or t.numel() != B * H * D):
            raise ValueError("quant_k_perchannel: scale buffers must be contiguous [B,H,1,D]")
    wsb = _lib.lib().hq_quant_k_workspace_bytes(B, H, D)
    ws = WORKSPACES.get(x.device, "quant_k", wsb)
    rc = _lib.lib().hq_quant_k_perchannel(
        x.data_ptr(), _dtype_code(x, "quant_k_perchannel"), _lib.strides(x.stride(), 4), B, H, S,
        D, q.data_ptr(), _lib.strides(q.stride(), 4), s32.data_ptr() if s32 is not None else None,
        s16.data_ptr() if s16 is not None else None, ws.data_ptr(), ws.numel(),
        _stream(x.device))
    check(rc, "hq_quant_k_perchannel")
    if status_into is not None:
        torch.minimum(status_into[:1], ws[:4].view(torch.int32), out=status_into[:1])
    if scale_dtype == torch.float32:
        return q, s32
    return q, s16


def _static_scale(scale: torch.Tensor, B: int, H: int, D: int, what: str):
    """A static K scale given as [H, D], [1|B, H, 1, D] or [1|B, H, D] -> (tensor, C strides
    (b, h, d)); a batch extent of 1 broadcasts over the batch."""
    _cuda(scale, what)
    if scale.dtype not in (torch.float16, torch.float32):
        raise TypeError(f"{what}: the static scale must be float16 or float32")
    t = scale
    if t.dim() == 2:
        t = t.unsqueeze(0)
    elif t.dim() == 4:
        if t.shape[2] != 1:
            raise ValueError(f"{what}: a 4-d static scale must be [B,H,1,D]")
        t = t[:, :, 0, :]
    if t.dim() != 3 or t.shape[1] != H or t.shape[2] != D or t.shape[0] not in (1, B):
        raise ValueError(f"{what}: static scale shape {tuple(scale.shape)} does not fit "
                         f"B={B}, H={H}, D={D}")
    sb = 0 if t.shape[0] == 1 else t.stride(0)
    return t, _lib.strides((sb, t.stride(1), t.stride(2)), 3)


def quant_k_static(x: torch.Tensor, scale: torch.Tensor, *,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """K per channel with a static (calibrated) scale: ``clamp(rint(x / scale[d]), +-127)``.

    The rule of ``quantize_int8`` (reference/page_attention_int8_pytorch.py:23-30)
    with the scale supplied instead of found - the reference roadmap's static
    quantization (README.md:140), which skips the per-step column maximum.
    ``scale``: ``[H, D]`` or ``[1|B, H, 1, D]`` (float32 or float16), positive.
    Returns int8 codes ``[B,H,S,D]`` (or writes ``out``).
    """
    _check_bhsd(x, "quant_k_static")
    B, H, S, D = x.shape
    x = _rowmajor(x)
    sc, sst = _static_scale(scale, B, H, D, "quant_k_static")
    q = out if out is not None else torch.empty((B, H, S, D), dtype=torch.int8, device=x.device)
    if q.shape != x.shape or q.dtype != torch.int8 or q.device != x.device:
        raise ValueError("quant_k_static: out must be int8 with x's shape and device")
    rc = _lib.lib().hq_quant_k_static(
        x.data_ptr(), _dtype_code(x, "quant_k_static"), _lib.strides(x.stride(), 4), B, H, S, D,
        sc.data_ptr(), _dtype_code(sc, "quant_k_static scale"), sst, q.data_ptr(),
        _lib.strides(q.stride(), 4), _stream(x.device))
    check(rc, "hq_quant_k_static")
    return q


def column_absmax(x: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-channel ``max(|x|)`` over the tokens of ``x [B,H,S,D]`` (``hq_column_absmax``):
    float32 ``[B,H,1,D]`` (or writes ``out``, a contiguous float32 tensor of that
    shape).  An empty ``x`` (S = 0) gives zeros.  The K scale's input for a bulk
    write whose tokens are split over ranks (``sharding.sequence_sharded_quant_k``)."""
    _cuda(x, "column_absmax")
    if x.dim() != 4:
        raise ValueError(f"column_absmax: expected [B, H, S, D], got {tuple(x.shape)}")
    B, H, S, D = x.shape
    x = _rowmajor(x) if S > 0 else x
    if out is None:
        out = torch.empty((B, H, 1, D), dtype=torch.float32, device=x.device)
    elif out.shape != (B, H, 1, D) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("column_absmax: out must be a contiguous float32 [B,H,1,D] tensor")
    rc = _lib.lib().hq_column_absmax(
        x.data_ptr() if S > 0 else out.data_ptr(), _dtype_code(x, "column_absmax"),
        _lib.strides(x.stride(), 4), B, H, S, D, out.data_ptr(), _stream(x.device))
    check(rc, "hq_column_absmax")
    return out


def k_scale_from_amax(amax: torch.Tensor, *, scale_dtype: torch.dtype | None = torch.float16):
    """The reference's per-channel scale ``RN(max(amax, 1e-8) / 127)`` of float32 column
    maxima (``hq_k_scale_from_amax``): returns ``(scale_f32, scale_in_scale_dtype)``
    (the second is None when ``scale_dtype`` is None), both of ``amax``'s shape."""
    _cuda(amax, "k_scale_from_amax amax")
    if amax.dtype != torch.float32 or not amax.is_contiguous():
        raise ValueError("k_scale_from_amax: amax must be contiguous float32")
    s32 = torch.empty_like(amax)
    s16 = None
    if scale_dtype is not None:
        if scale_dtype not in (torch.float16, torch.float32):
            raise TypeError("k_scale_from_amax: scale_dtype must be float16, float32 or None")
        s16 = torch.empty_like(amax, dtype=torch.float16) if scale_dtype == torch.float16 else None
    rc = _lib.lib().hq_k_scale_from_amax(amax.data_ptr(), amax.numel(), s32.data_ptr(),
                                         s16.data_ptr() if s16 is not None else None,
                                         _stream(amax.device))
    check(rc, "hq_k_scale_from_amax")
    return s32, (s16 if scale_dtype == torch.float16 else (s32 if scale_dtype is not None else None))


def calibrate_k_scale(samples, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Static per-channel K scales ``[1, H, 1, D]`` from calibration samples
    (K tensors ``[B, H, S, D]``): ``max(|x|) / 127`` over every sample, batch and
    token, clamped at 1e-8 as ``quantize_int8`` does; the division is done in
    float64 and rounded once."""
    amax = None
    for x in samples:
        m = x.detach().abs().amax(dim=(0, 2), keepdim=True).float()
        amax = m if amax is None else torch.maximum(amax, m)
    if amax is None:
        raise ValueError("calibrate_k_scale: no samples")
    return (amax.clamp(min=1e-8).double() / 127.0).to(dtype)


def quant_v_pertoken(x: torch.Tensor, *, out: torch.Tensor | None = None,
                     scale_dtype: torch.dtype | None = torch.float16,
                     scale_out: torch.Tensor | None = None,
                     scale_f32_out: torch.Tensor | None = None):
    """V per token: absmax over D of ``x [B,H,S,D]`` -> (int8 codes, scale ``[B,H,S,1]``).

    Same contract as ``quant_v_pertoken_triton`` (src/kernels/quant_kv_triton.py:105-117);
    options as ``quant_k_perchannel``.  Scale buffers may be strided ``[B,H,S,1]`` views.
    """
    _check_bhsd(x, "quant_v_pertoken")
    B, H, S, D = x.shape
    x = _rowmajor(x)
    q = out if out is not None else torch.empty((B, H, S, D), dtype=torch.int8, device=x.device)
    if q.shape != x.shape or q.dtype != torch.int8 or q.device != x.device:
        raise ValueError("quant_v_pertoken: out must be int8 with x's shape and device")
    s16 = scale_out
    s32 = scale_f32_out
    if s16 is None and scale_dtype == torch.float16:
        s16 = torch.empty((B, H, S, 1), dtype=torch.float16, device=x.device)
    if s32 is None and scale_dtype == torch.float32:
        s32 = torch.empty((B, H, S, 1), dtype=torch.float32, device=x.device)
    ref = s16 if s16 is not None else s32
    if s16 is not None and s32 is not None and s16.stride() != s32.stride():
        raise ValueError("quant_v_pertoken: both scale buffers must share strides")
    for t, dt in ((s16, torch.float16), (s32, torch.float32)):
        if t is not None and (t.dtype != dt or tuple(t.shape) != (B, H, S, 1)):
            raise ValueError("quant_v_pertoken: scale buffers must be [B,H,S,1]")
    sst = _lib.strides(ref.stride()[:3], 3) if ref is not None else None
    rc = _lib.lib().hq_quant_v_pertoken(
        x.data_ptr(), _dtype_code(x, "quant_v_pertoken"), _lib.strides(x.stride(), 4), B, H, S, D,
        q.data_ptr(), _lib.strides(q.stride(), 4), s32.data_ptr() if s32 is not None else None,
        s16.data_ptr() if s16 is not None else None, sst, _stream(x.device))
    check(rc, "hq_quant_v_pertoken")
    if scale_dtype == torch.float32:
        return q, s32
    return q, s16


def append_kv(k_new: torch.Tensor, v_new: torch.Tensor, k_dst: torch.Tensor, v_dst: torch.Tensor,
              v_scale_dst: torch.Tensor | None = None,
              v_scale_f32_dst: torch.Tensor | None = None,
              k_scale_static: torch.Tensor | None = None) -> None:
    """Append ``S_new <= 64`` tokens with the reference update rule in one launch.

    New K codes use the per-channel scale of the new tokens (not stored: the
    cache keeps its first K scale, tests/qwen_kvcache_full.py:54); V codes use
    per-token scales written to ``v_scale_dst`` (fp16 ``[B,H,S_new,1]`` view)
    and/or ``v_scale_f32_dst``.  ``k_dst`` / ``v_dst`` are int8 views of the
    cache rows at the append position.
    """
    _check_bhsd(k_new, "append_kv")
    _check_bhsd(v_new, "append_kv")
    if k_new.shape != v_new.shape or k_new.dtype != v_new.dtype:
        raise ValueError("append_kv: key and value must match in shape and dtype")
    B, H, S_new, D = k_new.shape
    if S_new > 64:
        raise ValueError("append_kv: at most 64 new tokens per call")
    for t in (k_dst, v_dst):
        if tuple(t.shape) != (B, H, S_new, D) or t.dtype != torch.int8 or t.stride(-1) != 1:
            raise ValueError("append_kv: destinations must be int8 [B,H,S_new,D] views")
    k_new = k_new if k_new.stride(-1) == 1 else k_new.contiguous()
    v_new = v_new if v_new.stride(-1) == 1 else v_new.contiguous()
    ref = v_scale_dst if v_scale_dst is not None else v_scale_f32_dst
    sst = _lib.strides(ref.stride()[:3], 3) if ref is not None else None
    if k_scale_static is not None:  # K codes with the static scale (hq_append_kv_static)
        ksc, kst = _static_scale(k_scale_static, B, H, D, "append_kv")
        rc = _lib.lib().hq_append_kv_static(
            k_new.data_ptr(), v_new.data_ptr(), _dtype_code(k_new, "append_kv"),
            _lib.strides(k_new.stride(), 4), _lib.strides(v_new.stride(), 4), B, H, S_new, D,
            ksc.data_ptr(), _dtype_code(ksc, "append_kv k scale"), kst,
            k_dst.data_ptr(), _lib.strides(k_dst.stride(), 4), v_dst.data_ptr(),
            _lib.strides(v_dst.stride(), 4),
            v_scale_f32_dst.data_ptr() if v_scale_f32_dst is not None else None,
            v_scale_dst.data_ptr() if v_scale_dst is not None else None, sst,
            _stream(k_new.device))
        check(rc, "hq_append_kv_static")
        return
    rc = _lib.lib().hq_append_kv(
        k_new.data_ptr(), v_new.data_ptr(), _dtype_code(k_new, "append_kv"),
        _lib.strides(k_new.stride(), 4), _lib.strides(v_new.stride(), 4), B, H, S_new, D,
        k_dst.data_ptr(), _lib.strides(k_dst.stride(), 4), v_dst.data_ptr(),
        _lib.strides(v_dst.stride(), 4),
        v_scale_f32_dst.data_ptr() if v_scale_f32_dst is not None else None,
        v_scale_dst.data_ptr() if v_scale_dst is not None else None, sst, _stream(k_new.device))
    check(rc, "hq_append_kv")


def append_kv_at(k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor,
                 v_cache: torch.Tensor, v_scale_cache: torch.Tensor, lens: torch.Tensor) -> None:
    """``append_kv`` at the device-resident length ``lens[0]`` (``hq_append_kv_at``).

    ``k_cache`` / ``v_cache`` are the whole int8 capacity buffers ``[B,H,cap,D]``
    and ``v_scale_cache`` their fp16 or fp32 per-token scales ``[B,H,cap,1]``;
    ``lens`` is an int32 ``[4]`` CUDA tensor ``{length, ticket, status, -}``.
    The new rows go to ``lens[0]`` onward and the launch advances ``lens[0]``
    by ``S_new`` on the device, so the same call can be captured in a CUDA
    graph and replayed for every later token.  A full cache writes nothing and
    sets ``lens[2]``.
    """
    _check_bhsd(k_new, "append_kv_at")
    _check_bhsd(v_new, "append_kv_at")
    if k_new.shape != v_new.shape or k_new.dtype != v_new.dtype:
        raise ValueError("append_kv_at: key and value must match in shape and dtype")
    B, H, S_new, D = k_new.shape
    if S_new > 64:
        raise ValueError("append_kv_at: at most 64 new tokens per call")
    cap = k_cache.shape[2]
    for t in (k_cache, v_cache):
        if (t.dim() != 4 or tuple(t.shape[:2]) != (B, H) or t.shape[3] != D or
                t.dtype != torch.int8 or t.stride(-1) != 1 or t.shape[2] != cap):
            raise ValueError("append_kv_at: caches must be int8 [B,H,cap,D] buffers")
    if tuple(v_scale_cache.shape[:3]) != (B, H, cap):
        raise ValueError("append_kv_at: v_scale_cache must be [B,H,cap,1]")
    if lens.dtype != torch.int32 or lens.numel() < 4 or not lens.is_cuda:
        raise ValueError("append_kv_at: lens must be an int32 CUDA tensor of 4 elements")
    k_new = k_new if k_new.stride(-1) == 1 else k_new.contiguous()
    v_new = v_new if v_new.stride(-1) == 1 else v_new.contiguous()
    f32 = v_scale_cache.dtype == torch.float32
    if not f32 and v_scale_cache.dtype != torch.float16:
        raise TypeError("append_kv_at: v_scale_cache must be float16 or float32")
    rc = _lib.lib().hq_append_kv_at(
        k_new.data_ptr(), v_new.data_ptr(), _dtype_code(k_new, "append_kv_at"),
        _lib.strides(k_new.stride(), 4), _lib.strides(v_new.stride(), 4), B, H, S_new, D,
        k_cache.data_ptr(), _lib.strides(k_cache.stride(), 4), v_cache.data_ptr(),
        _lib.strides(v_cache.stride(), 4), v_scale_cache.data_ptr() if f32 else None,
        None if f32 else v_scale_cache.data_ptr(), _lib.strides(v_scale_cache.stride()[:3], 3),
        cap, lens.data_ptr(), _stream(k_new.device))
    check(rc, "hq_append_kv_at")


def dequant(q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype, per_channel: bool,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """``dtype(float(q) * float(scale))`` for an int8 cache tensor ``[B,H,S,D]``.

    tests/qwen_kvcache_full.py:64-65; ``scale`` is ``[B,H,1,D]`` (K, per channel)
    or ``[B,H,S,1]`` (V, per token), float16 or float32.
    """
    _cuda(q, "dequant")
    B, H, S, D = q.shape
    if out is None:
        out = torch.empty((B, H, S, D), dtype=dtype, device=q.device)
    if per_channel:
        sst = (scale.stride(0), scale.stride(1), scale.stride(3))
    else:
        sst = (scale.stride(0), scale.stride(1), scale.stride(2))
    rc = _lib.lib().hq_dequant(
        q.data_ptr(), _lib.strides(q.stride(), 4), B, H, S, D, scale.data_ptr(),
        _dtype_code(scale, "dequant scale"), _lib.strides(sst, 3), int(per_channel),
        out.data_ptr(), _dtype_code(out, "dequant out"), _lib.strides(out.stride(), 4),
        _stream(q.device))
    check(rc, "hq_dequant")
    return out


# ---------------------------------------------------------------- decode attention
def _as_bhd(q: torch.Tensor):
    """q ``[Hq,1,D]`` / ``[B,Hq,1,D]`` / ``[B,Hq,D]`` -> (view ``[B,Hq,D]``, restore fn)."""
    if q.dim() == 3 and q.shape[1] == 1:          # reference layout [H_q, 1, D]
        return q[:, 0, :].unsqueeze(0), lambda o: o[0].unsqueeze(1)
    if q.dim() == 4 and q.shape[2] == 1:          # [B, H_q, 1, D]
        return q[:, :, 0, :], lambda o: o.unsqueeze(2)
    if q.dim() == 3:                              # [B, H_q, D]
        return q, lambda o: o
    raise ValueError(f"decode: q must be [Hq,1,D], [B,Hq,1,D] or [B,Hq,D], got {tuple(q.shape)}")


def _as_bhsd(t: torch.Tensor):
    return t.unsqueeze(0) if t.dim() == 3 else t


_decode_ws_bytes: dict = {}


def decode_workspace(dev, B, Hq, Hkv, S, D) -> torch.Tensor:
    """The (zero-initialised, reused) decode workspace for this shape on ``dev``.
    Its size depends on S only through the tile count, so it is cached per tile count."""
    key = (B, Hq, Hkv, (S + 127) // 128, D)
    nb = _decode_ws_bytes.get(key)
    if nb is None:
        # the size grows with S: the largest S of the 128-token bucket covers it
        nb = _lib.lib().hq_decode_workspace_bytes(B, Hq, Hkv, max(key[3] * 128, 1), D)
        if nb == 0:
            raise ValueError(f"decode: unsupported shape B={B} Hq={Hq} Hkv={Hkv} S={S} D={D}")
        _decode_ws_bytes[key] = nb
    return WORKSPACES.get(dev, f"decode/{B * Hkv}", nb)


_decode_ws = decode_workspace


def _kv_strides(k, v):
    if k.stride() != v.stride():
        raise ValueError("decode: K and V must share strides")
    if k.stride(3) != 1 or k.stride(2) != k.shape[3]:
        raise ValueError("decode: K/V token rows must be contiguous (stride(2) == D)")
    return _lib.strides((k.stride(0), k.stride(1), k.stride(2)), 3)


def _check_cache_shapes(what: str, B: int, D: int, k4, v4, ks4=None, vs4=None) -> None:
    """The library addresses K/V and their scales from the call's counts alone, so each
    tensor must have the shape those counts imply: K and V ``[B,Hkv,S,D]`` (B and D
    those of q), K scales ``[B,Hkv,1,D]``, V scales ``[B,Hkv,S,1]``."""
    _, Hkv, S, _ = k4.shape
    bad = k4.shape[0] != B or k4.shape[3] != D or tuple(v4.shape) != tuple(k4.shape)
    if ks4 is not None:
        bad = bad or tuple(ks4.shape) != (B, Hkv, 1, D) or tuple(vs4.shape) != (B, Hkv, S, 1)
    if bad:
        shapes = ", ".join(f"{n} {tuple(t.shape)}" for n, t in
                           (("k", k4), ("v", v4), ("k_sc", ks4), ("v_sc", vs4)) if t is not None)
        raise ValueError(f"{what}: shapes disagree with q's B={B}, D={D}: {shapes}")


def int8_decode_attn(q, k_i8, k_sc, v_i8, v_sc, n_rep=None, *, sm_scale=None, q_quant=False,
                     out=None, partial_out=None, peers=None, seq_len=None, s_plan=None,
                     overlap_prev=False, append=None, dynamic_tiles=False):
    """Int8 decode attention (split-KV), the contract of ``int8_decode_attn``
    (src/kernels/int8_decode_attn_triton.py:101-113), batched.

    q ``[Hq,1,D]`` | ``[B,Hq,1,D]`` | ``[B,Hq,D]`` (bf16/f16/f32); k_i8, v_i8
    int8 ``[Hkv,S,D]`` | ``[B,Hkv,S,D]``; k_sc ``[.., Hkv,1,D]``; v_sc
    ``[.., Hkv,S,1]`` (f16 or f32).  Returns the output in q's layout and dtype,
    or writes the float32 (m, l, o) partials to ``partial_out [B,Hq,D+2]`` and
    returns it.  ``q_quant`` applies the per-token fake quantization of the
    reference's patched attention (tests/qwen_kvcache_full.py:103).
    ``peers = (buffers, world, rank)`` (``sharding.PeerShardedDecode``): the
    cache holds this rank's token range only, and the kernel exchanges the
    partial softmax state with the other ranks over peer memory and returns
    the output over the whole sequence (``hq_decode_int8_peer``).
    ``seq_len`` (int32 CUDA tensor, first element): the cache length lives on
    the device and K/V/v_sc are capacity buffers; the kernel attends over the
    first ``seq_len[0]`` tokens with a split count planned for ``s_plan``
    tokens (default: the capacity) - ``hq_decode_int8_len``, replayable in a
    CUDA graph while the length grows.
    ``append=(k_new, v_new)`` (with ``seq_len``): the token ``[B,Hkv,1,D]`` (q's
    dtype) is quantized by the reference's update rule, written at row
    ``seq_len[0]`` and attended to in the same launch, which advances the length
    (``hq_decode_append_int8_len``; v_sc must then be the writable capacity buffer).
    ``overlap_prev``: the cache is not written by the kernel launched just
    before this call on the stream; the launch overlaps that kernel's tail
    (programmatic dependent launch, ``hq_decode_int8_ex``).
    ``dynamic_tiles``: the splits of a (sequence, kv head) claim their 128-token
    tiles as they go instead of streaming fixed runs (``HQ_DECODE_DYNAMIC_TILES``;
    needs token-contiguous V scales with 16-byte aligned rows, else the fixed
    runs are used): faster when the blocks are served unevenly, but the float32
    sums are grouped by timing, so results may differ in their last bits from
    call to call.
    """
    for t, n in ((q, "q"), (k_i8, "k_i8"), (k_sc, "k_sc"), (v_i8, "v_i8"), (v_sc, "v_sc")):
        _cuda(t, f"int8_decode_attn {n}")
    if peers is not None and partial_out is not None:
        raise ValueError("int8_decode_attn: peers and partial_out are exclusive")
    if seq_len is not None and (peers is not None or partial_out is not None):
        raise ValueError("int8_decode_attn: seq_len excludes peers and partial_out")
    if (overlap_prev or dynamic_tiles) and (peers is not None or seq_len is not None):
        raise ValueError("int8_decode_attn: overlap_prev and dynamic_tiles exclude peers and seq_len")
    qb, restore = _as_bhd(q)
    k4, v4, ks4, vs4 = _as_bhsd(k_i8), _as_bhsd(v_i8), _as_bhsd(k_sc), _as_bhsd(v_sc)
    B, Hq, D = qb.shape
    _, Hkv, S, _ = k4.shape
    if k4.dtype != torch.int8 or v4.dtype != torch.int8:
        raise TypeError("int8_decode_attn: K/V must be int8")
    _check_cache_shapes("int8_decode_attn", B, D, k4, v4, ks4, vs4)
    if out is not None and tuple(out.shape) != (B, Hq, D):
        raise ValueError(f"int8_decode_attn: out must be [B,Hq,D] = {(B, Hq, D)}")
    if partial_out is not None and tuple(partial_out.shape) != (B, Hq, D + 2):
        raise ValueError(f"int8_decode_attn: partial_out must be [B,Hq,D+2] = {(B, Hq, D + 2)}")
    if ks4.dtype != vs4.dtype or ks4.dtype not in (torch.float16, torch.float32):
        raise TypeError("int8_decode_attn: scales must both be float16 or float32")
    if n_rep is not None and n_rep * Hkv != Hq:
        raise ValueError("int8_decode_attn: n_rep * H_kv != H_q")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    res = None
    if partial_out is None:
        res = out if out is not None else torch.empty((B, Hq, D), dtype=qb.dtype, device=qb.device)
    if append is not None and seq_len is None:
        raise ValueError("int8_decode_attn: append needs seq_len")
    if seq_len is not None:
        if seq_len.dtype != torch.int32 or not seq_len.is_cuda or seq_len.numel() < 1:
            raise ValueError("int8_decode_attn: seq_len must be an int32 CUDA tensor")
        plan = S if s_plan is None else max(0, min(int(s_plan), S))
        if append is not None:
            kn, vn = (_as_bhsd(t) for t in append)
            for t in (kn, vn):
                _cuda(t, "int8_decode_attn append")
                if (tuple(t.shape) != (B, Hkv, 1, D) or t.dtype != qb.dtype or t.stride(3) != 1):
                    raise ValueError("int8_decode_attn: append tensors must be [B,Hkv,1,D] of q's dtype")
            ws = _decode_ws(qb.device, B, Hq, Hkv, plan + 128, D)
            rc = _lib.lib().hq_decode_append_int8_len(
                qb.data_ptr(), _dtype_code(qb, "int8_decode_attn q"), _lib.strides(qb.stride(), 3),
                kn.data_ptr(), vn.data_ptr(), _lib.strides(kn.stride()[:3], 3),
                _lib.strides(vn.stride()[:3], 3), k4.data_ptr(), v4.data_ptr(),
                _kv_strides(k4, v4), ks4.data_ptr(), vs4.data_ptr(), _dtype_code(ks4, "scale"),
                _lib.strides((ks4.stride(0), ks4.stride(1), ks4.stride(3)), 3),
                _lib.strides((vs4.stride(0), vs4.stride(1), vs4.stride(2)), 3), B, Hq, Hkv, S,
                seq_len.data_ptr(), plan, D, float(sm_scale), int(bool(q_quant)), res.data_ptr(),
                _lib.strides(res.stride(), 3), ws.data_ptr(), ws.numel(), _stream(qb.device))
            check(rc, "hq_decode_append_int8_len")
            return restore(res) if out is None else res
        ws = _decode_ws(qb.device, B, Hq, Hkv, plan, D)
        rc = _lib.lib().hq_decode_int8_len(
            qb.data_ptr(), _dtype_code(qb, "int8_decode_attn q"), _lib.strides(qb.stride(), 3),
            k4.data_ptr(), v4.data_ptr(), _kv_strides(k4, v4), ks4.data_ptr(), vs4.data_ptr(),
            _dtype_code(ks4, "scale"),
            _lib.strides((ks4.stride(0), ks4.stride(1), ks4.stride(3)), 3),
            _lib.strides((vs4.stride(0), vs4.stride(1), vs4.stride(2)), 3), B, Hq, Hkv, S,
            seq_len.data_ptr(), plan, D, float(sm_scale), int(bool(q_quant)), res.data_ptr(),
            _lib.strides(res.stride(), 3), ws.data_ptr(), ws.numel(), _stream(qb.device))
        check(rc, "hq_decode_int8_len")
        return restore(res) if out is None else res
    ws = _decode_ws(qb.device, B, Hq, Hkv, S, D)
    ost = _lib.strides(res.stride(), 3) if res is not None else None
    args = (qb.data_ptr(), _dtype_code(qb, "int8_decode_attn q"), _lib.strides(qb.stride(), 3),
            k4.data_ptr(), v4.data_ptr(), _kv_strides(k4, v4), ks4.data_ptr(), vs4.data_ptr(),
            _dtype_code(ks4, "scale"),
            _lib.strides((ks4.stride(0), ks4.stride(1), ks4.stride(3)), 3),
            _lib.strides((vs4.stride(0), vs4.stride(1), vs4.stride(2)), 3), B, Hq, Hkv, S, D,
            float(sm_scale), int(bool(q_quant)), res.data_ptr() if res is not None else None, ost)
    if peers is not None:
        bufs, world, rank = peers
        rc = _lib.lib().hq_decode_int8_peer(*args, ws.data_ptr(), ws.numel(), bufs, world, rank,
                                            _stream(qb.device))
        check(rc, "hq_decode_int8_peer")
        return restore(res) if out is None else res
    if overlap_prev or dynamic_tiles:
        flags = (1 if overlap_prev else 0) | (2 if dynamic_tiles else 0)
        rc = _lib.lib().hq_decode_int8_ex(
            *args, partial_out.data_ptr() if partial_out is not None else None, ws.data_ptr(),
            ws.numel(), flags, _stream(qb.device))
        check(rc, "hq_decode_int8_ex")
    else:
        rc = _lib.lib().hq_decode_int8(
            *args, partial_out.data_ptr() if partial_out is not None else None, ws.data_ptr(),
            ws.numel(), _stream(qb.device))
        check(rc, "hq_decode_int8")
    if partial_out is not None:
        return partial_out
    return restore(res) if out is None else res


def int8_prefill_attn(q, k_i8, k_sc, v_i8, v_sc, n_rep=None, *, sm_scale=None, q_quant=False,
                      out=None, status_into=None):
    """Causal prefill attention over an int8 cache (``hq_prefill_int8``).

    The prefill branch of the reference's patched attention
    (tests/qwen_kvcache_full.py:95-113) over the cache its update() returns
    dequantized (:64-65), in one launch: q ``[B,Hq,Sq,D]`` (bf16/f16), codes
    ``[B,Hkv,S,D]`` with ``S >= Sq`` (the last Sq tokens are the queries'),
    k_sc ``[B,Hkv,1,D]``, v_sc ``[B,Hkv,S,1]`` (f16/f32).  Query i attends keys
    ``0 .. S - Sq + i``.  Returns ``[B,Sq,Hq,D]`` in q's dtype (or writes ``out``,
    a tensor of that shape).  ``status_into``: an int32 CUDA word that receives
    ``HQ_ERR_DEVICE_TIMEOUT`` if a bounded device wait gave up (first error sticks).
    """
    for t, n in ((q, "q"), (k_i8, "k_i8"), (k_sc, "k_sc"), (v_i8, "v_i8"), (v_sc, "v_sc")):
        _cuda(t, f"int8_prefill_attn {n}")
    if q.dim() != 4 or k_i8.dim() != 4:
        raise ValueError("int8_prefill_attn: q [B,Hq,Sq,D] and K/V [B,Hkv,S,D] expected")
    B, Hq, Sq, D = q.shape
    _, Hkv, S, _ = k_i8.shape
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError("int8_prefill_attn: q must be bfloat16 or float16")
    if k_i8.dtype != torch.int8 or v_i8.dtype != torch.int8:
        raise TypeError("int8_prefill_attn: K/V must be int8")
    if k_sc.dtype != v_sc.dtype or k_sc.dtype not in (torch.float16, torch.float32):
        raise TypeError("int8_prefill_attn: scales must both be float16 or float32")
    _check_cache_shapes("int8_prefill_attn", B, D, k_i8, v_i8, k_sc, v_sc)
    if n_rep is not None and n_rep * Hkv != Hq:
        raise ValueError("int8_prefill_attn: n_rep * H_kv != H_q")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    q = q if _rows_ok(q) else q.contiguous()
    if out is None:
        out = torch.empty((B, Sq, Hq, D), dtype=q.dtype, device=q.device)
    elif tuple(out.shape) != (B, Sq, Hq, D) or out.dtype != q.dtype:
        raise ValueError("int8_prefill_attn: out must be [B,Sq,Hq,D] of q's dtype")
    os_ = out.stride()
    rc = _lib.lib().hq_prefill_int8(
        q.data_ptr(), _dtype_code(q, "int8_prefill_attn q"), _lib.strides(q.stride(), 4),
        k_i8.data_ptr(), v_i8.data_ptr(), _kv_strides(k_i8, v_i8), k_sc.data_ptr(),
        v_sc.data_ptr(), _dtype_code(k_sc, "scale"),
        _lib.strides((k_sc.stride(0), k_sc.stride(1), k_sc.stride(3)), 3),
        _lib.strides((v_sc.stride(0), v_sc.stride(1), v_sc.stride(2)), 3), B, Hq, Hkv, Sq, S, D,
        float(sm_scale), int(bool(q_quant)), out.data_ptr(),
        _lib.strides((os_[0], os_[2], os_[1], os_[3]), 4), _status_ptr(status_into, q.device),
        _stream(q.device))
    check(rc, "hq_prefill_int8")
    return out


def fp16_decode_attn(q, k, v, n_rep=None, *, sm_scale=None, q_quant=False, out=None,
                     partial_out=None, cuda_cores=False):
    """Dense twin with the int8 kernel's design (src/kernels/int8_decode_attn_triton.py:116-127):
    128-token TMA tiles, the same ring, split plan and merge, 16-bit tensor-core
    products (``hq_decode_dense``); K/V float16 or bfloat16 (q must match).
    ``cuda_cores=True``: the CUDA-core float32 version (``hq_decode_dense_fma``)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _cuda(t, f"fp16_decode_attn {n}")
    qb, restore = _as_bhd(q)
    k4, v4 = _as_bhsd(k), _as_bhsd(v)
    B, Hq, D = qb.shape
    _, Hkv, S, _ = k4.shape
    if not (k4.dtype == v4.dtype == qb.dtype) or k4.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("fp16_decode_attn: q, K, V must all be float16 or all bfloat16")
    _check_cache_shapes("fp16_decode_attn", B, D, k4, v4)
    if out is not None and tuple(out.shape) != (B, Hq, D):
        raise ValueError(f"fp16_decode_attn: out must be [B,Hq,D] = {(B, Hq, D)}")
    if partial_out is not None and tuple(partial_out.shape) != (B, Hq, D + 2):
        raise ValueError(f"fp16_decode_attn: partial_out must be [B,Hq,D+2] = {(B, Hq, D + 2)}")
    if n_rep is not None and n_rep * Hkv != Hq:
        raise ValueError("fp16_decode_attn: n_rep * H_kv != H_q")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    res = None
    if partial_out is None:
        res = out if out is not None else torch.empty((B, Hq, D), dtype=qb.dtype, device=qb.device)
    ws = _decode_ws(qb.device, B, Hq, Hkv, S, D)
    ost = _lib.strides(res.stride(), 3) if res is not None else None
    fn = _lib.lib().hq_decode_dense_fma if cuda_cores else _lib.lib().hq_decode_dense
    rc = fn(
        qb.data_ptr(), _lib.strides(qb.stride(), 3), k4.data_ptr(), v4.data_ptr(),
        _dtype_code(k4, "fp16_decode_attn kv"), _kv_strides(k4, v4), B, Hq, Hkv, S, D,
        float(sm_scale), int(bool(q_quant)), res.data_ptr() if res is not None else None, ost,
        partial_out.data_ptr() if partial_out is not None else None, ws.data_ptr(), ws.numel(),
        _stream(qb.device))
    check(rc, "hq_decode_dense")
    if partial_out is not None:
        return partial_out
    return restore(res) if out is None else res


dense_decode_attn = fp16_decode_attn


def decode_combine(parts: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """Merge ``parts [P, B, Hq, D+2]`` float32 (m, l, o) partials -> ``[B, Hq, D]``."""
    _cuda(parts, "decode_combine")
    if parts.dtype != torch.float32 or parts.dim() != 4 or not parts.is_contiguous():
        raise ValueError("decode_combine: parts must be contiguous float32 [P, B, Hq, D+2]")
    P, B, Hq, D2 = parts.shape
    D = D2 - 2
    if out is None:
        out = torch.empty((B, Hq, D), dtype=out_dtype, device=parts.device)
    rc = _lib.lib().hq_decode_combine(
        parts.data_ptr(), P, B * Hq * D2, B, Hq, D, out.data_ptr(),
        _dtype_code(out, "decode_combine out"), _lib.strides(out.stride(), 3),
        _stream(parts.device))
    check(rc, "hq_decode_combine")
    return out


def read_status(kind: str = "decode", device=None) -> int:
    """Device status word of this stream's ``kind`` workspaces (0 = ok; else the first
    error found among them)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    bufs = WORKSPACES.matching(dev, kind) or [WORKSPACES.get(dev, kind, 4096)]
    for ws in bufs:
        st = _lib.lib().hq_read_status(ws.data_ptr(), _stream(dev))
        if st != 0:
            return st
    return 0


def set_plan_sms(sms: int, device=None) -> None:
    """Plan this device's grids for ``sms`` SMs (0: the device's own count) -
    ``hq_set_plan_sms``.  Cached decode workspace sizes are dropped, since they
    depend on the planned count."""
    dev = torch.cuda.current_device() if device is None else torch.device(device).index
    check(_lib.lib().hq_set_plan_sms(int(dev), int(sms)), "hq_set_plan_sms")
    _decode_ws_bytes.clear()


# ---------------------------------------------------------------- block-wise per-channel K
KBLOCK_TOKENS = (64, 128, 256)


def kblock_alloc(B: int, H: int, capacity: int, D: int, *, block_tokens: int = 128,
                 dtype: torch.dtype = torch.bfloat16, v_scale_dtype: torch.dtype = torch.float16,
                 device=None) -> dict:
    """Capacity buffers of a block-wise K cache (the layout ``kblock_write`` /
    ``kblock_decode`` use): K / V codes ``[B,H,capacity,D]`` int8, K block scales
    ``[B,H,ceil(capacity/BT),D]`` float32, the K tail ``[B,H,BT,D]`` of ``dtype``
    (originals of the open block) and V scales ``[B,H,capacity]``."""
    if block_tokens not in KBLOCK_TOKENS:
        raise ValueError(f"kblock: block_tokens must be one of {KBLOCK_TOKENS}")
    dev = torch.device("cuda") if device is None else torch.device(device)
    nblk = -(-capacity // block_tokens)
    return {
        "k": torch.zeros((B, H, capacity, D), dtype=torch.int8, device=dev),
        "k_scale": torch.zeros((B, H, nblk, D), dtype=torch.float32, device=dev),
        "k_tail": torch.zeros((B, H, block_tokens, D), dtype=dtype, device=dev),
        "v": torch.zeros((B, H, capacity, D), dtype=torch.int8, device=dev),
        "v_scale": torch.zeros((B, H, capacity), dtype=v_scale_dtype, device=dev),
        "block_tokens": block_tokens,
    }


def _kblock_check(cache: dict, device, B: int, H: int, D: int, what: str) -> None:
    """The cache's buffers must match the call's (B, H, D) and device: the library
    addresses them from the call's counts and cannot see their sizes."""
    kc = cache["k"]
    cap, bt = kc.shape[2], cache["block_tokens"]
    want = {"k": (B, H, cap, D), "v": (B, H, cap, D), "k_scale": (B, H, -(-cap // bt), D),
            "k_tail": (B, H, bt, D), "v_scale": (B, H, cap)}
    for name, shape in want.items():
        t = cache[name]
        if tuple(t.shape) != shape or t.device != device:
            raise ValueError(f"{what}: cache['{name}'] is {tuple(t.shape)} on {t.device}, "
                             f"expected {shape} on {device}")


def kblock_write(k_new: torch.Tensor, v_new: torch.Tensor | None, pos: int | None, cache: dict,
                 lens: torch.Tensor | None = None) -> None:
    """Quantize tokens ``pos .. pos+S_new-1`` (``[B,H,S_new,D]``) into a block-wise K
    cache from ``kblock_alloc`` (``hq_kblock_write``): K per (block, channel), V per
    token, the open block re-coded when a scale grows.  Writes must come in order.
    ``lens`` (int32 CUDA tensor ``{length, ticket, status, -}``): one token written at
    row ``lens[0]``, which the launch advances (``hq_kblock_write_at``; ``pos`` is
    ignored) - the same call for every token, so it replays in a CUDA graph."""
    _check_bhsd(k_new, "kblock_write k")
    k_new = k_new if k_new.stride(3) == 1 else k_new.contiguous()
    B, H, S_new, D = k_new.shape
    kc, ks, kt = cache["k"], cache["k_scale"], cache["k_tail"]
    if kt.dtype != k_new.dtype:
        raise TypeError("kblock_write: k_new must have the tail's dtype")
    _kblock_check(cache, k_new.device, B, H, D, "kblock_write")
    if lens is not None:
        if S_new != 1 or lens.dtype != torch.int32 or not lens.is_cuda or lens.numel() < 4:
            raise ValueError("kblock_write: lens (int32 CUDA [4]) writes one token per call")
    elif int(pos) < 0 or int(pos) + S_new > kc.shape[2]:
        raise ValueError(f"kblock_write: tokens {int(pos)}..{int(pos) + S_new - 1} are outside "
                         f"the capacity {kc.shape[2]}")
    vc = vs = None
    if v_new is not None:
        _check_bhsd(v_new, "kblock_write v")
        v_new = v_new if v_new.stride(3) == 1 else v_new.contiguous()
        if v_new.shape != k_new.shape or v_new.dtype != k_new.dtype:
            raise ValueError("kblock_write: v_new must match k_new")
        vc, vs = cache["v"], cache["v_scale"]
    vs32 = vs if vs is not None and vs.dtype == torch.float32 else None
    vs16 = vs if vs is not None and vs.dtype == torch.float16 else None
    if lens is not None:
        rc = _lib.lib().hq_kblock_write_at(
            k_new.data_ptr(), v_new.data_ptr() if v_new is not None else None,
            _dtype_code(k_new, "kblock_write"), _lib.strides(k_new.stride(), 4),
            _lib.strides(v_new.stride(), 4) if v_new is not None else None, B, H, D,
            int(cache["block_tokens"]), kc.data_ptr(), _lib.strides(kc.stride(), 4),
            ks.data_ptr(), _lib.strides(ks.stride()[:3], 3), kt.data_ptr(),
            _lib.strides(kt.stride(), 4), vc.data_ptr() if vc is not None else None,
            _lib.strides(vc.stride(), 4) if vc is not None else None,
            vs32.data_ptr() if vs32 is not None else None,
            vs16.data_ptr() if vs16 is not None else None,
            _lib.strides(vs.stride()[:3], 3) if vs is not None else None, kc.shape[2],
            lens.data_ptr(), _stream(k_new.device))
        check(rc, "hq_kblock_write_at")
        return
    rc = _lib.lib().hq_kblock_write(
        k_new.data_ptr(), v_new.data_ptr() if v_new is not None else None,
        _dtype_code(k_new, "kblock_write"), _lib.strides(k_new.stride(), 4),
        _lib.strides(v_new.stride(), 4) if v_new is not None else None, B, H, int(pos), S_new, D,
        int(cache["block_tokens"]), kc.data_ptr(), _lib.strides(kc.stride(), 4), ks.data_ptr(),
        _lib.strides(ks.stride()[:3], 3), kt.data_ptr(), _lib.strides(kt.stride(), 4),
        vc.data_ptr() if vc is not None else None,
        _lib.strides(vc.stride(), 4) if vc is not None else None,
        vs32.data_ptr() if vs32 is not None else None,
        vs16.data_ptr() if vs16 is not None else None,
        _lib.strides(vs.stride()[:3], 3) if vs is not None else None, kc.shape[2],
        _stream(k_new.device))
    check(rc, "hq_kblock_write")


def kblock_decode(q: torch.Tensor, cache: dict, S: int, *, sm_scale: float | None = None,
                  out: torch.Tensor | None = None, seq_len: torch.Tensor | None = None,
                  s_plan: int | None = None) -> torch.Tensor:
    """Decode attention of ``q`` (``[B,Hq,D]`` or ``[B,Hq,1,D]``) over the first ``S``
    tokens of a block-wise K cache (``hq_kblock_decode``); output in q's layout and dtype.
    ``seq_len`` (int32 CUDA tensor, first element): the length lives on the device
    (``hq_kblock_decode_len``; ``S`` is ignored, the split count planned for ``s_plan``
    tokens) - replayable in a CUDA graph while the length grows."""
    _cuda(q, "kblock_decode q")
    qb, restore = _as_bhd(q)
    if qb.stride(2) != 1:
        qb = qb.contiguous()
    B, Hq, D = qb.shape
    kc, ks, vc, vs = cache["k"], cache["k_scale"], cache["v"], cache["v_scale"]
    Hkv = kc.shape[1]
    _kblock_check(cache, qb.device, B, Hkv, D, "kblock_decode")
    if Hq % Hkv:
        raise ValueError(f"kblock_decode: {Hq} query heads over {Hkv} kv heads")
    if seq_len is None and not 1 <= int(S) <= kc.shape[2]:
        raise ValueError(f"kblock_decode: S={int(S)} outside 1..{kc.shape[2]} (the capacity)")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    res = out if out is not None else torch.empty((B, Hq, D), dtype=qb.dtype, device=qb.device)
    if seq_len is not None:
        if seq_len.dtype != torch.int32 or not seq_len.is_cuda or seq_len.numel() < 1:
            raise ValueError("kblock_decode: seq_len must be an int32 CUDA tensor")
        cap = kc.shape[2]
        plan = cap if s_plan is None else max(1, min(int(s_plan), cap))
        # sized for the capacity: a captured step never has to grow it
        nb = _lib.lib().hq_kblock_decode_workspace_bytes(B, Hq, Hkv, cap, D)
        if nb == 0:
            raise ValueError(f"kblock_decode: unsupported shape B={B} Hq={Hq} Hkv={Hkv} D={D}")
        ws = WORKSPACES.get(qb.device, f"kblock/{B * Hkv}", nb)
        rc = _lib.lib().hq_kblock_decode_len(
            qb.data_ptr(), _dtype_code(qb, "kblock_decode q"), _lib.strides(qb.stride(), 3),
            kc.data_ptr(), _lib.strides(kc.stride()[:3], 3), ks.data_ptr(),
            _lib.strides(ks.stride()[:3], 3), vc.data_ptr(), _lib.strides(vc.stride()[:3], 3),
            vs.data_ptr(), _dtype_code(vs, "kblock_decode v_scale"),
            _lib.strides(vs.stride()[:3], 3), B, Hq, Hkv, cap, seq_len.data_ptr(), plan, D,
            int(cache["block_tokens"]), float(sm_scale), res.data_ptr(),
            _lib.strides(res.stride(), 3), ws.data_ptr(), ws.numel(), _stream(qb.device))
        check(rc, "hq_kblock_decode_len")
        return restore(res)
    nb = _lib.lib().hq_kblock_decode_workspace_bytes(B, Hq, Hkv, max(int(S), 1), D)
    if nb == 0:
        raise ValueError(f"kblock_decode: unsupported shape B={B} Hq={Hq} Hkv={Hkv} D={D}")
    ws = WORKSPACES.get(qb.device, f"kblock/{B * Hkv}", nb)
    rc = _lib.lib().hq_kblock_decode(
        qb.data_ptr(), _dtype_code(qb, "kblock_decode q"), _lib.strides(qb.stride(), 3),
        kc.data_ptr(), _lib.strides(kc.stride()[:3], 3), ks.data_ptr(),
        _lib.strides(ks.stride()[:3], 3), vc.data_ptr(), _lib.strides(vc.stride()[:3], 3),
        vs.data_ptr(), _dtype_code(vs, "kblock_decode v_scale"), _lib.strides(vs.stride()[:3], 3),
        B, Hq, Hkv, int(S), D, int(cache["block_tokens"]), float(sm_scale), res.data_ptr(),
        _lib.strides(res.stride(), 3), ws.data_ptr(), ws.numel(), _stream(qb.device))
    check(rc, "hq_kblock_decode")
    return restore(res)


def kblock_dequant(cache: dict, S: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """K of the first ``S`` tokens, dequantized (``hq_kblock_dequant``): ``[B,H,S,D]``."""
    kc, ks = cache["k"], cache["k_scale"]
    B, H, _, D = kc.shape
    if not 0 <= int(S) <= kc.shape[2]:
        raise ValueError(f"kblock_dequant: S={int(S)} outside 0..{kc.shape[2]} (the capacity)")
    out = torch.empty((B, H, int(S), D), dtype=dtype, device=kc.device)
    rc = _lib.lib().hq_kblock_dequant(
        kc.data_ptr(), _lib.strides(kc.stride()[:3], 3), ks.data_ptr(),
        _lib.strides(ks.stride()[:3], 3), B, H, int(S), D, int(cache["block_tokens"]),
        out.data_ptr(), _dtype_code(out, "kblock_dequant"), _lib.strides(out.stride(), 4),
        _stream(kc.device))
    check(rc, "hq_kblock_dequant")
    return out
