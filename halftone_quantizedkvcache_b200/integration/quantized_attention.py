"""Drop-in surface of the reference: an int8 HF cache and the patched Qwen3 attention.

* ``QuantizedKVCache`` keeps the API of the reference class
  (tests/qwen_kvcache_full.py:27-89): no-argument constructor,
  ``update(key_states, value_states, layer_idx, cache_kwargs=None)``,
  ``get_seq_length``, ``__len__``, ``storage_bytes``, ``fp16_equiv_bytes`` and
  the per-layer dicts ``_k_i8 / _v_i8 / _k_sc / _v_sc / _lens`` (int8
  ``[B,H,S,D]`` codes, fp16 scales ``[B,H,1,D]`` and ``[B,H,S,1]``).
  Storage is a preallocated capacity buffer per layer (no ``torch.cat``);
  the prefill is quantized by the CUDA K-per-channel / V-per-token kernels and
  every later update by the fused append kernel, with the reference's rule
  (the first K scale is kept, tests/qwen_kvcache_full.py:54).
* ``quantized_attention_forward`` has the signature of the reference's patch
  (tests/qwen_kvcache_full.py:95-113).  For a decode step over this cache it
  runs the split-KV int8 CUDA kernel directly on the codes (with the
  per-token q fake quantization of ``Q_DIMS = (3,)`` fused into its
  prologue); for a prefill it dequantizes the cache with the CUDA dequant
  kernel and evaluates the reference's attention math.

What ``update`` returns follows ``mode``:
  ``"dequant"`` - the whole cache dequantized to the model dtype, exactly the
                  reference's return value (lines 64-66); works with any
                  attention implementation;
  ``"fused"``   - int8 code views tagged with the layer's storage, consumed by
                  ``quantized_attention_forward`` without any dequantization;
  ``"auto"``    - ``"fused"`` while ``quantized_attention_forward`` is installed
                  as Qwen3's eager attention, else ``"dequant"``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from transformers.cache_utils import DynamicCache

from .. import _lib, kernels

Q_DIMS = (3,)  # per-token q fake quantization, as the reference default (line 93)
_ALIGN = 256   # token capacity granularity


def _round_up(n: int, m: int) -> int:
    return (n + m - 1) // m * m


class _DeviceStatus:
    """The device status words a cache's kernels report into: the K quantizer's
    and the fused prefill's (one int32 per device: the quantizer's folded in after
    each call, on the stream; the prefill writes it directly), the
    sticky status words of the decode workspaces its attention used, and the
    status word of each device-length layer (``lens[2]``).  ``eager`` checks
    after every call (synchronises)."""

    def __init__(self, eager: bool = False):
        self.eager = eager
        self.quant: dict = {}       # device index -> int32 [1]
        self.decode: dict = {}      # data_ptr -> decode workspace (uint8)

    def quant_word(self, device) -> torch.Tensor:
        t = self.quant.get(device.index)
        if t is None:
            t = self.quant[device.index] = torch.zeros(1, dtype=torch.int32, device=device)
        return t

    def note_decode(self, ws: torch.Tensor) -> None:
        if ws.data_ptr() not in self.decode:
            self.decode[ws.data_ptr()] = ws

    def words(self, stores):
        """(what, status) of every word; synchronises."""
        out = [(f"quantize-K / prefill on cuda:{d}", int(t.item())) for d, t in self.quant.items()]
        out += [("decode workspace", int(ws[:4].view(torch.int32).item()))
                for ws in self.decode.values()]
        out += [(f"layer {i} device length", int(st.lens[2].item()))
                for i, st in stores.items() if st.lens is not None]
        return out

    def reset(self, stores) -> None:
        for t in self.quant.values():
            t.zero_()
        for ws in self.decode.values():
            ws[:4].zero_()
        for st in stores.values():
            if st.lens is not None:
                st.lens[2].zero_()


class _LayerStore:
    """Capacity buffers of one layer: codes ``[B,H,cap,D]``, fp16 scales."""

    __slots__ = ("k", "v", "k_sc", "v_sc", "length", "st", "lens", "prefill", "pending",
                 "status")

    def __init__(self, B, H, D, cap, device, device_length=False):
        self.k = torch.empty((B, H, cap, D), dtype=torch.int8, device=device)
        self.v = torch.empty((B, H, cap, D), dtype=torch.int8, device=device)
        self.k_sc = torch.empty((B, H, 1, D), dtype=torch.float16, device=device)
        self.v_sc = torch.empty((B, H, cap, 1), dtype=torch.float16, device=device)
        self.length = 0
        # {length, ticket, status, -} on the device (graph-replayable decode steps)
        self.lens = torch.zeros(4, dtype=torch.int32, device=device) if device_length else None
        self.prefill = False  # fused int8 prefill attention over this store
        self.pending = None   # a one-token append left to the next decode (fused_append)
        self.status = None    # the owning cache's _DeviceStatus
        self._strides()

    def _strides(self) -> None:
        """C stride arrays of the buffers, for the direct decode-step calls."""
        k, v, ksc, vsc = self.k, self.v, self.k_sc, self.v_sc
        self.st = (
            _lib.strides(k.stride(), 4), _lib.strides(v.stride(), 4),                # append dst
            _lib.strides(vsc.stride()[:3], 3),                                        # append v scale
            _lib.strides((k.stride(0), k.stride(1), k.stride(2)), 3),                 # decode K/V
            _lib.strides((ksc.stride(0), ksc.stride(1), ksc.stride(3)), 3),           # decode K scale
            _lib.strides((vsc.stride(0), vsc.stride(1), vsc.stride(2)), 3))           # decode V scale

    @property
    def capacity(self) -> int:
        return self.k.shape[2]

    def reserve(self, n: int) -> None:
        if n <= self.capacity:
            return
        if self.lens is not None:
            # captured graphs hold the buffer addresses: no reallocation in this mode
            raise RuntimeError(
                f"QuantizedKVCache: capacity {self.capacity} exhausted ({n} tokens) with "
                "device_lengths=True; construct the cache with a larger capacity")
        B, H, cap, D = self.k.shape
        new = _LayerStore(B, H, D, _round_up(max(2 * cap, n), _ALIGN), self.k.device)
        L = self.length
        new.k[:, :, :L].copy_(self.k[:, :, :L])
        new.v[:, :, :L].copy_(self.v[:, :, :L])
        new.v_sc[:, :, :L].copy_(self.v_sc[:, :, :L])
        new.k_sc.copy_(self.k_sc)
        self.k, self.v, self.k_sc, self.v_sc = new.k, new.v, new.k_sc, new.v_sc
        self.st = new.st

    def flush(self) -> None:
        """Writes a pending one-token append with its own kernel (no decode followed it)."""
        if self.pending is not None:
            k_new, v_new = self.pending
            self.pending = None
            _append_at(self, k_new, v_new, 1)

    def codes(self):
        self.flush()
        L = self.length
        return self.k[:, :, :L], self.v[:, :, :L], self.k_sc, self.v_sc[:, :, :L]


def _tag(t: torch.Tensor, store: _LayerStore) -> torch.Tensor:
    t._hq_store = store
    return t


class _BlockStore:
    """One layer in the block-wise per-channel K layout (``kernels.kblock_alloc``
    buffers): K per (block of ``block_tokens`` tokens, channel), V per token."""

    __slots__ = ("c", "length", "lens")

    def __init__(self, B, H, D, cap, block, dtype, device, device_length=False):
        self.c = kernels.kblock_alloc(B, H, cap, D, block_tokens=block, dtype=dtype,
                                      device=device)
        self.length = 0
        # {length, ticket, status, -} on the device (graph-replayable decode steps)
        self.lens = torch.zeros(4, dtype=torch.int32, device=device) if device_length else None

    def reserve(self, n: int) -> None:
        cap = self.c["k"].shape[2]
        if n <= cap:
            return
        if self.lens is not None:
            # captured graphs hold the buffer addresses: no reallocation in this mode
            raise RuntimeError(
                f"QuantizedKVCache: capacity {cap} exhausted ({n} tokens) with "
                "device_lengths=True; construct the cache with a larger capacity")
        B, H, _, D = self.c["k"].shape
        L, bt = self.length, self.c["block_tokens"]
        new = kernels.kblock_alloc(B, H, _round_up(max(n, 2 * cap), _ALIGN), D, block_tokens=bt,
                                   dtype=self.c["k_tail"].dtype,
                                   v_scale_dtype=self.c["v_scale"].dtype, device=self.c["k"].device)
        nb = -(-L // bt)
        for key in ("k", "v", "v_scale"):
            new[key][:, :, :L].copy_(self.c[key][:, :, :L])
        new["k_scale"][:, :, :nb].copy_(self.c["k_scale"][:, :, :nb])
        new["k_tail"].copy_(self.c["k_tail"])
        self.c = new

    def codes(self):
        L = self.length
        return self.c["k"][:, :, :L], self.c["v"][:, :, :L]

    def nbytes(self) -> int:
        L, bt = self.length, self.c["block_tokens"]
        k = self.c["k"][:, :, :L]
        return (2 * k.numel() + 4 * self.c["k_scale"][:, :, :-(-L // bt)].numel()
                + self.c["v_scale"].element_size() * self.c["v_scale"][:, :, :L].numel())


_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16,
           torch.float16: _lib.DTYPE_F16}


def _append_direct(st: _LayerStore, k_new: torch.Tensor, v_new: torch.Tensor, L: int,
                   S_new: int) -> bool:
    """The append of a decode step straight through the C ABI (``hq_append_kv``): the
    destinations are rows L.. of the layer's own buffers, addressed by pointer
    offset.  Returns False (caller takes the general path) for unusual inputs."""
    dt = _DTYPES.get(k_new.dtype)
    if (dt is None or v_new.dtype != k_new.dtype or k_new.shape != v_new.shape or
            not k_new.is_cuda or k_new.stride(-1) != 1 or v_new.stride(-1) != 1):
        return False
    B, H, _, D = k_new.shape
    k, v, vsc = st.k, st.v, st.v_sc
    s_k, s_v, s_vsc = st.st[0], st.st[1], st.st[2]
    rc = _lib.lib().hq_append_kv(
        k_new.data_ptr(), v_new.data_ptr(), dt, _lib.strides(k_new.stride(), 4),
        _lib.strides(v_new.stride(), 4), B, H, S_new, D,
        k.data_ptr() + L * k.stride(2), s_k, v.data_ptr() + L * v.stride(2), s_v,
        None, vsc.data_ptr() + 2 * L * vsc.stride(2), s_vsc, kernels._stream(k_new.device))
    _lib.check(rc, "hq_append_kv")
    return True


def _append_at(st: _LayerStore, k_new: torch.Tensor, v_new: torch.Tensor, S_new: int) -> None:
    """Device-length append (``hq_append_kv_at``): rows at ``lens[0]``, which the
    launch advances; the call is the same for every token, so it replays in a graph."""
    dt = _DTYPES.get(k_new.dtype)
    if (dt is None or v_new.dtype != k_new.dtype or k_new.shape != v_new.shape or
            not k_new.is_cuda or k_new.stride(-1) != 1 or v_new.stride(-1) != 1):
        kernels.append_kv_at(k_new, v_new, st.k, st.v, st.v_sc, st.lens)
        return
    B, H, _, D = k_new.shape
    k, v, vsc = st.k, st.v, st.v_sc
    rc = _lib.lib().hq_append_kv_at(
        k_new.data_ptr(), v_new.data_ptr(), dt, _lib.strides(k_new.stride(), 4),
        _lib.strides(v_new.stride(), 4), B, H, S_new, D, k.data_ptr(), st.st[0], v.data_ptr(),
        st.st[1], None, vsc.data_ptr(), st.st[2], k.shape[2], st.lens.data_ptr(),
        kernels._stream(k_new.device))
    _lib.check(rc, "hq_append_kv_at")


def _decode_direct(st: _LayerStore, query: torch.Tensor, n_rep: int, scaling: float,
                   q_quant: bool):
    """The decode step straight through the C ABI (``hq_decode_int8``) on the layer's
    buffers: q ``[B,Hq,1,D]`` in, ``[B,1,Hq,D]`` out.  None for unusual inputs."""
    dt = _DTYPES.get(query.dtype)
    B, Hq, _, D = query.shape
    k, v, ksc, vsc = st.k, st.v, st.k_sc, st.v_sc
    Hkv, S = k.shape[1], st.length
    if dt is None or query.stride(3) != 1 or k.stride(2) != D or Hkv * n_rep != Hq:
        return None
    out = torch.empty((B, 1, Hq, D), dtype=query.dtype, device=query.device)
    # with the length on the device a captured step replays at every later length, so the
    # workspace is sized once for the buffer's capacity: a capture never has to grow it
    cap = k.shape[2] if st.lens is not None else S
    ws = kernels.decode_workspace(query.device, B, Hq, Hkv, cap, D)
    qs = query.stride()
    if st.lens is not None and st.pending is not None:
        k_new, v_new = st.pending
        if k_new.dtype == query.dtype and k_new.shape == (B, Hkv, 1, D):
            # the pending one-token append, inside the decode launch
            st.pending = None
            wsa = kernels.decode_workspace(query.device, B, Hq, Hkv, cap + 128, D)
            rc = _lib.lib().hq_decode_append_int8_len(
                query.data_ptr(), dt, _lib.strides((qs[0], qs[1], 1), 3), k_new.data_ptr(),
                v_new.data_ptr(), _lib.strides(k_new.stride()[:3], 3),
                _lib.strides(v_new.stride()[:3], 3), k.data_ptr(), v.data_ptr(), st.st[3],
                ksc.data_ptr(), vsc.data_ptr(), _lib.DTYPE_F16, st.st[4], st.st[5], B, Hq, Hkv,
                k.shape[2], st.lens.data_ptr(), S - 1, D, float(scaling), int(q_quant),
                out.data_ptr(), _lib.strides((Hq * D, D, 1), 3), wsa.data_ptr(), wsa.numel(),
                kernels._stream(query.device))
            _lib.check(rc, "hq_decode_append_int8_len")
            _note_decode(st, wsa)
            return out
        st.flush()
    if st.lens is not None:
        # length on the device; the split count is planned for the host's count
        rc = _lib.lib().hq_decode_int8_len(
            query.data_ptr(), dt, _lib.strides((qs[0], qs[1], 1), 3), k.data_ptr(), v.data_ptr(),
            st.st[3], ksc.data_ptr(), vsc.data_ptr(), _lib.DTYPE_F16, st.st[4], st.st[5],
            B, Hq, Hkv, k.shape[2], st.lens.data_ptr(), S, D, float(scaling), int(q_quant),
            out.data_ptr(), _lib.strides((Hq * D, D, 1), 3), ws.data_ptr(), ws.numel(),
            kernels._stream(query.device))
        _lib.check(rc, "hq_decode_int8_len")
        _note_decode(st, ws)
        return out
    rc = _lib.lib().hq_decode_int8(
        query.data_ptr(), dt, _lib.strides((qs[0], qs[1], 1), 3), k.data_ptr(), v.data_ptr(),
        st.st[3], ksc.data_ptr(), vsc.data_ptr(), _lib.DTYPE_F16, st.st[4], st.st[5],
        B, Hq, Hkv, S, D, float(scaling), int(q_quant), out.data_ptr(),
        _lib.strides((Hq * D, D, 1), 3), None, ws.data_ptr(), ws.numel(),
        kernels._stream(query.device))
    _lib.check(rc, "hq_decode_int8")
    _note_decode(st, ws)
    return out


def _note_decode(st: _LayerStore, ws: torch.Tensor) -> None:
    """Records the decode workspace whose status word this layer's decode reports into."""
    status = st.status
    if status is not None:
        status.note_decode(ws)
        if status.eager:
            _raise_on_status(status.words({}))


def _raise_on_status(words) -> None:
    bad = [(what, v) for what, v in words if v != 0]
    if bad:
        raise RuntimeError("QuantizedKVCache: device status: " + "; ".join(
            f"{what}: {_lib.status_string(v)} ({v})" for what, v in bad))


class QuantizedKVCache(DynamicCache):
    """int8 KV cache, drop-in for the reference's ``QuantizedKVCache``.

    ``device_lengths=True`` keeps each layer's length on the device as well:
    single-token (<= 64) appends write at the device length and advance it, and
    the fused decode reads it, so a decode step (``update`` + the patched
    attention for every layer) captured once with ``torch.cuda.graph`` replays
    for every later token.  It needs ``mode="fused"`` and a ``capacity`` that
    covers the whole session (buffers are never reallocated in this mode).
    The host-side length (``get_seq_length``, the ``_lens`` view) advances on
    eager calls only; after graph replays call ``sync_lengths()``.

    ``fused_prefill=True`` (fused mode): multi-token steps (prefill, or an
    append of several tokens) under a causal mask attend over the int8 cache
    with one CUDA kernel (``kernels.int8_prefill_attn``) instead of
    dequantizing it and running the reference's torch math; the result is the
    same attention in float32 on the same 16-bit inputs (the reference rounds
    its scores to bf16 first).

    ``static_k_scale``: calibrated per-channel K scales (``kernels.calibrate_k_scale``),
    one tensor for every layer or a sequence / dict indexed by layer; each is
    ``[H, D]`` or ``[1|B, H, 1, D]``.  K is then coded with that scale on every
    write (``kernels.quant_k_static``; appends with ``hq_append_kv_static``), no
    per-step column maximum is searched, and the stored K scale is that scale
    (float16).  This is the reference roadmap's static quantization
    (README.md:140), not its default rule; V stays per token.

    ``fused_append=True`` (with ``device_lengths``): a one-token ``update`` is left
    pending and the patched attention that follows performs it inside the decode
    launch (``hq_decode_append_int8_len``) - one kernel per layer and step instead
    of two.  Anything that reads the cache first (another ``update``, the code
    views, ``sync_lengths``) writes the pending token with the append kernel.

    Device status: kernels whose blocks wait for one another give up after a
    bounded wait and report ``HQ_ERR_DEVICE_TIMEOUT`` in a status word instead of
    hanging; a device-length append into a full layer reports there too.
    ``check()`` reads every status word this cache's kernels report into and
    raises ``RuntimeError`` if any is set (it synchronises); ``reset_status()``
    clears them.  ``check_status=True`` runs ``check()`` after every ``update``
    and every decode step of this cache (a host synchronisation per call: for
    debugging, or where a silent failure must never pass).
    """

    def __init__(self, mode: str = "auto", capacity: int | None = None,
                 device_lengths: bool = False, fused_prefill: bool = False,
                 static_k_scale=None, fused_append: bool = False,
                 k_block_tokens: int | None = None, check_status: bool = False):
        super().__init__()
        self._status = _DeviceStatus(eager=check_status)
        if k_block_tokens is not None:
            if k_block_tokens not in kernels.KBLOCK_TOKENS:
                raise ValueError(f"k_block_tokens must be one of {kernels.KBLOCK_TOKENS}")
            if mode != "fused" or fused_append or static_k_scale is not None or fused_prefill:
                raise ValueError("k_block_tokens needs mode='fused' and excludes fused_append, "
                                 "fused_prefill and static_k_scale")
        self.k_block_tokens = k_block_tokens
        self._kblock: dict[int, _BlockStore] = {}
        if mode not in ("auto", "fused", "dequant"):
            raise ValueError(f"mode must be auto, fused or dequant, not {mode!r}")
        if device_lengths and mode != "fused":
            raise ValueError("device_lengths=True needs mode='fused'")
        if fused_prefill and mode != "fused":
            raise ValueError("fused_prefill=True needs mode='fused'")
        self.mode = mode
        self.capacity = capacity
        self.device_lengths = device_lengths
        self.fused_prefill = fused_prefill
        if static_k_scale is not None and device_lengths:
            raise ValueError("static_k_scale and device_lengths are not combined")
        if fused_append and not device_lengths:
            raise ValueError("fused_append needs device_lengths=True")
        self.fused_append = fused_append
        self.static_k_scale = static_k_scale
        self._store: dict[int, _LayerStore] = {}

    def sync_lengths(self) -> dict:
        """Read the device lengths back into the host view (synchronises);
        raises if a device-side append found its layer full."""
        self._flush()
        stores = list(self._store.items()) + list(self._kblock.items())
        for i, st in stores:
            if st.lens is not None:
                length, _, status, _ = (int(x) for x in st.lens.tolist())
                if status != 0:
                    raise RuntimeError(f"QuantizedKVCache: layer {i}: append past the capacity "
                                       f"{st.c['k'].shape[2] if hasattr(st, 'c') else st.capacity}"
                                       f" (status {status})")
                st.length = length
        return self._lens

    def _flush(self) -> None:
        for st in self._store.values():
            st.flush()

    def check(self) -> None:
        """Raises ``RuntimeError`` if a status word of this cache's kernels is set:
        a bounded device-side wait that gave up (``HQ_ERR_DEVICE_TIMEOUT``) in the
        K quantizer or the decode, or a device-length append past the capacity.
        Synchronises."""
        self._flush()
        _raise_on_status(self._status.words({**self._store, **self._kblock}))

    def reset_status(self) -> None:
        """Clears the status words ``check`` reads (on the current stream)."""
        self._status.reset({**self._store, **self._kblock})

    # -- reference-compatible views (tests/qwen_kvcache_full.py:34-36)
    @property
    def _k_i8(self):
        self._flush()
        return {i: s.k[:, :, : s.length] for i, s in self._store.items()}

    @property
    def _v_i8(self):
        self._flush()
        return {i: s.v[:, :, : s.length] for i, s in self._store.items()}

    @property
    def _k_sc(self):
        return {i: s.k_sc for i, s in self._store.items()}

    @property
    def _v_sc(self):
        self._flush()
        return {i: s.v_sc[:, :, : s.length] for i, s in self._store.items()}

    @property
    def _lens(self):
        lens = {i: s.length for i, s in self._store.items()}
        lens.update({i: s.length for i, s in self._kblock.items()})
        return lens

    def _fused(self) -> bool:
        return self.mode == "fused" or (self.mode == "auto" and is_installed())

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        """Quantize the new K/V into the layer's int8 storage (tests/qwen_kvcache_full.py:38-66)."""
        if key_states.shape != value_states.shape:
            raise ValueError("QuantizedKVCache.update: key and value shapes differ")
        B, H, S_new, D = key_states.shape
        if self.k_block_tokens is not None:
            return self._update_blockwise(key_states, value_states, layer_idx)
        st = self._store.get(layer_idx)
        if st is None:
            cap = _round_up(max(S_new + _ALIGN, self.capacity or 0), _ALIGN)
            st = _LayerStore(B, H, D, cap, key_states.device, self.device_lengths)
            st.prefill = self.fused_prefill
            st.status = self._status
            ks = self._static_scale(layer_idx)
            if ks is not None:
                kernels.quant_k_static(key_states, ks, out=st.k[:, :, :S_new])
                st.k_sc.copy_(ks.reshape(-1, H, 1, D).expand(B, H, 1, D))
            else:
                kernels.quant_k_perchannel(key_states, out=st.k[:, :, :S_new], scale_out=st.k_sc,
                                           status_into=self._status.quant_word(key_states.device))
            kernels.quant_v_pertoken(value_states, out=st.v[:, :, :S_new],
                                     scale_out=st.v_sc[:, :, :S_new])
            st.length = S_new
            if st.lens is not None:
                st.lens[0].fill_(S_new)
            self._store[layer_idx] = st
        else:
            if st.k.shape[0] != B or st.k.shape[1] != H or st.k.shape[3] != D:
                raise ValueError("QuantizedKVCache.update: batch/head shape changed for this layer")
            st.flush()
            L = st.length
            st.reserve(L + S_new)
            ks = self._static_scale(layer_idx)
            if ks is not None:
                kdst, vdst = st.k[:, :, L:L + S_new], st.v[:, :, L:L + S_new]
                vsc = st.v_sc[:, :, L:L + S_new]
                if S_new <= 64:
                    kernels.append_kv(key_states, value_states, kdst, vdst, v_scale_dst=vsc,
                                      k_scale_static=ks)
                else:
                    kernels.quant_k_static(key_states, ks, out=kdst)
                    kernels.quant_v_pertoken(value_states, out=vdst, scale_out=vsc)
            elif (st.lens is not None and S_new == 1 and self.fused_append and
                  key_states.dtype == value_states.dtype and key_states.stride(-1) == 1 and
                  value_states.stride(-1) == 1):
                st.pending = (key_states, value_states)  # written by the decode launch
            elif st.lens is not None and S_new <= 64:
                _append_at(st, key_states, value_states, S_new)  # position on the device
            elif S_new <= 64 and _append_direct(st, key_states, value_states, L, S_new):
                pass  # the decode-step path: one launch, no views
            else:
                kdst, vdst = st.k[:, :, L:L + S_new], st.v[:, :, L:L + S_new]
                vsc = st.v_sc[:, :, L:L + S_new]
                if S_new <= 64:
                    kernels.append_kv(key_states, value_states, kdst, vdst, v_scale_dst=vsc)
                else:
                    # codes with the new tokens' own per-channel scale; that scale is not kept
                    kernels.quant_k_perchannel(
                        key_states, out=kdst, scale_dtype=None,
                        status_into=self._status.quant_word(key_states.device))
                    kernels.quant_v_pertoken(value_states, out=vdst, scale_out=vsc)
                if st.lens is not None:  # eager multi-token append: host length is current
                    st.lens[0].fill_(L + S_new)
            st.length = L + S_new
        L = st.length
        if self._status.eager:  # (no flush: a pending fused append stays pending)
            _raise_on_status(self._status.words(self._store))
        k, v = st.k[:, :, :L], st.v[:, :, :L]
        if self._fused():
            return _tag(k, st), _tag(v, st)
        return (kernels.dequant(k, st.k_sc, key_states.dtype, per_channel=True),
                kernels.dequant(v, st.v_sc[:, :, :L], value_states.dtype, per_channel=False))

    def _update_blockwise(self, key_states, value_states, layer_idx):
        """The opt-in block-wise per-channel K layout: every write goes through
        ``kernels.kblock_write`` (K per block of tokens and channel, the open block
        re-coded as it grows; V per token).  Returns the codes tagged for the
        patched attention, which decodes them with ``kernels.kblock_decode``."""
        B, H, S_new, D = key_states.shape
        st = self._kblock.get(layer_idx)
        if st is None:
            cap = _round_up(max(S_new + _ALIGN, self.capacity or 0), _ALIGN)
            st = _BlockStore(B, H, D, cap, self.k_block_tokens, key_states.dtype,
                             key_states.device, self.device_lengths)
            self._kblock[layer_idx] = st
        elif tuple(st.c["k"].shape[:2]) != (B, H) or st.c["k"].shape[3] != D:
            raise ValueError("QuantizedKVCache.update: batch/head shape changed for this layer")
        st.reserve(st.length + S_new)
        if st.lens is not None and S_new == 1:
            kernels.kblock_write(key_states, value_states, None, st.c, lens=st.lens)  # at lens[0]
        else:
            kernels.kblock_write(key_states, value_states, st.length, st.c)
            if st.lens is not None:  # eager multi-token write: the host length is current
                st.lens[0].fill_(st.length + S_new)
        st.length += S_new
        k, v = st.codes()
        k._hq_kblock = st
        v._hq_kblock = st
        return k, v

    def _static_scale(self, layer_idx):
        s = self.static_k_scale
        if s is None or isinstance(s, torch.Tensor):
            return s
        return s[layer_idx]

    def get_seq_length(self, layer_idx=0, cache_position=None):
        st = self._store.get(layer_idx) or self._kblock.get(layer_idx)
        return st.length if st is not None else 0

    def __len__(self):
        return len(self._store) + len(self._kblock)

    def storage_bytes(self):
        """int8 codes at 1 B, fp16 scales at 2 B (tests/qwen_kvcache_full.py:75-82);
        block-wise K scales at 4 B."""
        b = sum(s.nbytes() for s in self._kblock.values())
        for s in self._store.values():
            b += 2 * s.k[:, :, : s.length].numel()
            b += 2 * (s.k_sc.numel() + s.v_sc[:, :, : s.length].numel())
        return b

    def fp16_equiv_bytes(self):
        """Same K/V held in fp16 (tests/qwen_kvcache_full.py:84-89)."""
        return (sum(4 * s.k[:, :, : s.length].numel() for s in self._store.values())
                + sum(4 * s.codes()[0].numel() for s in self._kblock.values()))


# ---------------------------------------------------------------- attention patch
def _fake_quant(x: torch.Tensor, dims) -> torch.Tensor:
    """tests/qwen_kvcache_full.py:19-23, with IEEE true divisions on the GPU."""
    xf = x.float()
    amax = xf.abs().amax(dim=dims, keepdim=True).clamp(min=1e-8)
    scale = amax / torch.full((), 127.0, device=x.device)
    codes = torch.clamp(torch.round(xf / scale), -127, 127)
    return (codes * scale).to(x.dtype)


def _reference_math(module, q, key, value, attention_mask, scaling, dropout):
    """The reference's attention math (tests/qwen_kvcache_full.py:104-113)."""
    n_rep = module.num_key_value_groups
    k = key if n_rep == 1 else key.repeat_interleave(n_rep, dim=1)
    v = value if n_rep == 1 else value.repeat_interleave(n_rep, dim=1)
    scores = torch.matmul(q, k.transpose(2, 3)) * scaling
    if attention_mask is not None:
        m = attention_mask[:, :, :, : k.shape[-2]]
        if m.shape[-1] != k.shape[-2] and m.shape[-1] != 1:
            # an append of several tokens onto a cache: causal over the whole cache
            Sq, Sk = q.shape[2], k.shape[2]
            pos_q = torch.arange(Sk - Sq, Sk, device=q.device)[:, None]
            allowed = torch.arange(Sk, device=q.device)[None, :] <= pos_q
            m = torch.zeros((Sq, Sk), dtype=scores.dtype, device=q.device).masked_fill(
                ~allowed, torch.finfo(scores.dtype).min)
        scores = scores + m
    attn = F.softmax(scores, dim=-1, dtype=torch.float32).to(q.dtype)
    attn = F.dropout(attn, p=dropout, training=module.training)
    return torch.matmul(attn, v).transpose(1, 2).contiguous()


def _is_causal(mask, Sq: int, S: int) -> bool:
    """True when the additive mask is the causal mask of the last Sq of S tokens
    (0 where key j <= S - Sq + i, a large negative value elsewhere), which the
    fused prefill kernel applies itself.  Synchronises (prefill only)."""
    if mask is None:
        return Sq == 1
    m = mask[..., :S]
    if m.shape[-2] != Sq or m.shape[-1] != S:
        return False
    allowed = torch.arange(S, device=m.device)[None, :] <= (
        torch.arange(Sq, device=m.device)[:, None] + (S - Sq))
    blocked = m <= torch.finfo(m.dtype).min / 2 if m.dtype.is_floating_point else m == 0
    ok = torch.where(allowed, m == 0, blocked)
    return bool(ok.all())


def _kernel_mask(mask, length: int) -> bool:
    """True when the decode kernel applies ``mask`` exactly: none, one column
    (what HF builds for this cache during decode: one value added to every
    score, which the softmax cancels) or a one-token cache.  A mask with a
    column per cached token may be nonzero anywhere (padding), so that step
    takes the reference's math over the dequantized cache instead; deciding
    this needs no look at the mask's values (no host synchronisation)."""
    return mask is None or mask.shape[-1] == 1 or length <= 1


def _blockwise_attention(module, query, st: _BlockStore, attention_mask, scaling, dropout):
    """Attention over a block-wise K layer: decode steps with ``kernels.kblock_decode``;
    multi-token steps on the dequantized cache with the reference's math."""
    B, Hq, Sq, D = query.shape
    L = st.length
    q = _fake_quant(query, Q_DIMS) if Q_DIMS is not None else query
    if Sq == 1 and not (module.training and dropout > 0.0):
        if attention_mask is not None and attention_mask.shape[-1] not in (1, L):
            raise ValueError("quantized_attention_forward: unexpected decode mask width")
        if _kernel_mask(attention_mask, L):
            if st.lens is not None:  # length on the device: replayable in a CUDA graph
                return kernels.kblock_decode(q[:, :, 0, :], st.c, L, sm_scale=scaling,
                                             seq_len=st.lens, s_plan=L).unsqueeze(1)
            return kernels.kblock_decode(q[:, :, 0, :], st.c, L, sm_scale=scaling).unsqueeze(1)
    key = kernels.kblock_dequant(st.c, L, query.dtype)
    value = kernels.dequant(st.c["v"][:, :, :L], st.c["v_scale"][:, :, :L].unsqueeze(-1),
                            query.dtype, per_channel=False)
    return _reference_math(module, q, key, value, attention_mask, scaling, dropout)


def quantized_attention_forward(module, query, key, value, attention_mask, scaling=None,
                                dropout=0.0, **kwargs):
    """Replacement for Qwen3's ``eager_attention_forward`` (tests/qwen_kvcache_full.py:95-113).

    Returns ``(attn_output [B, Sq, Hq, D], None)``.
    """
    if scaling is None:
        scaling = module.head_dim ** -0.5
    kb = getattr(key, "_hq_kblock", None)
    if kb is not None:
        return _blockwise_attention(module, query, kb, attention_mask, scaling, dropout), None
    st = getattr(key, "_hq_store", None)
    B, Hq, Sq, D = query.shape
    if st is not None and Sq == 1 and not (module.training and dropout > 0.0):
        if attention_mask is not None and attention_mask.shape[-1] not in (1, st.length):
            raise ValueError("quantized_attention_forward: unexpected decode mask width")
    if (st is not None and Sq == 1 and not (module.training and dropout > 0.0)
            and _kernel_mask(attention_mask, st.length)):
        q_quant = Q_DIMS is not None and tuple(Q_DIMS) == (3,)
        q = query if (Q_DIMS is None or q_quant) else _fake_quant(query, Q_DIMS)
        out = _decode_direct(st, q, module.num_key_value_groups, scaling, q_quant)
        if out is None:
            st.flush()
            out = torch.empty((B, 1, Hq, D), dtype=query.dtype, device=query.device)
            if st.lens is not None:  # capacity buffers, length on the device
                kernels.int8_decode_attn(q[:, :, 0, :], st.k, st.k_sc, st.v, st.v_sc,
                                         module.num_key_value_groups, sm_scale=scaling,
                                         q_quant=q_quant, out=out[:, 0], seq_len=st.lens,
                                         s_plan=st.length)
            else:
                k, v, k_sc, v_sc = st.codes()
                kernels.int8_decode_attn(q[:, :, 0, :], k, k_sc, v, v_sc,
                                         module.num_key_value_groups, sm_scale=scaling,
                                         q_quant=q_quant, out=out[:, 0])
        return out, None
    if st is not None:
        k, v, k_sc, v_sc = st.codes()
        if (st.prefill and Sq > 1 and Q_DIMS in (None, (3,))
                and query.dtype in (torch.bfloat16, torch.float16)
                and D == 128 and not (module.training and dropout > 0.0)
                and _is_causal(attention_mask, Sq, st.length)):
            out = kernels.int8_prefill_attn(
                query, k, k_sc, v, v_sc, module.num_key_value_groups, sm_scale=scaling,
                q_quant=Q_DIMS is not None,
                status_into=st.status.quant_word(query.device) if st.status is not None else None)
            return out, None
        key = kernels.dequant(k, k_sc, query.dtype, per_channel=True)
        value = kernels.dequant(v, v_sc, query.dtype, per_channel=False)
    q = _fake_quant(query, Q_DIMS) if Q_DIMS is not None else query
    return _reference_math(module, q, key, value, attention_mask, scaling, dropout), None


# ---------------------------------------------------------------- installation
_saved = {}


def install(module=None) -> None:
    """Install ``quantized_attention_forward`` as Qwen3's eager attention
    (the reference assigns the module global, tests/qwen_kvcache_full.py:161)."""
    if module is None:
        import transformers.models.qwen3.modeling_qwen3 as module
    if module.eager_attention_forward is not quantized_attention_forward:
        _saved[module.__name__] = module.eager_attention_forward
        module.eager_attention_forward = quantized_attention_forward


def uninstall(module=None) -> None:
    """Restore the original eager attention (tests/qwen_kvcache_full.py:186)."""
    if module is None:
        import transformers.models.qwen3.modeling_qwen3 as module
    orig = _saved.pop(module.__name__, None)
    if orig is not None:
        module.eager_attention_forward = orig


_qwen3 = None


def is_installed(module=None) -> bool:
    global _qwen3
    if module is None:
        if _qwen3 is None:
            import transformers.models.qwen3.modeling_qwen3 as mod
            _qwen3 = mod
        module = _qwen3
    return module.eager_attention_forward is quantized_attention_forward


class installed:
    """Context manager around ``install`` / ``uninstall``."""

    def __init__(self, module=None):
        self.module = module

    def __enter__(self):
        install(self.module)
        return self

    def __exit__(self, *exc):
        uninstall(self.module)
        return False
