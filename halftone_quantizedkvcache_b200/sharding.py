"""Multi-GPU sharding of the decode path (one process per GPU, torch.distributed).

Two partitions, as the workloads define them:

* **batch / kv-head sharding** (batched serving decode, bulk quantize-on-write):
  sequences are independent, so each rank owns a contiguous batch range and
  runs the single-GPU kernels on it; there is no collective on the data path.
  A bulk write split along the sequence instead (``sequence_sharded_quant_k``)
  has one exchange: an ``all_reduce(MAX)`` of the K column maxima.
* **sequence sharding** (one very long sequence): each rank owns a contiguous
  token range of the int8 cache (a multiple of the 64-token kernel tile) plus
  the replicated per-channel K scales and computes the float32 (m, l, o)
  softmax partials of its range.  ``PeerShardedDecode`` exchanges them inside
  the decode kernel: the block that finishes a (sequence, kv head) stores its
  partial straight into every rank's receive buffer (CUDA IPC mappings over
  NVLink), raises a flag per rank, waits for the other ranks' flags and
  merges - one launch per layer, no collective library call.
  ``SequenceShardedDecode`` is the library baseline of the same exchange: the
  kernel writes the partials, NCCL ``all_gather`` moves them
  (``B * Hq * (D + 2) * 4`` bytes per rank) and the combine kernel merges.

The reference is single-GPU (no collectives anywhere); the partial format and
the combine follow the flash-decoding rule its roadmap names (README.md:137).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

TILE = 64


def batch_range(B: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous batch slice of ``rank`` (sizes differ by at most one)."""
    base, extra = divmod(B, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def sequence_range(S: int, world: int, rank: int, align: int = TILE) -> tuple[int, int]:
    """Contiguous token range of ``rank``; boundaries are multiples of ``align``
    (the last rank takes the remainder)."""
    units = (S + align - 1) // align
    u0, u1 = batch_range(units, world, rank)
    return min(S, u0 * align), min(S, u1 * align)


def sequence_sharded_quant_k(x_shard: torch.Tensor, *, group=None,
                             scale_dtype: torch.dtype | None = torch.float16,
                             out: torch.Tensor | None = None,
                             column_absmax=None, scale_from_amax=None, quant_static=None):
    """K per channel for a bulk write whose tokens are split over ranks (each rank
    holds ``x_shard [B, H, S_rank, D]``, its ``sequence_range`` of every sequence).

    The per-channel scale is that of the whole sequence, as an unsharded
    ``quant_k_perchannel`` computes it (quantize_int8 with dims (2,),
    reference/page_attention_int8_pytorch.py:23-30): each rank reduces its own
    tokens to column maxima (``hq_column_absmax``), one ``all_reduce(MAX)`` of the
    ``B * H * D`` float32 maxima combines them - the write's only exchange - and
    every rank derives the scale ``RN(max(amax, 1e-8) / 127)``
    (``hq_k_scale_from_amax``) and codes its tokens with the static-scale kernel
    (``hq_quant_k_static``).  The codes and the scale are bit-identical to the
    unsharded quantization's; an empty shard contributes zeros to the maximum.

    Returns ``(codes [B, H, S_rank, D] int8, scale [B, H, 1, D])`` with the scale in
    ``scale_dtype`` (float32 when None).  ``column_absmax`` / ``scale_from_amax`` /
    ``quant_static`` replace the three steps (host-side tests pass CPU versions);
    the defaults are this library's kernels.
    """
    from . import kernels
    column_absmax = column_absmax or kernels.column_absmax
    quant_static = quant_static or kernels.quant_k_static
    if scale_from_amax is None:
        def scale_from_amax(a):
            return kernels.k_scale_from_amax(a, scale_dtype=scale_dtype)
    amax = column_absmax(x_shard)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    s32, s_out = scale_from_amax(amax)
    if x_shard.shape[2] == 0:
        codes = torch.empty(x_shard.shape, dtype=torch.int8, device=x_shard.device)
    else:
        codes = quant_static(x_shard, s32, out=out)
    return codes, (s_out if s_out is not None else s32)


def gather_partials(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather the per-rank partial tensor ``[B, Hq, D+2]`` -> ``[world, B, Hq, D+2]``."""
    world = dist.get_world_size(group)
    flat = torch.empty((world * local.shape[0], *local.shape[1:]), dtype=local.dtype,
                       device=local.device)
    dist.all_gather_into_tensor(flat, local.contiguous(), group=group)
    return flat.view(world, *local.shape)


class SequenceShardedDecode:
    """Decode attention over a cache whose tokens are split across ranks.

    Holds a preallocated partial buffer so a step does one kernel, one
    ``all_gather`` and one combine, all on the current stream.
    """

    def __init__(self, B: int, Hq: int, D: int, device, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.local = torch.empty((B, Hq, D + 2), dtype=torch.float32, device=device)
        self.flat = torch.empty((self.world * B, Hq, D + 2), dtype=torch.float32, device=device)
        self.gathered = self.flat.view(self.world, B, Hq, D + 2)

    def __call__(self, q, k_i8, k_sc, v_i8, v_sc, *, sm_scale=None, q_quant=False, out=None):
        from . import kernels
        kernels.int8_decode_attn(q, k_i8, k_sc, v_i8, v_sc, sm_scale=sm_scale, q_quant=q_quant,
                                 partial_out=self.local)
        dist.all_gather_into_tensor(self.flat, self.local, group=self.group)
        return kernels.decode_combine(self.gathered, out_dtype=q.dtype, out=out)


class PeerShardedDecode:
    """Decode attention over a cache whose tokens are split across ranks, with
    the partial exchange fused into the decode kernel (``hq_decode_int8_peer``).

    The constructor is collective over ``group``: every rank allocates its
    receive buffer, the CUDA IPC handles go round with ``all_gather_object``
    and each rank maps the others' buffers.  One instance serves one
    ``(B, Hq, Hkv)``; every rank must call it the same number of times, in the
    same order (eagerly or by CUDA graph replay).  ``close()`` (collective)
    unmaps and frees the buffers.  The ranks must be on distinct GPUs: the
    kernel of one rank waits for the kernels of the others.
    """

    def __init__(self, B: int, Hq: int, Hkv: int, device, group=None):
        L = _lib.lib()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        if self.world > 8:
            raise ValueError("PeerShardedDecode: at most 8 ranks")
        nbytes = L.hq_peer_buffer_bytes(self.world, B, Hq, Hkv)
        if nbytes == 0:
            raise ValueError(f"PeerShardedDecode: bad shape B={B} Hq={Hq} Hkv={Hkv}")
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        with torch.cuda.device(self.device):
            _lib.check(L.hq_peer_alloc(nbytes, ctypes.byref(own), handle), "hq_peer_alloc")
        self._own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, (str(torch.cuda.get_device_properties(self.device).uuid),
                                         bytes(handle)), group=group)
        if len({h[0] for h in handles}) != self.world:
            L.hq_peer_free(self._own)
            raise RuntimeError("PeerShardedDecode: two ranks share a GPU")
        self._opened = []
        self.buffers = (ctypes.c_void_p * self.world)()
        with torch.cuda.device(self.device):
            for w, (_, h) in enumerate(handles):
                if w == self.rank:
                    self.buffers[w] = self._own
                    continue
                ptr = ctypes.c_void_p()
                _lib.check(L.hq_peer_open(ctypes.create_string_buffer(h, 64), ctypes.byref(ptr)),
                           "hq_peer_open")
                self._opened.append(ptr.value)
                self.buffers[w] = ptr.value
        dist.barrier(group)

    def __call__(self, q, k_i8, k_sc, v_i8, v_sc, *, sm_scale=None, q_quant=False, out=None):
        from . import kernels
        return kernels.int8_decode_attn(q, k_i8, k_sc, v_i8, v_sc, sm_scale=sm_scale,
                                        q_quant=q_quant, out=out,
                                        peers=(self.buffers, self.world, self.rank))

    def close(self) -> None:
        """Collective: unmap the other ranks' buffers, then free this rank's."""
        if self._own is None:
            return
        L = _lib.lib()
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                _lib.check(L.hq_peer_close(ptr), "hq_peer_close")
        self._opened = []
        dist.barrier(self.group)
        with torch.cuda.device(self.device):
            _lib.check(L.hq_peer_free(self._own), "hq_peer_free")
        self._own = None
