"""Multi-GPU sharding of the decode path (one process per GPU, torch.distributed).

Two partitions, as the workloads define them:

* **batch / kv-head sharding** (batched serving decode, bulk quantize-on-write):
  sequences are independent, so each rank owns a contiguous batch range and
  runs the single-GPU kernels on it; there is no collective on the data path.
* **sequence sharding** (one very long sequence): each rank owns a contiguous
  token range of the int8 cache (a multiple of the 64-token kernel tile) plus
  the replicated per-channel K scales, computes the float32 (m, l, o) softmax
  partials of its range with the split-KV kernel, exchanges them with one
  ``all_gather`` (``B * Hq * (D + 2) * 4`` bytes per rank, into local memory)
  and merges them on the device with the log-sum-exp combine kernel.

The reference is single-GPU (no collectives anywhere); the partial format and
the combine follow the flash-decoding rule its roadmap names (README.md:137).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

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
