"""Sequence-sharded K bulk write on the GPU (``hq_column_absmax``,
``hq_k_scale_from_amax``, ``hq_quant_k_static``): ranks are emulated on one GPU by
splitting the tokens with ``sharding.sequence_range`` and combining the per-rank
column maxima with an elementwise maximum (what ``all_reduce(MAX)`` computes).
The codes and scales must equal the unsharded ``quant_k_perchannel``'s bit for bit.
"""
import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200 import kernels, sharding
from oracle import inputs as oin

pytestmark = pytest.mark.gpu
TDT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


@pytest.mark.parametrize("dt,D,S", [("bf16", 128, 4096 + 37), ("f16", 64, 700), ("f32", 256, 300),
                                    ("bf16", 128, 50)])
@pytest.mark.parametrize("world", [2, 3])
def test_sharded_write_equals_unsharded(dt, D, S, world):
    x = torch.from_numpy(oin.outlier_k(np.random.default_rng(S + D), 2, 4, S, D)).to(TDT[dt]).cuda()
    ref_q, ref_s16 = kernels.quant_k_perchannel(x)
    _, ref_s32 = kernels.quant_k_perchannel(x, scale_dtype=torch.float32)
    spans = [sharding.sequence_range(S, world, r) for r in range(world)]
    maxima = [kernels.column_absmax(x[:, :, s0:s1]) for s0, s1 in spans]
    amax = maxima[0]
    for m in maxima[1:]:
        amax = torch.maximum(amax, m)
    assert torch.equal(amax, x.float().abs().amax(dim=2, keepdim=True))
    s32, s16 = kernels.k_scale_from_amax(amax)
    assert torch.equal(s32, ref_s32) and torch.equal(s16, ref_s16)
    for s0, s1 in spans:
        if s1 > s0:
            q = kernels.quant_k_static(x[:, :, s0:s1], s32)
            assert torch.equal(q, ref_q[:, :, s0:s1]), (s0, s1)


def test_single_rank_helper_and_empty_shard():
    x = torch.from_numpy(oin.outlier_k(np.random.default_rng(3), 1, 8, 513, 128)).to(torch.bfloat16).cuda()
    q, s = sharding.sequence_sharded_quant_k(x)  # no process group: the whole sequence
    ref_q, ref_s = kernels.quant_k_perchannel(x)
    assert torch.equal(q, ref_q) and torch.equal(s, ref_s)
    empty = kernels.column_absmax(x[:, :, :0])
    assert empty.shape == (1, 8, 1, 128) and not bool(empty.any())
