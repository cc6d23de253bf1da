"""Host logic of the multi-GPU paths on CPU ``gloo`` ranks (world size 2).

The kernels need a GPU, so each rank computes its softmax partials with the
oracle (float64 numpy) on its token range; the product's range planning and
its partial exchange (``sharding.gather_partials``) run unchanged, and the
oracle combine of the gathered partials must equal the unsplit attention.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from halftone_quantizedkvcache_b200 import sharding


def test_batch_and_sequence_ranges_partition():
    for B in (1, 5, 8, 64):
        for world in (1, 2, 3, 8):
            spans = [sharding.batch_range(B, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    for S in (1, 63, 64, 65, 32768, 131072, 100000):
        for world in (1, 2, 4, 8):
            spans = [sharding.sequence_range(S, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == S
            for i in range(world - 1):
                assert spans[i][1] == spans[i + 1][0]
                assert spans[i][1] % sharding.TILE == 0 or spans[i][1] == S


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, S, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from oracle import attention as oa
        from oracle import inputs as oin
        from oracle import quant as oq
        c = oin.decode_case(11, 2, 16, 8, S, 128)
        k = oq.dequantize_int8(c["k_i8"], c["k_sc"])
        v = oq.dequantize_int8(c["v_i8"], c["v_sc"])
        sm = 1.0 / np.sqrt(128)
        s0, s1 = sharding.sequence_range(S, world, rank)
        (m, l, o), = oa.split_partials(c["q"], k, v, [(s0, s1)], 2, sm)
        local = torch.from_numpy(np.concatenate([m[..., None], l[..., None], o], axis=-1))
        gathered = sharding.gather_partials(local.to(torch.float64))
        parts = [(g[..., 0].numpy(), g[..., 1].numpy(), g[..., 2:].numpy()) for g in gathered]
        got = oa.lse_combine(parts)
        ref = oa.decode_dense(c["q"], k, v, 2, sm, acc="f64")
        result[rank] = float(np.max(np.abs(got - ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("S", [100, 4096 + 17])
def test_sequence_sharded_exchange_gloo(S):
    world = 2
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, S, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert len(result) == world
    assert max(result.values()) < 1e-10


def _write_rank_main(rank, world, port, S, result):
    """One rank of a sequence-sharded K bulk write: the product's
    ``sequence_sharded_quant_k`` (range, all_reduce(MAX), scale, codes) with its three
    steps done by the oracle on the CPU."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from oracle import inputs as oin
        from oracle import quant as oq
        x = oin.outlier_k(np.random.default_rng(5), 2, 4, S, 64)
        s0, s1 = sharding.sequence_range(S, world, rank)
        shard = torch.from_numpy(np.ascontiguousarray(x[:, :, s0:s1]))

        def absmax(t):  # column maxima of this rank's tokens (zeros for no tokens)
            a = np.abs(t.numpy()).max(axis=2, keepdims=True) if t.shape[2] else np.zeros(
                (t.shape[0], t.shape[1], 1, t.shape[3]), np.float32)
            return torch.from_numpy(a.astype(np.float32))

        def scale(a):  # quantize_int8's scale of a maximum
            s = (np.maximum(a.numpy(), np.float32(1e-8)) / np.float32(127)).astype(np.float32)
            return torch.from_numpy(s), None

        def codes(t, s, out=None):
            return torch.from_numpy(oq.quant_k_static(t.numpy(), s.numpy()))
        q, sc = sharding.sequence_sharded_quant_k(shard, column_absmax=absmax,
                                                  scale_from_amax=scale, quant_static=codes)
        ref_q, ref_s = oq.quant_k_perchannel(x)
        result[rank] = (bool(np.array_equal(q.numpy(), ref_q[:, :, s0:s1])),
                        bool(np.array_equal(sc.numpy(), ref_s)), s1 - s0)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("S", [50, 1000])
def test_sequence_sharded_k_write_gloo(S):
    """Codes and scales of a K bulk write split over two ranks equal the unsharded
    per-channel quantization (S=50: the second rank holds no tokens)."""
    world = 2
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_write_rank_main, args=(r, world, port, S, result))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert len(result) == world
    assert all(r[0] and r[1] for r in result.values()), dict(result)
    assert sum(r[2] for r in result.values()) == S
