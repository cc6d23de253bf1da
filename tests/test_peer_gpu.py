"""Sequence-sharded decode with the partial exchange inside the decode kernel
(``hq_decode_int8_peer``, ``sharding.PeerShardedDecode``).

One GPU: a world of one rank must give exactly the output of
``hq_decode_int8``, eagerly and under CUDA graph replay.  The merge is checked
by playing one rank of a world of 2 or 3 whose other ranks' words are already
in its receive buffer (written beforehand from their partials, with the
epoch of the launch): the launch stores its own words into the other buffers
(checked bit for bit), merges without waiting and must match the oracle over
the whole sequence, identically for every rank played.  A world of two whose
second rank never runs must stop waiting, report HQ_ERR_DEVICE_TIMEOUT in the
status word and leave the context usable (the word nothing writes is the
planted failure; no GPU fault is involved).

Two or more GPUs: ``tests/mp_peer_decode.py`` runs under torchrun, one rank
per GPU, and checks every rank's output against the oracle over the whole
sequence (tolerance of the stored bf16 output: 1e-3 absolute, 2^-7 relative).
"""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200 import _lib, kernels
from oracle import inputs as oin

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _case(seed, B, Hq, Hkv, S):
    c = oin.decode_case(seed, B, Hq, Hkv, max(S, 1), 128)
    c["k_i8"], c["v_i8"], c["v_sc"] = c["k_i8"][:, :, :S], c["v_i8"][:, :, :S], c["v_sc"][:, :, :S]
    t = {k: torch.from_numpy(np.ascontiguousarray(c[k])).cuda()
         for k in ("q", "k_i8", "k_sc", "v_i8", "v_sc")}
    t["q"] = t["q"].to(torch.bfloat16)
    return t


def _alloc(world, B, Hq, Hkv):
    L = _lib.lib()
    n = L.hq_peer_buffer_bytes(world, B, Hq, Hkv)
    ptr, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
    _lib.check(L.hq_peer_alloc(n, ctypes.byref(ptr), handle), "hq_peer_alloc")
    return ptr.value


@pytest.mark.parametrize("B,Hq,Hkv,S", [
    (1, 16, 8, 32768),   # split over the whole GPU, last-block merge
    (2, 32, 8, 5000),    # ragged tail
    (1, 8, 8, 100),      # one split per unit
    (3, 16, 4, 0),       # empty shard: m = -inf, l = 0
    (1, 32, 8, 1),
])
def test_world_of_one_equals_single_gpu(B, Hq, Hkv, S):
    c = _case(7 + S, B, Hq, Hkv, S)
    args = (c["q"], c["k_i8"], c["k_sc"], c["v_i8"], c["v_sc"])
    ref = kernels.int8_decode_attn(*args)
    buf = _alloc(1, B, Hq, Hkv)
    try:
        peers = ((ctypes.c_void_p * 1)(buf), 1, 0)
        for _ in range(3):       # epochs 1..3 use both halves of the buffer
            got = kernels.int8_decode_attn(*args, peers=peers)
            torch.cuda.synchronize()
            assert kernels.read_status("decode") == 0
            if S == 0:
                assert torch.count_nonzero(got) == 0
            assert torch.equal(got, ref)
        out = torch.empty_like(ref)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            kernels.int8_decode_attn(*args, peers=peers, out=out)   # warm-up outside capture
            with torch.cuda.graph(g, stream=s):
                for _ in range(3):
                    kernels.int8_decode_attn(*args, peers=peers, out=out)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(2):
            out.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
        del g
    finally:
        _lib.lib().hq_peer_free(buf)


def _rows(part, epoch):
    """float32 partial [B, Hq, D+2] (m, l, o) -> u64 words [B*Hq, D+4] (m, l, -, -, o),
    value bits low, epoch high."""
    B, Hq, D2 = part.shape
    rows = torch.zeros((B * Hq, D2 + 2), dtype=torch.float32, device=part.device)
    rows[:, 0:2] = part.reshape(B * Hq, D2)[:, 0:2]
    rows[:, 4:] = part.reshape(B * Hq, D2)[:, 2:]
    return (rows.view(torch.int32).to(torch.int64) & 0xFFFFFFFF) | (int(epoch) << 32)


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("B,Hq,Hkv,S", [(1, 16, 8, 32768), (2, 32, 8, 5000), (1, 16, 4, 100)])
def test_rank_merge_with_prewritten_words(world, B, Hq, Hkv, S):
    from halftone_quantizedkvcache_b200 import sharding
    from oracle import attention as oa
    c = _case(40 + S, B, Hq, Hkv, S)
    full = kernels.int8_decode_attn(c["q"], c["k_i8"], c["k_sc"], c["v_i8"], c["v_sc"])
    ref = oa.decode_int8(c["q"].float().cpu().numpy(), c["k_i8"].cpu().numpy(),
                         c["k_sc"].cpu().numpy(), c["v_i8"].cpu().numpy(),
                         c["v_sc"].cpu().numpy(), acc="f64")
    shards, parts = [], []
    for r in range(world):
        s0, s1 = sharding.sequence_range(S, world, r)
        sh = (c["k_i8"][:, :, s0:s1].contiguous(), c["v_i8"][:, :, s0:s1].contiguous(),
              c["v_sc"][:, :, s0:s1].contiguous())
        part = torch.empty((B, Hq, 130), dtype=torch.float32, device="cuda")
        kernels.int8_decode_attn(c["q"], sh[0], c["k_sc"], sh[1], sh[2], partial_out=part)
        shards.append(sh)
        parts.append(part)
    L = _lib.lib()
    nbytes = L.hq_peer_buffer_bytes(world, B, Hq, Hkv)
    poff = (4 * B * Hkv + 255) // 256 * 256
    outs = []
    for me in range(world):
        bufs = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(world)]
        words = [b[poff:].view(torch.int64).view(2, world, B * Hq, 132) for b in bufs]
        ptrs = (ctypes.c_void_p * world)(*[b.data_ptr() for b in bufs])
        for epoch in (1, 2, 3):
            for w in range(world):
                if w != me:
                    words[me][epoch & 1, w] = _rows(parts[w], epoch)
            k8, v8, vs = shards[me]
            out = kernels.int8_decode_attn(c["q"], k8, c["k_sc"], v8, vs,
                                           peers=(ptrs, world, me))
            torch.cuda.synchronize()
            assert kernels.read_status("decode") == 0
            gen = bufs[me][:4 * B * Hkv].view(torch.int32)
            assert torch.all(gen == epoch)
            for w in range(world):
                if w != me:   # this rank's words, bit for bit, in every other buffer
                    assert torch.equal(words[w][epoch & 1, me][:, [0, 1] + list(range(4, 132))],
                                       _rows(parts[me], epoch)[:, [0, 1] + list(range(4, 132))])
            np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=1e-3, rtol=2.0 ** -7)
            torch.testing.assert_close(out.float(), full.float(), atol=1e-3, rtol=2.0 ** -7)
        outs.append(out)
    for o in outs[1:]:
        assert torch.equal(o, outs[0])   # every rank merges in rank order: same output


def test_absent_rank_times_out_and_context_survives():
    B, Hq, Hkv, S = 1, 16, 8, 4096
    c = _case(3, B, Hq, Hkv, S)
    args = (c["q"], c["k_i8"], c["k_sc"], c["v_i8"], c["v_sc"])
    ref = kernels.int8_decode_attn(*args)
    L = _lib.lib()
    mine, other = _alloc(2, B, Hq, Hkv), _alloc(2, B, Hq, Hkv)
    wsb = L.hq_decode_workspace_bytes(B, Hq, Hkv, S, 128)
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    out = torch.full_like(ref, 7.0)
    q = c["q"]
    st3 = lambda t: _lib.strides(t.stride(), 3)  # noqa: E731
    try:
        rc = L.hq_decode_int8_peer(
            q.data_ptr(), _lib.DTYPE_BF16, st3(q), c["k_i8"].data_ptr(), c["v_i8"].data_ptr(),
            _lib.strides(c["k_i8"].stride()[:3], 3), c["k_sc"].data_ptr(), c["v_sc"].data_ptr(),
            _lib.DTYPE_F32, _lib.strides((c["k_sc"].stride(0), c["k_sc"].stride(1),
                                          c["k_sc"].stride(3)), 3),
            _lib.strides(c["v_sc"].stride()[:3], 3), B, Hq, Hkv, S, 128, 128 ** -0.5, 0,
            out.data_ptr(), st3(out), ws.data_ptr(), wsb, (ctypes.c_void_p * 2)(mine, other),
            2, 0, None)
        assert rc == 0
        torch.cuda.synchronize()
        assert L.hq_read_status(ws.data_ptr(), None) == _lib.ERR_DEVICE_TIMEOUT
        assert torch.all(out == 7.0)           # no output after giving up
        again = kernels.int8_decode_attn(*args)  # the context is still usable
        torch.cuda.synchronize()
        assert torch.equal(again, ref)
    finally:
        L.hq_peer_free(mine)
        L.hq_peer_free(other)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_every_gpu_a_rank_over_nvlink():
    """One rank per visible GPU (up to 8), each decoding its share of one sequence and
    exchanging (m, l, o) inside the decode kernel over NVLink."""
    world = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr=127.0.0.1",
           "--master-port=29533", os.path.join(ROOT, "tests", "mp_peer_decode.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    assert r.stdout.count("PEER OK") == world, r.stdout[-4000:]
