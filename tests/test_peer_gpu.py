"""Sequence-sharded decode with the partial exchange inside the decode kernel
(``hq_decode_int8_peer``, ``sharding.PeerShardedDecode``).

One GPU: a world of one rank (the kernel stores its partial into its own
receive buffer, raises and waits for its own flag, merges one partial) must
give exactly the output of ``hq_decode_int8``, eagerly, on repeated calls (the
two buffer halves alternate) and under CUDA graph replay; a world of two
ranks whose second rank never runs must stop waiting, report
HQ_ERR_DEVICE_TIMEOUT in the status word and leave the context usable (the
flag nothing sets is the planted failure; no GPU fault is involved).

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
def test_two_ranks_over_nvlink():
    world = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr=127.0.0.1",
           "--master-port=29533", os.path.join(ROOT, "tests", "mp_peer_decode.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    assert r.stdout.count("PEER OK") == world, r.stdout[-4000:]
