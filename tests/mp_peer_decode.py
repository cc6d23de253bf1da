"""Worker of tests/test_peer_gpu.py::test_two_ranks_over_nvlink (torchrun, one
rank per GPU; not collected by pytest).

Every rank builds the same seeded sequences, quantizes them with the product
kernels, keeps its own token range (``sharding.sequence_range``) and runs
``PeerShardedDecode``; the output of every rank must match the oracle over the
whole sequence (1e-3 absolute, 2^-7 relative: the stored bf16 output) and the
single-GPU kernel over the whole sequence (within one bf16 step).  Covered:
split shards, a rank with an empty shard, repeated calls and CUDA graph replay.
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from halftone_quantizedkvcache_b200 import kernels, sharding  # noqa: E402
from oracle import attention as oa  # noqa: E402
from oracle import inputs as oin  # noqa: E402

CASES = [  # B, Hq, Hkv, S (whole sequence)
    (1, 16, 8, 32768),
    (2, 32, 8, 5000),
    (1, 16, 8, 100),    # the last ranks hold no tokens
    (4, 16, 4, 2048),
]


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    if torch.cuda.device_count() < world:
        raise SystemExit("one GPU per rank is required (the kernels of the ranks wait on each other)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        for B, Hq, Hkv, S in CASES:
            c = oin.decode_case(100 + S, B, Hq, Hkv, S, 128)
            q = torch.from_numpy(c["q"]).to(dev).to(torch.bfloat16)
            k = torch.from_numpy(c["k"]).to(dev).to(torch.bfloat16)
            v = torch.from_numpy(c["v"]).to(dev).to(torch.bfloat16)
            k8, ks = kernels.quant_k_perchannel(k, scale_dtype=torch.float32)
            v8, vs = kernels.quant_v_pertoken(v, scale_dtype=torch.float32)
            full = kernels.int8_decode_attn(q, k8, ks, v8, vs)
            ref = oa.decode_int8(c["q"], k8.cpu().numpy(), ks.cpu().numpy(), v8.cpu().numpy(),
                                 vs.cpu().numpy(), acc="f64")
            s0, s1 = sharding.sequence_range(S, world, rank)
            mk, mv, mvs = (k8[:, :, s0:s1].contiguous(), v8[:, :, s0:s1].contiguous(),
                           vs[:, :, s0:s1].contiguous())
            peer = sharding.PeerShardedDecode(B, Hq, Hkv, dev)
            outs = [peer(q, mk, ks, mv, mvs) for _ in range(3)]
            out = torch.empty_like(full)
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                peer(q, mk, ks, mv, mvs, out=out)   # this stream's workspace, outside capture
                with torch.cuda.graph(g, stream=s):
                    for _ in range(2):
                        peer(q, mk, ks, mv, mvs, out=out)
            torch.cuda.current_stream().wait_stream(s)
            for _ in range(2):
                out.zero_()
                g.replay()
            torch.cuda.synchronize()
            outs.append(out.clone())
            del g
            assert kernels.read_status("decode") == 0, "peer wait timed out"
            with torch.cuda.stream(s):
                assert kernels.read_status("decode") == 0, "peer wait timed out (graph)"
            for o in outs:
                got = o.float().cpu().numpy()
                np.testing.assert_allclose(got, ref, atol=1e-3, rtol=2.0 ** -7,
                                           err_msg=f"rank {rank} case {(B, Hq, Hkv, S)}")
                torch.testing.assert_close(o.float(), full.float(), atol=1e-3, rtol=2.0 ** -7)
            peer.close()
            print(f"rank {rank} case {(B, Hq, Hkv, S)} shard [{s0}, {s1}) ok", flush=True)
        dist.barrier()
        print(f"PEER OK rank {rank}", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
