#!/usr/bin/env python
"""Headline benchmark: int8 split-KV decode attention at S=32K, plus quantize-on-write.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

Workload (decode-attention length sweep at S = 32768, B=1, Hq=16, Hkv=8, D=128):
bf16 q, int8 K/V with float32 scales, codes made by the product's own
quantize-on-write kernels from K ~ N(0,1) with 4 outlier channels per head x20
and V ~ N(0,1) (synthetic, seeded).  A step decodes one token through 28
layers, each with its own cache (28 x 68 MB = 1.9 GB > L2, read round-robin,
so no layer's cache is still in L2 when it is read again); the 28 launches are
one CUDA graph.  At N > 1 GPUs the headline is batch-sharded (weak scaling):
every rank decodes its own sequence's 28 layers with no collective on the data
path.  The ``seq_sharded`` extra at N > 1 is the case with a real exchange: one
sequence of N x 32768 tokens split across the ranks, the softmax partials
exchanged inside the decode kernel over peer memory (and, for comparison, with
an NCCL all_gather plus a combine kernel).

metric / value: algorithmic HBM GB/s of the decode kernel (K+V codes, scales,
q and output bytes) over the whole job; ``us_per_layer`` and the fraction of
the measured HBM peak ride along.  ``e2e`` is the same metric through the
public API (``QuantizedKVCache.update`` + ``quantized_attention_forward``)
with each step's q / new K / new V copied from pinned host memory and the
outputs read back.  The extra keys report the int8 / bf16-twin speedup, the S
sweep and the bulk quantize-on-write GB/s (B=8, Hkv=8, S=32768, bf16).

``cpu_baseline`` (N = 1) and ``--impl reference`` time the reference's CPU
PyTorch path on the host cores, all threads: its decode ops
(``dequantize_int8`` + ``page_attention_reference``, restated in
``oracle/torch_cpu.py``) on the same workload and config as the GPU arm, its
``QuantizedKVCache.update`` for bulk writes and appends (config 4, batch
scaled down), and its whole Qwen3 path (config 1) per token.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, HQ, HKV, D, S_HEAD, LAYERS = 1, 16, 8, 128, 32768, 28
METRIC = "int8 decode-attn HBM GB/s at S=32K (B=1, Hq=16, Hkv=8, D=128)"
FALLBACK_HBM = 6650.0
L2_BYTES = 126 * 2 ** 20


def decode_bytes(b, hq, hkv, s, d, kv_bytes=1, scale_bytes=4):
    """Algorithmic bytes of one decode launch: K+V, scales, q in and out (bf16)."""
    kv = 2 * b * hkv * s * d * kv_bytes
    sc = (b * hkv * s * scale_bytes + b * hkv * d * scale_bytes) if kv_bytes == 1 else 0
    return kv + sc + 2 * b * hq * d * 2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true", help="skip sweep / twin / quant extras")
    ap.add_argument("--no-e2e", action="store_true", help="skip the public-API end-to-end leg")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layer caches per step (profiling runs use a few; default 28)")
    ap.add_argument("--only", choices=["all", "decode", "twin", "quant", "prefill", "kstatic", "kblock"],
                    default="all",
                    help="profiling: run one kernel family on a small case and exit")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


def profile_traffic():
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "decode_int8_s32k_ncu.txt")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1]))
    except OSError:
        pass
    return None


# ---------------------------------------------------------------- clocks
class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during a timed region."""

    Q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        import torch
        try:
            self.index = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:
            self.index = str(device_index)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()
        return False

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = sorted(sm)[len(sm) // 4:] or sm   # drop the idle head of the window
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- workload
def make_layer_caches(torch, kernels, n_layers, S, device, gen, kv="int8"):
    """n_layers caches [B, Hkv, S, D]: int8 codes + fp32 scales (made by the
    product's quantizers) or bf16 K/V for the twin."""
    caches = []
    for _ in range(n_layers):
        k = torch.randn((B, HKV, S, D), generator=gen, device=device)
        ch = torch.stack([torch.randperm(D, generator=gen, device=device)[:4] for _ in range(B * HKV)])
        gain = torch.ones((B * HKV, D), device=device).scatter_(1, ch, 20.0).view(B, HKV, 1, D)
        k = (k * gain).to(torch.bfloat16)
        v = torch.randn((B, HKV, S, D), generator=gen, device=device).to(torch.bfloat16)
        if kv == "int8":
            k8, ks = kernels.quant_k_perchannel(k, scale_dtype=torch.float32)
            v8, vs = kernels.quant_v_pertoken(v, scale_dtype=torch.float32)
            caches.append((k8, ks, v8, vs))
        else:
            caches.append((k, v))
        del k, v
    return caches


def time_graph(torch, fn, steps, warmup, stream, clocks_index=None, label=None, barrier=None):
    """Capture fn() in a CUDA graph, replay warmup + steps; returns (ms/step, clocks).
    ``label`` names an NVTX range around the timed replays (for ncu --nvtx-include);
    ``barrier`` (multi-rank runs) is called after a synchronize on both sides of
    the timed replays."""
    fn()  # first call outside capture: kernel attributes, workspaces
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if barrier:
        barrier()
        torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = Clocks(clocks_index) if clocks_index is not None else None
    if clk:
        clk.__enter__()
    if label:
        torch.cuda.nvtx.range_push(label)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(steps):
            g.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    if barrier:
        barrier()
    if label:
        torch.cuda.nvtx.range_pop()
    if clk:
        clk.__exit__()
    del g
    return ev0.elapsed_time(ev1) / steps, (clk.summary() if clk else None)


# ---------------------------------------------------------------- CPU baseline
def _cpu_threads():
    import torch
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    return cores


def cpu_decode(seconds=10.0, max_layers=None):
    """The reference's CPU PyTorch decode path (``oracle/torch_cpu.py``:
    ``dequantize_int8`` of K and V, then ``page_attention_reference``) on all
    host cores, over S=32768 layers of the headline workload (B=1, Hq=16,
    Hkv=8, D=128, int8 K/V + fp32 scales, float32 q as in the reference's CPU
    chain), one layer after another until ``seconds`` pass.  Returns (GB/s of
    the algorithmic decode bytes, cores, layers, seconds)."""
    import torch

    from oracle import inputs as oin
    from oracle import torch_cpu
    cores = _cpu_threads()
    c = oin.decode_case(0, 1, HQ, HKV, S_HEAD, D, kv_dtype="bf16", q_dtype="bf16")
    t = {k: torch.from_numpy(c[k][0].copy()) for k in ("k_i8", "k_sc", "v_i8", "v_sc")}
    q = torch.from_numpy(c["q"][0].copy())[:, None, :].float()
    torch_cpu.decode_layer(q, t["k_i8"], t["k_sc"], t["v_i8"], t["v_sc"])  # warm-up
    layers, t0 = 0, time.perf_counter()
    while True:
        torch_cpu.decode_layer(q, t["k_i8"], t["k_sc"], t["v_i8"], t["v_sc"])
        layers += 1
        el = time.perf_counter() - t0
        if el >= seconds or (max_layers and layers >= max_layers):
            break
    return layers * decode_bytes(B, HQ, HKV, S_HEAD, D) / el / 1e9, cores, layers, el


def cpu_quant_write(n_appends=8):
    """Config 4 through the reference's ``QuantizedKVCache.update`` on the host
    (``oracle.hf_reference.OracleQuantizedKVCache``, its torch restatement):
    one bulk write of fresh bf16 K/V [1, 8, 32768, 128] (batch 1 of the
    config's 8; K with 4 outlier channels per head x20) and ``n_appends``
    single-token appends (of the config's 1024).  Each call also returns the
    whole cache dequantized, as the reference does."""
    import torch

    from oracle.hf_reference import OracleQuantizedKVCache
    cores = _cpu_threads()
    g = torch.Generator().manual_seed(0)
    Bc, H, Sq = 1, 8, 32768
    gain = torch.ones((H, D))
    for h in range(H):
        gain[h, torch.randperm(D, generator=g)[:4]] = 20.0
    k = (torch.randn((Bc, H, Sq, D), generator=g) * gain[None, :, None, :]).bfloat16()
    v = torch.randn((Bc, H, Sq, D), generator=g).bfloat16()
    cache = OracleQuantizedKVCache()
    t0 = time.perf_counter()
    cache.update(k, v, 0)
    t_bulk = time.perf_counter() - t0
    kn, vn = k[:, :, :1].clone(), v[:, :, :1].clone()
    t0 = time.perf_counter()
    for _ in range(n_appends):
        cache.update(kn, vn, 0)
    t_app = (time.perf_counter() - t0) / n_appends
    n = Bc * H * Sq * D
    nbytes = (3 * n + Bc * H * D * 4) + (3 * n + Bc * H * Sq * 4)   # K and V, as the GPU line
    return {"bulk_gbs": round(nbytes / t_bulk / 1e9, 3), "bulk_s": round(t_bulk, 3),
            "append_us": round(t_app * 1e6, 1), "cores": cores, "kind": "port",
            "sample": f"QuantizedKVCache.update restated in torch on {cores} threads: bulk write of "
                      f"K and V [{Bc},{H},{Sq},{D}] bf16 (batch {Bc} of 8), then {n_appends} "
                      f"single-token appends (of 1024) at S~{Sq}"}


def cpu_model_step(n0=512, budget_s=10.0):
    """Config 1 on the host: the Qwen3-0.6B architecture (random init, bf16) through
    HF transformers with the reference's cache and patched attention (their torch
    restatements in ``oracle.hf_reference``): prefill ``n0`` tokens, then decode
    steps until ``budget_s`` pass (at least one).  Per-token time."""
    import torch
    from transformers import Qwen3ForCausalLM

    from oracle.hf_reference import (OracleQuantizedKVCache, oracle_attention_forward,
                                     patched_attention, qwen3_config)
    cores = _cpu_threads()
    cfg = qwen3_config(num_layers=LAYERS)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
    ids = torch.randint(0, cfg.vocab_size, (1, n0 + 64), generator=torch.Generator().manual_seed(1))
    with torch.no_grad(), patched_attention(oracle_attention_forward):
        cache = OracleQuantizedKVCache()
        t0 = time.perf_counter()
        model(ids[:, :n0], past_key_values=cache, use_cache=True)
        t_pre = time.perf_counter() - t0
        steps, t0 = 0, time.perf_counter()
        while steps < 64:
            model(ids[:, n0 + steps:n0 + steps + 1], past_key_values=cache, use_cache=True)
            steps += 1
            if time.perf_counter() - t0 >= budget_s:
                break
        t_dec = (time.perf_counter() - t0) / steps
    del model
    return {"prefill_s": round(t_pre, 3), "ms_per_token": round(t_dec * 1e3, 2), "cores": cores,
            "kind": "port",
            "sample": f"Qwen3-0.6B architecture (random init, bf16, {LAYERS} layers) through HF "
                      f"transformers with the reference's QuantizedKVCache and patched attention "
                      f"(torch restatements) on {cores} threads: prefill {n0} tokens, then "
                      f"{steps} decode step(s)"}


def arm_config(nl, world, per_layer):
    """The workload both arms report on (the reference arm samples it on the CPU)."""
    return {"workload": f"decode attention over {nl} layer caches, S={S_HEAD} per "
                        f"rank, B={B}, Hq={HQ}, Hkv={HKV}, D={D}, bf16 q, int8 K/V, "
                        "fp32 scales",
            "l2": f"inputs larger than L2: {nl} caches x {per_layer / 1e6:.1f} MB read round-robin",
            "parallelism": (f"batch-sharded x{world}: one sequence per GPU, no collective"
                            if world > 1 else "single GPU"),
            "graph": f"{nl} launches per step in one CUDA graph"}


# ---------------------------------------------------------------- reference arm
def reference_arm(args):
    """The reference's CPU PyTorch decode path on the host cores (rank 0 only),
    on the GPU arm's workload: each step decodes one layer (a bounded sample of
    the 28-layer step; the metric is per-layer bandwidth, so the sample does not
    change it), whole run capped at ~150 s."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    per = []
    cores = layers = 0
    for i in range(args.warmup + args.steps):
        gbs, cores, layers, el = cpu_decode(seconds=0.0, max_layers=1)
        if i >= args.warmup:
            per.append(el)
        if sum(per) > 150:   # keep the whole run within a few minutes
            break
    t = sum(per) / len(per)
    per_layer = decode_bytes(B, HQ, HKV, S_HEAD, D)
    value = per_layer / t / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": len(per), "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": arm_config(args.layers, args.gpus, per_layer),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"one layer of S={S_HEAD} per step (of the {args.layers}-layer "
                                   "GPU step): the reference's dequantize_int8 + "
                                   "page_attention_reference torch ops (oracle/torch_cpu.py) on "
                                   f"{cores} threads"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_seq_sharded(torch, dist, sharding, kernels, caches, q, out, sm_scale, device, stream,
                    world, args):
    """One long sequence split across the ranks (S_HEAD tokens each): the
    exchange fused into the decode kernel over peer memory, and the library
    baseline (partials, NCCL all_gather, combine kernel), both per layer."""
    nl = len(caches)
    res = {"workload": f"one sequence of S={S_HEAD * world} split across {world} ranks "
                       f"({S_HEAD} tokens each), B={B}, Hq={HQ}, Hkv={HKV}, {nl} layers"}
    gbs = lambda ms: round(world * nl * decode_bytes(B, HQ, HKV, S_HEAD, D) / (ms * 1e-3) / 1e9, 1)  # noqa: E731

    def timed(fn, label):
        with torch.cuda.stream(stream):
            ms, _ = time_graph(torch, fn, min(args.steps, 100), min(args.warmup, 5), stream,
                               label=label, barrier=dist.barrier)
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    peer = sharding.PeerShardedDecode(B, HQ, HKV, device)

    def fused_step():
        for l, (k8, ks, v8, vs) in enumerate(caches):
            peer(q[l], k8, ks, v8, vs, sm_scale=sm_scale, out=out[l])

    ms = timed(fused_step, "seq_sharded_fused_step")
    with torch.cuda.stream(stream):
        st = kernels.read_status("decode")
    peer.close()
    res["fused"] = {"us_per_layer": round(ms * 1e3 / nl, 3), "gbs": gbs(ms),
                    "device_status": st,
                    "exchange": "inside the decode kernel: each rank's last block per (b, kv "
                                "head) stores its (m, l, o) into every rank's buffer over "
                                "NVLink, release flags, bounded acquire wait, merge"}
    seq = sharding.SequenceShardedDecode(B, HQ, D, device)

    def nccl_step():
        for l, (k8, ks, v8, vs) in enumerate(caches):
            seq(q[l], k8, ks, v8, vs, sm_scale=sm_scale, out=out[l])

    ms = timed(nccl_step, "seq_sharded_nccl_step")
    res["nccl"] = {"us_per_layer": round(ms * 1e3 / nl, 3), "gbs": gbs(ms),
                   "exchange": "per layer: split kernel writes (m, l, o) partials, NCCL "
                               "all_gather, combine kernel"}
    return res


# ---------------------------------------------------------------- our arm
def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=120))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from halftone_quantizedkvcache_b200 import kernels, sharding
    from halftone_quantizedkvcache_b200.integration import QuantizedKVCache
    from halftone_quantizedkvcache_b200.integration.quantized_attention import (
        quantized_attention_forward)

    peak, peak_kind = load_peaks()
    gen = torch.Generator(device=device).manual_seed(1234 + rank)
    stream = torch.cuda.Stream(device)
    nl = args.layers
    if args.only != "all":
        return profile_only(args, torch, kernels, device, gen, stream)
    caches = make_layer_caches(torch, kernels, nl, S_HEAD, device, gen)
    q = torch.randn((nl, B, HQ, D), generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty((nl, B, HQ, D), dtype=torch.bfloat16, device=device)
    sm_scale = 1.0 / math.sqrt(D)
    # One sequence per GPU (batch sharding): every rank decodes its own caches,
    # no collective on the data path.  The sequence-sharded mode (one long
    # sequence split across ranks, partials exchanged) is measured separately.
    def step():
        for l, (k8, ks, v8, vs) in enumerate(caches):
            kernels.int8_decode_attn(q[l], k8, ks, v8, vs, HQ // HKV, sm_scale=sm_scale,
                                     out=out[l])

    with torch.cuda.stream(stream):
        ms, clocks = time_graph(torch, step, args.steps, args.warmup, stream,
                                clocks_index=torch.cuda.current_device() if rank == 0 else None,
                                label="decode_step", barrier=dist.barrier if world > 1 else None)
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    batched = None
    if not args.no_extras:
        batched = run_batched(torch, kernels, device, stream, world, dist, peak)

    seq_sharded = None
    if world > 1 and not args.no_extras:
        seq_sharded = run_seq_sharded(torch, dist, sharding, kernels, caches, q, out, sm_scale,
                                      device, stream, world, args)
    per_layer = decode_bytes(B, HQ, HKV, S_HEAD, D)
    value = world * nl * per_layer / (ms * 1e-3) / 1e9
    us_layer = ms * 1e3 / nl
    achieved = per_layer / (us_layer * 1e-6) / 1e9

    # ---- e2e through the public API (cache + patched attention), host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(torch, kernels, QuantizedKVCache, quantized_attention_forward, caches,
                      device, stream, min(args.steps, 100), min(args.warmup, 5), world, dist)

    extras = {}
    if world == 1 and not args.no_extras:
        extras = run_extras(torch, kernels, device, gen, stream, us_layer, peak)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": arm_config(nl, world, per_layer),
            "us_per_layer": round(us_layer, 3),
            "frac_of_peak": round(achieved / peak, 4),
            "frac_of_8tbs": round(achieved / 8000.0, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": profile_traffic(), "peak_kind": peak_kind,
                         "kernel": "hq::dec::mmak::decode_mma_kernel<2, f32 scales, bf16 q>",
                         "algorithmic_bytes_per_launch": per_layer},
            "clocks": clocks or {},
            "e2e": e2e,
            "gpu_launches": args.steps * nl,
        }
        if batched:
            line["batched_decode"] = batched
        if seq_sharded:
            line["seq_sharded"] = seq_sharded
        line.update(extras)
        if world == 1 and not args.no_cpu:
            gbs, cores, layers, el = cpu_decode(seconds=10.0)
            line["cpu_baseline"] = {
                "value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                "sample": f"{layers} layers of S={S_HEAD} decode in {el:.1f} s: the reference's "
                          "dequantize_int8 + page_attention_reference torch ops "
                          f"(oracle/torch_cpu.py) on {cores} threads"}
            if not args.no_extras:
                line["cpu_baseline"]["quant_write"] = cpu_quant_write()
                line["cpu_baseline"]["model_decode_step"] = cpu_model_step()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


class _Attn:
    """The attributes ``quantized_attention_forward`` reads from Qwen3Attention."""

    def __init__(self, n_rep, head_dim):
        self.num_key_value_groups = n_rep
        self.head_dim = head_dim
        self.training = False


def run_e2e(torch, kernels, QuantizedKVCache, attn_fwd, caches, device, stream, steps, warmup,
            world, dist):
    """Public-API decode: per step, per layer ``cache.update`` (append one token)
    and ``quantized_attention_forward`` (split-KV decode); inputs copied from
    pinned host memory, outputs copied back, inside the timed region.  With
    several ranks every rank runs its own sequence (batch sharding).

    The cache keeps its lengths on the device (``device_lengths=True``), so the
    whole step - host-to-device copy, 28 x (update + attention), device-to-host
    copy - is captured once as a CUDA graph and replayed per token, the way a
    serving loop runs it; the same calls made eagerly are timed beside it."""
    import transformers.models.qwen3.modeling_qwen3 as qwen3_mod  # noqa: F401
    from halftone_quantizedkvcache_b200.integration import quantized_attention as qa
    module = _Attn(HQ // HKV, D)
    nl = len(caches)
    eager_steps = min(steps, 50)
    cache = QuantizedKVCache(mode="fused", device_lengths=True, fused_append=True,
                             capacity=S_HEAD + 2 * (steps + warmup) + eager_steps + 512)
    # prefill through the public API: dequantize our codes back to bf16 and update()
    with torch.cuda.stream(stream):
        for l, (k8, ks, v8, vs) in enumerate(caches):
            kd = kernels.dequant(k8, ks, torch.bfloat16, per_channel=True)
            vd = kernels.dequant(v8, vs, torch.bfloat16, per_channel=False)
            cache.update(kd, vd, l)
            del kd, vd
    torch.cuda.synchronize()
    per_layer_in = (B * HQ * D + 2 * B * HKV * D) * 2
    h_in = torch.randn((nl, per_layer_in // 2), dtype=torch.float32).to(torch.bfloat16).pin_memory()
    h_out = torch.empty((nl, B, 1, HQ, D), dtype=torch.bfloat16).pin_memory()
    d_in = torch.empty_like(h_in, device=device)
    d_out = torch.empty((nl, B, 1, HQ, D), dtype=torch.bfloat16, device=device)
    nq, nk = B * HQ * D, B * HKV * D

    def one_step():
        d_in.copy_(h_in, non_blocking=True)
        outs = []
        for l in range(nl):
            qv = d_in[l, :nq].view(B, 1, HQ, D).transpose(1, 2)
            kn = d_in[l, nq:nq + nk].view(B, 1, HKV, D).transpose(1, 2)
            vn = d_in[l, nq + nk:].view(B, 1, HKV, D).transpose(1, 2)
            k, v = cache.update(kn, vn, l)
            o, _ = attn_fwd(module, qv, k, v, None, scaling=1.0 / math.sqrt(D))
            outs.append(o)
        torch.stack(outs, out=d_out)  # the step's result, gathered by one kernel
        h_out.copy_(d_out, non_blocking=True)

    def timed(run, n, label):
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push(label)
        ev0.record(stream)
        for _ in range(n):
            run()
        ev1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        if world > 1:
            dist.barrier()
        ms = ev0.elapsed_time(ev1) / n
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with torch.cuda.stream(stream):
        for _ in range(2):
            one_step()               # eager: workspaces and kernel attributes set up
        torch.cuda.synchronize()
        ms_eager = timed(one_step, eager_steps, "e2e_eager_step")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            one_step()               # recorded, not run: the device lengths stay
        for _ in range(warmup):
            g.replay()
        torch.cuda.synchronize()
        ms = timed(g.replay, steps, "e2e_step")
        done = 2 + eager_steps + warmup + steps
        lens = cache.sync_lengths()
        if any(n != S_HEAD + done for n in lens.values()):
            raise RuntimeError(f"e2e: device lengths {set(lens.values())} != {S_HEAD + done}")
        del g
    S_mid = S_HEAD + done - steps // 2
    per_step = world * nl * decode_bytes(B, HQ, HKV, S_mid, D, scale_bytes=2)
    gbs = per_step / (ms * 1e-3) / 1e9
    del cache
    return {"value": round(gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": nl * per_layer_in,
            "d2h_bytes_per_step": nl * B * HQ * D * 2, "ms_per_step": round(ms, 4),
            "path": "QuantizedKVCache(device_lengths=True, fused_append=True).update + "
                    "quantized_attention_forward per layer (append inside the decode launch), the "
                    "step (H2D copy, 28 layers, D2H copy) captured once as a CUDA graph and "
                    "replayed per token; fp16 cache scales",
            "eager": {"value": round(per_step / (ms_eager * 1e-3) / 1e9, 2),
                      "ms_per_step": round(ms_eager, 4),
                      "path": "the same calls made eagerly from Python every step"}}


def run_batched(torch, kernels, device, stream, world, dist, peak, B_all=64, S=8192, nl=LAYERS):
    """Batched decode (B=64 sequences of S=8192, 28 layers): the batch is split
    across ranks (B/N per GPU, no collective); one CUDA graph per 28-layer step."""
    if B_all % world:
        return None
    b = B_all // world
    gen = torch.Generator(device=device).manual_seed(77 + (dist.get_rank() if world > 1 else 0))
    caches = []
    for _ in range(nl):
        k8 = torch.randint(-127, 128, (b, HKV, S, D), generator=gen, device=device, dtype=torch.int8)
        v8 = torch.randint(-127, 128, (b, HKV, S, D), generator=gen, device=device, dtype=torch.int8)
        ks = torch.rand((b, HKV, 1, D), generator=gen, device=device) * 0.1
        vs = torch.rand((b, HKV, S, 1), generator=gen, device=device) * 0.02
        caches.append((k8, ks, v8, vs))
    q = torch.randn((nl, b, HQ, D), generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    sm_scale = 1.0 / math.sqrt(D)

    def step():
        for l, (k8, ks, v8, vs) in enumerate(caches):
            kernels.int8_decode_attn(q[l], k8, ks, v8, vs, HQ // HKV, sm_scale=sm_scale, out=out[l])

    with torch.cuda.stream(stream):
        ms, _ = time_graph(torch, step, 20, 3, stream, label="batched_step",
                           barrier=dist.barrier if world > 1 else None)
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    per_layer = decode_bytes(b, HQ, HKV, S, D)
    del caches, q, out
    torch.cuda.empty_cache()
    return {"workload": f"B={B_all} sequences ({b} per GPU), S={S}, Hq={HQ}, Hkv={HKV}, D={D}, "
                        f"{nl} layers, int8 K/V + fp32 scales; one CUDA graph per step",
            "ms_per_step": round(ms, 4), "us_per_layer": round(ms * 1e3 / nl, 2),
            "gbs": round(world * nl * per_layer / (ms * 1e-3) / 1e9, 1),
            "frac_of_peak_per_gpu": round(nl * per_layer / (ms * 1e-3) / 1e9 / peak, 4)}


def run_extras(torch, kernels, device, gen, stream, us_int8, peak):
    """bf16-twin speedup at S=32K, the S sweep, bulk quantize-on-write GB/s."""
    res = {}
    sm_scale = 1.0 / math.sqrt(D)
    # -- twin at S=32K (28 bf16 layers: 3.8 GB)
    twin = make_layer_caches(torch, kernels, LAYERS, S_HEAD, device, gen, kv="bf16")
    q = torch.randn((LAYERS, B, HQ, D), generator=gen, device=device).to(torch.bfloat16)
    o = torch.empty_like(q)

    def tstep(cuda_cores):
        def run():
            for l, (k, v) in enumerate(twin):
                kernels.fp16_decode_attn(q[l], k, v, HQ // HKV, sm_scale=sm_scale, out=o[l],
                                         cuda_cores=cuda_cores)
        return run
    with torch.cuda.stream(stream):
        ms, _ = time_graph(torch, tstep(False), 200, 10, stream)
        ms_fma, _ = time_graph(torch, tstep(True), 200, 10, stream)
    us_bf16, us_fma = ms * 1e3 / LAYERS, ms_fma * 1e3 / LAYERS
    # the same-design twin (128-token TMA tiles, same ring / split plan / merge, bf16 tensor cores)
    res["bf16_twin_us_per_layer"] = round(us_bf16, 3)
    res["int8_vs_bf16_speedup"] = round(us_bf16 / us_int8, 3)
    res["bf16_twin_frac_of_peak"] = round(decode_bytes(B, HQ, HKV, S_HEAD, D, kv_bytes=2) /
                                          (us_bf16 * 1e-6) / 1e9 / peak, 4)
    # second comparison point: the CUDA-core float32 twin over 64-token bulk-copied tiles
    res["bf16_fma_twin_us_per_layer"] = round(us_fma, 3)
    res["int8_vs_bf16_fma_speedup"] = round(us_fma / us_int8, 3)
    del twin
    torch.cuda.empty_cache()
    # -- sweep
    sweep = []
    for S in (64, 512, 4096, 32768, 131072):
        per8 = decode_bytes(B, HQ, HKV, S, D)
        n = max(4, min(2048, math.ceil(3 * L2_BYTES / per8)))
        c8 = make_sweep_caches(torch, n, S, device, gen, "int8")
        c16 = make_sweep_caches(torch, max(4, min(2048, math.ceil(3 * L2_BYTES / (2 * per8)))),
                                S, device, gen, "bf16")
        qq = torch.randn((B, HQ, D), generator=gen, device=device).to(torch.bfloat16)
        oo = torch.empty_like(qq)

        def s8():
            for (k8, ks, v8, vs) in c8:
                kernels.int8_decode_attn(qq, k8, ks, v8, vs, HQ // HKV, sm_scale=sm_scale, out=oo)

        def s16():
            for (k, v) in c16:
                kernels.fp16_decode_attn(qq, k, v, HQ // HKV, sm_scale=sm_scale, out=oo)
        reps = max(3, min(200, int(2e5 / (n * max(1.0, S / 4096)))))
        with torch.cuda.stream(stream):
            m8, _ = time_graph(torch, s8, reps, 3, stream)
            m16, _ = time_graph(torch, s16, reps, 3, stream)
        u8, u16 = m8 * 1e3 / len(c8), m16 * 1e3 / len(c16)
        sweep.append({"S": S, "us_int8": round(u8, 3), "us_bf16": round(u16, 3),
                      "speedup": round(u16 / u8, 3), "gbs_int8": round(per8 / u8 / 1e3, 1),
                      "layers": len(c8)})
        del c8, c16
        torch.cuda.empty_cache()
    res["decode_sweep"] = sweep
    # -- bulk quantize-on-write, config B=8, Hkv=8, S=32768, D=128 bf16
    Bq, Hq_, Sq = 8, 8, 32768
    k = torch.randn((Bq, Hq_, Sq, D), generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn((Bq, Hq_, Sq, D), generator=gen, device=device).to(torch.bfloat16)
    k8 = torch.empty((Bq, Hq_, Sq, D), dtype=torch.int8, device=device)
    v8 = torch.empty_like(k8)
    ks = torch.empty((Bq, Hq_, 1, D), dtype=torch.float32, device=device)
    vs = torch.empty((Bq, Hq_, Sq, 1), dtype=torch.float32, device=device)
    n = Bq * Hq_ * Sq * D
    kb = 3 * n + Bq * Hq_ * D * 4
    vb = 3 * n + Bq * Hq_ * Sq * 4
    with torch.cuda.stream(stream):
        mk, _ = time_graph(torch, lambda: kernels.quant_k_perchannel(
            k, out=k8, scale_dtype=None, scale_f32_out=ks), 20, 3, stream)
        mv, _ = time_graph(torch, lambda: kernels.quant_v_pertoken(
            v, out=v8, scale_dtype=None, scale_f32_out=vs), 20, 3, stream)
        ks_static = kernels.calibrate_k_scale([k])
        ms_, _ = time_graph(torch, lambda: kernels.quant_k_static(k, ks_static, out=k8), 20, 3,
                            stream)
    res["quant_write"] = {
        "workload": "B=8, Hkv=8, S=32768, D=128 bf16 -> int8 + fp32 scales (1.07 GB input, > L2)",
        "k_gbs": round(kb / (mk * 1e-3) / 1e9, 1), "k_us": round(mk * 1e3, 2),
        "k_frac_of_peak": round(kb / (mk * 1e-3) / 1e9 / peak, 4),
        "v_gbs": round(vb / (mv * 1e-3) / 1e9, 1), "v_us": round(mv * 1e3, 2),
        "v_frac_of_peak": round(vb / (mv * 1e-3) / 1e9 / peak, 4),
        "k_static_gbs": round((3 * n + Hq_ * D * 4) / (ms_ * 1e-3) / 1e9, 1),
        "k_static_us": round(ms_ * 1e3, 2),
        "k_static_frac_of_peak": round((3 * n + Hq_ * D * 4) / (ms_ * 1e-3) / 1e9 / peak, 4),
        "k_static_note": "K with calibrated static per-channel scales (no column maximum)"}
    # -- 1024 single-token appends (B=8, Hkv=8): fused append kernel latency
    kn = torch.randn((Bq, Hq_, 1, D), generator=gen, device=device).to(torch.bfloat16)
    vn = torch.randn((Bq, Hq_, 1, D), generator=gen, device=device).to(torch.bfloat16)
    vs16 = torch.empty((Bq, Hq_, Sq, 1), dtype=torch.float16, device=device)

    def app():
        for i in range(1024):
            p = Sq - 1024 + i
            kernels.append_kv(kn, vn, k8[:, :, p:p + 1], v8[:, :, p:p + 1],
                              v_scale_dst=vs16[:, :, p:p + 1])
    with torch.cuda.stream(stream):
        ma, _ = time_graph(torch, app, 5, 2, stream)
    res["quant_write"]["append_us"] = round(ma * 1e3 / 1024, 3)
    del k, v, k8, v8
    torch.cuda.empty_cache()
    res["prefill"] = run_prefill(torch, kernels, device, gen, stream)
    res["kblock"] = run_kblock(torch, kernels, device, gen, stream, us_int8, peak)
    res["model_decode_step"] = run_model_step(torch, device)
    return res


def make_kblock_caches(torch, kernels, n_layers, S, device, gen, block=128):
    """n_layers block-wise K caches (K per 128-token block and channel, V per token,
    fp16 V scales) of outlier K and normal V, written by the product's kernel."""
    caches = []
    for _ in range(n_layers):
        k = torch.randn((B, HKV, S, D), generator=gen, device=device)
        ch = torch.stack([torch.randperm(D, generator=gen, device=device)[:4] for _ in range(B * HKV)])
        gain = torch.ones((B * HKV, D), device=device).scatter_(1, ch, 20.0).view(B, HKV, 1, D)
        k = (k * gain).to(torch.bfloat16)
        v = torch.randn((B, HKV, S, D), generator=gen, device=device).to(torch.bfloat16)
        c = kernels.kblock_alloc(B, HKV, S, D, block_tokens=block, device=device)
        kernels.kblock_write(k, v, 0, c)
        caches.append(c)
        del k, v
    return caches


def kblock_decode_bytes(b, hq, hkv, s, d, block=128):
    """K and V codes, fp16 V scales, f32 K block scales, q in and out (bf16)."""
    return b * (hkv * s * (2 * d + 2) + hkv * (-(-s // block)) * d * 4 + 2 * hq * d * 2)


def run_kblock(torch, kernels, device, gen, stream, us_int8, peak, S=S_HEAD):
    """The opt-in block-wise per-channel K layout: decode at config 2's shape
    (28 layers per CUDA graph), the bulk write of config 4 and the one-token append."""
    sm_scale = 1.0 / math.sqrt(D)
    res = {"workload": f"B={B}, Hq={HQ}, Hkv={HKV}, D={D}, S={S}, 128-token K blocks, "
                       f"{LAYERS} layers per CUDA graph; write: B=8, Hkv=8, S=32768 bf16"}
    caches = make_kblock_caches(torch, kernels, LAYERS, S, device, gen)
    q = torch.randn((LAYERS, B, HQ, D), generator=gen, device=device).to(torch.bfloat16)
    o = torch.empty_like(q)

    def step():
        for l, c in enumerate(caches):
            kernels.kblock_decode(q[l], c, S, sm_scale=sm_scale, out=o[l])
    with torch.cuda.stream(stream):
        ms, _ = time_graph(torch, step, 200, 10, stream)
    us = ms * 1e3 / LAYERS
    gbs = kblock_decode_bytes(B, HQ, HKV, S, D) / us / 1e3
    res.update({"decode_us_per_layer": round(us, 3), "decode_gbs": round(gbs, 1),
                "decode_frac_of_peak": round(gbs / peak, 4),
                "vs_int8_decode": round(us_int8 / us, 3)})
    # one-token append into an open block (re-codes the block's channels whose scale grew)
    c0 = caches[0]
    kn = torch.randn((B, HKV, 1, D), generator=gen, device=device).to(torch.bfloat16)
    big = kernels.kblock_alloc(B, HKV, S + 512, D, device=device)
    kernels.kblock_write(torch.randn((B, HKV, S - 64, D), generator=gen, device=device)
                         .to(torch.bfloat16), None, 0, big)
    with torch.cuda.stream(stream):
        kernels.kblock_write(kn, kn, S - 64, big)   # first launch outside the capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(64):   # 64 consecutive tokens: the open block re-coded as it grows
                kernels.kblock_write(kn, kn, S - 63 + i, big)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del g
    res["append_us"] = round(e0.elapsed_time(e1) * 1e3 / 64, 3)
    del caches, big, c0
    torch.cuda.empty_cache()
    # bulk write of config 4 (K block-wise + V per token)
    Bw, Hw, Sw = 8, 8, 32768
    x = torch.randn((Bw, Hw, Sw, D), generator=gen, device=device).to(torch.bfloat16)
    cw = kernels.kblock_alloc(Bw, Hw, Sw, D, device=device)

    def wr():
        kernels.kblock_write(x, x, 0, cw)
    with torch.cuda.stream(stream):
        mw, _ = time_graph(torch, wr, 20, 3, stream)
    nbytes = Bw * Hw * Sw * D * (2 + 2 + 1 + 1) + Bw * Hw * Sw * 2 + Bw * Hw * (Sw // 128) * D * 4
    res.update({"write_us": round(mw * 1e3, 2), "write_gbs": round(nbytes / mw / 1e6, 1),
                "write_frac_of_peak": round(nbytes / mw / 1e6 / peak, 4)})
    del x, cw
    torch.cuda.empty_cache()
    return res


def run_model_step(torch, device, n0=512, nd=64):
    """Config 1's model (Qwen3-0.6B architecture, random init, bf16, 28 layers) through
    HF transformers with QuantizedKVCache and the patched attention: prefill 512 tokens,
    then one decode step per token - the whole forward (all layers, the int8 cache
    update and attention, the LM head) captured once as a CUDA graph and replayed,
    against the same step run eagerly.  Per-token latency."""
    from transformers import Qwen3Config, Qwen3ForCausalLM

    from halftone_quantizedkvcache_b200.integration import QuantizedKVCache, installed
    cfg = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072,
                      num_hidden_layers=LAYERS, num_attention_heads=HQ, num_key_value_heads=HKV,
                      head_dim=D, rope_theta=1e6, max_position_embeddings=40960, rms_norm_eps=1e-6,
                      tie_word_embeddings=True, attention_bias=False, use_sliding_window=False)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    with torch.device(device):
        model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (1, n0 + 2 * nd + 8), generator=g).to(device)
    res = {"workload": f"Qwen3-0.6B architecture (random init, bf16, {LAYERS} layers), prefill "
                       f"{n0} tokens, decode steps at S~{n0}-{n0 + 2 * nd}, batch 1"}
    with torch.no_grad(), installed():
        def run(graph):
            cache = QuantizedKVCache(mode="fused", capacity=n0 + 2 * nd + 256,
                                     device_lengths=graph, fused_append=graph)
            model(ids[:, :n0], past_key_values=cache, use_cache=True)
            tok = torch.empty((1, 1), dtype=torch.long, device=device)
            pos = torch.empty((1, 1), dtype=torch.long, device=device)
            masks = {"full_attention": None}
            st = torch.cuda.Stream(device)
            st.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(st):
                def step():
                    return model(input_ids=tok, position_ids=pos, attention_mask=masks,
                                 past_key_values=cache, use_cache=True).logits
                t = n0
                tok.copy_(ids[:, t:t + 1])
                pos.fill_(t)
                step()
                t += 1
                run_step = step
                if graph:
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr, stream=st):
                        step()
                    run_step = gr.replay
                for _ in range(3):
                    tok.copy_(ids[:, t:t + 1])
                    pos.fill_(t)
                    run_step()
                    t += 1
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                for _ in range(nd):
                    tok.copy_(ids[:, t:t + 1])
                    pos.fill_(t)
                    run_step()
                    t += 1
                e1.record(st)
                torch.cuda.synchronize()
                if graph:
                    del gr
            return e0.elapsed_time(e1) / nd

        ms_graph = run(True)
        ms_eager = run(False)
    del model
    torch.cuda.empty_cache()
    res.update({"ms_per_token_graph": round(ms_graph, 4), "ms_per_token_eager": round(ms_eager, 4),
                "speedup": round(ms_eager / ms_graph, 2)})
    return res


def run_prefill(torch, kernels, device, gen, stream, S=512, nl=LAYERS):
    """Prefill attention of config 1 (B=1, Hq=16, Hkv=8, D=128, 512 tokens, causal)
    over the int8 cache of 28 layers: the fused kernel against the reference's
    path (dequantize K and V, then its torch attention math), one CUDA graph each."""
    from halftone_quantizedkvcache_b200.integration.quantized_attention import (
        _fake_quant, _reference_math)
    sm_scale = 1.0 / math.sqrt(D)
    caches = make_layer_caches(torch, kernels, nl, S, device, gen)
    caches = [(k8, ks.half(), v8, vs.half()) for (k8, ks, v8, vs) in caches]  # fp16 cache scales
    q = torch.randn((nl, B, HQ, S, D), generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty((nl, B, S, HQ, D), dtype=torch.bfloat16, device=device)
    allowed = torch.arange(S, device=device)[None, :] <= torch.arange(S, device=device)[:, None]
    mask = torch.zeros((S, S), dtype=torch.bfloat16, device=device).masked_fill(
        ~allowed, torch.finfo(torch.bfloat16).min)[None, None]
    module = _Attn(HQ // HKV, D)

    def fused():
        for l, (k8, ks, v8, vs) in enumerate(caches):
            kernels.int8_prefill_attn(q[l], k8, ks, v8, vs, HQ // HKV, sm_scale=sm_scale,
                                      q_quant=True, out=out[l])

    def reference_path():
        for l, (k8, ks, v8, vs) in enumerate(caches):
            kd = kernels.dequant(k8, ks, torch.bfloat16, per_channel=True)
            vd = kernels.dequant(v8, vs, torch.bfloat16, per_channel=False)
            out[l].copy_(_reference_math(module, _fake_quant(q[l], (3,)), kd, vd, mask, sm_scale,
                                         0.0))
    with torch.cuda.stream(stream):
        mf, _ = time_graph(torch, fused, 100, 5, stream)
        mr, _ = time_graph(torch, reference_path, 100, 5, stream)
    flops = 4 * B * HQ * D * S * (S + 1) / 2  # causal QK^T and PV
    del caches
    torch.cuda.empty_cache()
    return {"workload": f"causal prefill B={B}, Hq={HQ}, Hkv={HKV}, D={D}, {S} tokens over the "
                        f"int8 cache (fp16 scales), {nl} layers per CUDA graph",
            "fused_us_per_layer": round(mf * 1e3 / nl, 3),
            "reference_path_us_per_layer": round(mr * 1e3 / nl, 3),
            "speedup": round(mr / mf, 3),
            "fused_tflops": round(flops / (mf * 1e-3 / nl) / 1e12, 2)}


def profile_only(args, torch, kernels, device, gen, stream):
    """A few launches of one kernel family on a small case, for ncu captures."""
    sm_scale = 1.0 / math.sqrt(D)
    with torch.cuda.stream(stream):
        if args.only in ("decode", "twin"):
            kind = "int8" if args.only == "decode" else "bf16"
            caches = make_layer_caches(torch, kernels, args.layers, S_HEAD, device, gen, kv=kind)
            q = torch.randn((B, HQ, D), generator=gen, device=device).to(torch.bfloat16)
            o = torch.empty_like(q)
            torch.cuda.synchronize()
            for _ in range(args.warmup + args.steps):
                for c in caches:
                    if kind == "int8":
                        kernels.int8_decode_attn(q, *c, HQ // HKV, sm_scale=sm_scale, out=o)
                    else:
                        kernels.fp16_decode_attn(q, *c, HQ // HKV, sm_scale=sm_scale, out=o)
        elif args.only == "kblock":
            caches = make_kblock_caches(torch, kernels, args.layers, S_HEAD, device, gen)
            q = torch.randn((B, HQ, D), generator=gen, device=device).to(torch.bfloat16)
            o = torch.empty_like(q)
            torch.cuda.synchronize()
            for _ in range(args.warmup + args.steps):
                for c in caches:
                    kernels.kblock_decode(q, c, S_HEAD, sm_scale=sm_scale, out=o)
        elif args.only == "kstatic":
            x = torch.randn((2, 8, 32768, D), generator=gen, device=device).to(torch.bfloat16)
            y = torch.empty(x.shape, dtype=torch.int8, device=device)
            s = kernels.calibrate_k_scale([x])
            torch.cuda.synchronize()
            for _ in range(args.warmup + args.steps):
                kernels.quant_k_static(x, s, out=y)
        elif args.only == "prefill":
            caches = make_layer_caches(torch, kernels, args.layers, 512, device, gen)
            caches = [(k8, ks.half(), v8, vs.half()) for (k8, ks, v8, vs) in caches]
            q = torch.randn((B, HQ, 512, D), generator=gen, device=device).to(torch.bfloat16)
            torch.cuda.synchronize()
            for _ in range(args.warmup + args.steps):
                for c in caches:
                    kernels.int8_prefill_attn(q, *c, HQ // HKV, sm_scale=sm_scale, q_quant=True)
        else:
            x = torch.randn((8, 8, 32768, D), generator=gen, device=device).to(torch.bfloat16)
            y = torch.empty(x.shape, dtype=torch.int8, device=device)
            s32k = torch.empty((8, 8, 1, D), dtype=torch.float32, device=device)
            s32v = torch.empty((8, 8, 32768, 1), dtype=torch.float32, device=device)
            torch.cuda.synchronize()
            for _ in range(args.warmup + args.steps):
                kernels.quant_k_perchannel(x, out=y, scale_dtype=None, scale_f32_out=s32k)
                kernels.quant_v_pertoken(x, out=y, scale_dtype=None, scale_f32_out=s32v)
    torch.cuda.synchronize()
    print(json.dumps({"profile_only": args.only, "steps": args.steps, "layers": args.layers}))
    return 0


def make_sweep_caches(torch, n, S, device, gen, kind):
    out = []
    for _ in range(n):
        if kind == "int8":
            k8 = torch.randint(-127, 128, (B, HKV, S, D), generator=gen, device=device,
                               dtype=torch.int8)
            v8 = torch.randint(-127, 128, (B, HKV, S, D), generator=gen, device=device,
                               dtype=torch.int8)
            ks = torch.rand((B, HKV, 1, D), generator=gen, device=device) * 0.1
            vs = torch.rand((B, HKV, S, 1), generator=gen, device=device) * 0.02
            out.append((k8, ks, v8, vs))
        else:
            k = torch.randn((B, HKV, S, D), generator=gen, device=device).to(torch.bfloat16)
            v = torch.randn((B, HKV, S, D), generator=gen, device=device).to(torch.bfloat16)
            out.append((k, v))
    return out


if __name__ == "__main__":
    sys.exit(main())
