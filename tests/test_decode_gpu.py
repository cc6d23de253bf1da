"""Decode-attention parity on the GPU (split-KV int8 kernel, dense twin, combine).

Oracle: ``oracle.attention`` (reference/page_attention_reference.py:31-54 on the
cache dequantized as reference/page_attention_int8_pytorch.py:33-34), pinned to
the reference's outputs by tests/test_oracle_golden.py.  Tolerance (north
star): max-abs 1e-3 and relative 1e-3 on the float32 result, checked on the
kernel's float32 partial output; outputs stored in bf16 add their own
rounding (<= 2^-9 relative), checked separately.
"""
import math

import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200 import kernels
from oracle import attention as oa
from oracle import inputs as oin
from oracle import quant as oq

pytestmark = pytest.mark.gpu
TDT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
ATOL = RTOL = 1e-3


def dev(x, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(x))
    return (t.to(TDT[dt]) if dt else t).cuda()


def run_int8(c, q_dt="bf16", scale_dt="f32", q_quant=False, n_rep=None):
    q = dev(c["q"], q_dt)
    ks, vs = c["k_sc"], c["v_sc"]
    if scale_dt == "f16":
        ks, vs = oq.to_f16(ks), oq.to_f16(vs)
    args = (q, dev(c["k_i8"]), dev(ks), dev(c["v_i8"]), dev(vs))
    B, Hq, D = q.shape
    part = torch.empty((B, Hq, D + 2), dtype=torch.float32, device="cuda")
    kernels.int8_decode_attn(*args, n_rep, q_quant=q_quant, partial_out=part)
    out = kernels.int8_decode_attn(*args, n_rep, q_quant=q_quant)
    torch.cuda.synchronize()
    p = part.cpu().numpy()
    f32 = p[..., 2:] / p[..., 1:2]
    return f32, out.float().cpu().numpy()


def oracle_int8(c, scale_dt="f32", q_in=None):
    ks, vs = c["k_sc"], c["v_sc"]
    if scale_dt == "f16":
        ks, vs = oq.to_f16(ks).astype(np.float32), oq.to_f16(vs).astype(np.float32)
    q = c["q"] if q_in is None else q_in
    return oa.decode_int8(q, c["k_i8"], ks, c["v_i8"], vs, acc="f64")


def close(got, ref, atol=ATOL, rtol=RTOL, msg=""):
    np.testing.assert_allclose(got, ref, atol=atol, rtol=rtol, err_msg=msg)


def test_golden_cases(golden):
    g = golden("decode_golden.npz")
    for name in sorted({k.split("/")[0] for k in g.files}):
        dt = str(g[f"{name}/dtype"])
        c = {"q": oq.unpack(g[f"{name}/q"], dt)}
        for key in ("k_i8", "k_sc", "v_i8", "v_sc"):
            c[key] = g[f"{name}/{key}"]
        f32, out = run_int8(c, q_dt=dt)
        ref = g[f"{name}/out"]
        close(f32, ref, msg=name)
        close(out, ref, atol=ATOL, rtol=2.0 ** -7, msg=name + " stored")


def test_config0_fp32(golden):
    g = golden("config0_golden.npz")
    q, k, v = oin.config0(int(g["seed"]))
    k_i8, k_sc = oq.quantize_int8(k, (2,))
    v_i8, v_sc = oq.quantize_int8(v, (3,))
    c = dict(q=q, k_i8=k_i8, k_sc=k_sc, v_i8=v_i8, v_sc=v_sc)
    f32, out = run_int8(c, q_dt="f32")
    close(f32[0], g["attn_out"])
    close(out[0], g["attn_out"])


@pytest.mark.parametrize("S", [1, 2, 63, 64, 65, 127, 1000, 4096, 32768])
@pytest.mark.parametrize("B", [1, 3])
def test_length_sweep(S, B):
    c = oin.decode_case(1000 + S + B, B, 16, 8, S, 128)
    f32, out = run_int8(c)
    ref = oracle_int8(c)
    close(f32, ref, msg=f"S={S} B={B}")
    close(out, ref, atol=ATOL, rtol=2.0 ** -7)


def test_long_131072():
    c = oin.decode_case(7, 1, 16, 8, 131072, 128)
    f32, out = run_int8(c)
    close(f32, oracle_int8(c))


@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 8), (16, 4), (32, 8)])
@pytest.mark.parametrize("scale_dt", ["f32", "f16"])
def test_group_sizes_and_scale_dtypes(hq, hkv, scale_dt):
    c = oin.decode_case(hq * 100 + hkv, 2, hq, hkv, 777, 128)
    f32, _ = run_int8(c, scale_dt=scale_dt)
    close(f32, oracle_int8(c, scale_dt))


@pytest.mark.parametrize("q_dt", ["f32", "f16"])
def test_q_dtypes(q_dt):
    c = oin.decode_case(55, 2, 16, 8, 513, 128, q_dtype=q_dt)
    f32, out = run_int8(c, q_dt=q_dt)
    ref = oracle_int8(c)
    close(f32, ref)
    close(out, ref)


def test_q_fake_quant_prologue():
    """tests/qwen_kvcache_full.py:103: q -> bf16(code * scale) per token before attention."""
    c = oin.decode_case(66, 2, 16, 8, 900, 128)
    q_in = oa.quant_dequant(c["q"], (2,), "bf16")
    f32, _ = run_int8(c, q_quant=True)
    close(f32, oracle_int8(c, q_in=q_in))


@pytest.mark.parametrize("cuda_cores", [False, True], ids=["tensor_cores", "cuda_cores"])
@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("S", [5, 4096, 32768])
def test_dense_twin(dt, S, cuda_cores):
    c = oin.decode_case(77 + S, 2, 16, 8, S, 128, kv_dtype=dt, q_dtype=dt)
    q, k, v = dev(c["q"], dt), dev(c["k"], dt), dev(c["v"], dt)
    B, Hq, D = q.shape
    part = torch.empty((B, Hq, D + 2), dtype=torch.float32, device="cuda")
    kernels.fp16_decode_attn(q, k, v, 2, partial_out=part, cuda_cores=cuda_cores)
    out = kernels.fp16_decode_attn(q, k, v, 2, cuda_cores=cuda_cores)
    p = part.cpu().numpy()
    ref = oa.decode_dense(c["q"], c["k"], c["v"], 2, 1 / math.sqrt(128), acc="f64")
    close(p[..., 2:] / p[..., 1:2], ref)
    close(out.float().cpu().numpy(), ref, atol=ATOL, rtol=2.0 ** -7)


@pytest.mark.parametrize("B,Hq,Hkv,S", [(1, 8, 8, 1), (3, 16, 4, 777), (1, 32, 8, 131072),
                                        (2, 4, 4, 129), (1, 16, 8, 0)])
@pytest.mark.parametrize("q_quant", [False, True])
def test_dense_twin_shapes(B, Hq, Hkv, S, q_quant):
    """The tensor-core twin over every group size it serves (n_rep 1, 2, 4), ragged
    lengths, a single token, an empty cache and the per-token q fake quantization."""
    c = oin.decode_case(5 + S + B, B, Hq, Hkv, max(S, 1), 128, kv_dtype="bf16", q_dtype="bf16")
    k, v = c["k"][:, :, :S], c["v"][:, :, :S]
    q, kt, vt = dev(c["q"], "bf16"), dev(np.ascontiguousarray(k), "bf16"), dev(np.ascontiguousarray(v), "bf16")
    part = torch.empty((B, Hq, 130), dtype=torch.float32, device="cuda")
    kernels.fp16_decode_attn(q, kt, vt, Hq // Hkv, partial_out=part, q_quant=q_quant)
    p = part.cpu().numpy()
    if S == 0:
        assert np.all(p[..., 1] == 0) and np.all(p[..., 2:] == 0)
        return
    qin = oa.quant_dequant(c["q"], (2,), "bf16") if q_quant else c["q"]
    ref = oa.decode_dense(qin, k, v, Hq // Hkv, 1 / math.sqrt(128), acc="f64")
    close(p[..., 2:] / p[..., 1:2], ref)


def test_reference_layout_and_partial_combine():
    """Reference layout q [Hq,1,D], K/V [Hkv,S,D]; two halves combined == whole."""
    c = oin.decode_case(88, 1, 16, 8, 3000, 128)
    q = dev(c["q"][0][:, None, :], "bf16")
    k, v = dev(c["k_i8"][0]), dev(c["v_i8"][0])
    ks, vs = dev(c["k_sc"][0]), dev(c["v_sc"][0])
    out = kernels.int8_decode_attn(q, k, ks, v, vs, 2)
    assert out.shape == (16, 1, 128) and out.dtype == torch.bfloat16
    parts = torch.empty((2, 1, 16, 130), dtype=torch.float32, device="cuda")
    for i, (s0, s1) in enumerate(((0, 1280), (1280, 3000))):
        kernels.int8_decode_attn(q, k[:, s0:s1], ks, v[:, s0:s1], vs[:, s0:s1], 2,
                                 partial_out=parts[i])
    comb = kernels.decode_combine(parts, out_dtype=torch.float32)
    ref = oracle_int8(c)
    close(comb.cpu().numpy(), ref)
    close(out[:, 0].float().cpu().numpy(), ref[0], atol=ATOL, rtol=2.0 ** -7)


def test_empty_cache_gives_zeros():
    q = torch.randn((1, 16, 128), device="cuda").bfloat16()
    k = torch.zeros((1, 8, 0, 128), dtype=torch.int8, device="cuda")
    ks = torch.ones((1, 8, 1, 128), device="cuda")
    vs = torch.ones((1, 8, 0, 1), device="cuda")
    out = kernels.int8_decode_attn(q, k, ks, k, vs)
    assert torch.count_nonzero(out) == 0


def test_repeatable_and_status_clean():
    c = oin.decode_case(99, 1, 16, 8, 32768, 128)
    a = run_int8(c)[1]
    b = run_int8(c)[1]
    np.testing.assert_array_equal(a, b)
    assert kernels.read_status("decode") == 0


@pytest.mark.parametrize("S", [700, 32768])
def test_overlapped_launches_match_serial(S):
    """HQ_DECODE_OVERLAP_PREVIOUS (programmatic dependent launch): consecutive
    decodes of several layers, eagerly and replayed from a CUDA graph, give the
    serial launches' outputs bit for bit; each layer's q is written by the kernel
    just before its decode, so q must wait for it."""
    layers = 6
    cs = [oin.decode_case(300 + S + i, 1, 16, 8, S, 128) for i in range(layers)]
    caches = [(dev(c["k_i8"]), dev(c["k_sc"]), dev(c["v_i8"]), dev(c["v_sc"])) for c in cs]
    q_src = torch.stack([dev(c["q"], "bf16") for c in cs])
    q = torch.empty_like(q_src)
    serial = torch.empty_like(q_src)
    over = torch.empty_like(q_src)

    def step(out, overlap):
        for i, (k8, ks, v8, vs) in enumerate(caches):
            q[i].copy_(q_src[i])  # the kernel before each decode writes its q
            kernels.int8_decode_attn(q[i], k8, ks, v8, vs, 2, out=out[i], overlap_prev=overlap)

    step(serial, False)
    step(over, True)
    torch.cuda.synchronize()
    assert torch.equal(serial, over)
    for i, c in enumerate(cs):
        close(over[i].float().cpu().numpy(), oracle_int8(c), atol=2e-2, rtol=2e-2)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step(over, True)  # this stream's workspace exists before the capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step(over, True)
        over.zero_()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
    assert torch.equal(serial, over)
    assert kernels.read_status("decode") == 0
    del g


def test_wrappers_reject_shapes_that_disagree():
    """The library reads K/V and scales by the call's counts: the torch wrappers
    reject tensors whose shapes disagree with q before anything is launched."""
    q = torch.zeros((2, 16, 128), dtype=torch.bfloat16, device="cuda")
    k = torch.zeros((1, 8, 64, 128), dtype=torch.int8, device="cuda")
    ks = torch.ones((1, 8, 1, 128), device="cuda")
    vs = torch.ones((1, 8, 64, 1), device="cuda")
    with pytest.raises(ValueError):
        kernels.int8_decode_attn(q, k, ks, k, vs, 2)              # two sequences, cache of one
    with pytest.raises(ValueError):
        kernels.int8_decode_attn(q[:1], k, ks, k, vs[:, :, :32], 2)  # V scales of 32 tokens
    with pytest.raises(ValueError):
        kernels.int8_decode_attn(q[:1], k, ks, k, vs, 2, out=torch.empty_like(q))
    d = torch.zeros((1, 8, 64, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        kernels.fp16_decode_attn(q, d, d, 2)
    qp = torch.zeros((1, 16, 8, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        kernels.int8_prefill_attn(qp, k, ks, k, vs, 2)            # head dim 64 against 128
    assert kernels.int8_decode_attn(q[:1], k, ks, k, vs, 2).shape == (1, 16, 128)


@pytest.mark.parametrize("B,Hq,Hkv,S", [(1, 16, 8, 32768), (2, 32, 8, 5000), (3, 16, 4, 777),
                                        (1, 8, 8, 1), (1, 4, 1, 131072), (2, 16, 8, 100)])
def test_dynamic_tile_schedule(B, Hq, Hkv, S):
    """HQ_DECODE_DYNAMIC_TILES: splits claim tiles as they go (V scales by tensor map).
    Within 1e-3 of the oracle, repeated calls included (the claim counters reset);
    fp16 V scales (the cache's layout) and fp32 ones."""
    c = oin.decode_case(31 + S + B, B, Hq, Hkv, S, 128)
    q = dev(c["q"], "bf16")
    k8, v8 = dev(c["k_i8"]), dev(c["v_i8"])
    for sdt, name in ((torch.float32, "f32"), (torch.float16, "f16")):
        ks, vs = dev(c["k_sc"]).to(sdt), dev(c["v_sc"]).to(sdt)
        ref = oracle_int8(c, scale_dt=name)
        part = torch.empty((B, Hq, 130), dtype=torch.float32, device="cuda")
        for _ in range(3):
            part.fill_(float("nan"))
            kernels.int8_decode_attn(q, k8, ks, v8, vs, Hq // Hkv, partial_out=part,
                                     dynamic_tiles=True)
            p = part.cpu().numpy()
            close(p[..., 2:] / p[..., 1:2], ref)
