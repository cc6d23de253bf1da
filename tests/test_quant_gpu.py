"""Quantize-on-write parity on the GPU: codes and scales bit-exact with the oracle.

Oracle: ``oracle.quant`` (numpy restatement of quantize_int8,
reference/page_attention_int8_pytorch.py:23-30, pinned to the reference's own
outputs by tests/test_oracle_golden.py).  Every case calls the CUDA kernels
through the C ABI (``halftone_quantizedkvcache_b200.kernels``).
"""
import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200 import kernels
from oracle import inputs as oin
from oracle import quant as oq

pytestmark = pytest.mark.gpu
TDT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def dev(x, dt):
    return torch.from_numpy(np.ascontiguousarray(x)).to(TDT[dt]).cuda()


def run_k(xt):
    B, H, S, D = xt.shape
    s16 = torch.empty((B, H, 1, D), dtype=torch.float16, device="cuda")
    s32 = torch.empty((B, H, 1, D), dtype=torch.float32, device="cuda")
    q, _ = kernels.quant_k_perchannel(xt, scale_out=s16, scale_f32_out=s32, scale_dtype=None)
    torch.cuda.synchronize()
    return q.cpu().numpy(), s32.cpu().numpy(), s16.cpu().numpy()


def run_v(xt):
    B, H, S, D = xt.shape
    s16 = torch.empty((B, H, S, 1), dtype=torch.float16, device="cuda")
    s32 = torch.empty((B, H, S, 1), dtype=torch.float32, device="cuda")
    q, _ = kernels.quant_v_pertoken(xt, scale_out=s16, scale_f32_out=s32, scale_dtype=None)
    torch.cuda.synchronize()
    return q.cpu().numpy(), s32.cpu().numpy(), s16.cpu().numpy()


def assert_bits(a, b, msg):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    assert a.dtype == b.dtype and a.shape == b.shape, msg
    np.testing.assert_array_equal(a.view(np.uint8), b.view(np.uint8), err_msg=msg)


def check_case(x, dt, xt=None, tag=""):
    xt = dev(x, dt) if xt is None else xt
    for name, run, ref in (("K", run_k, oq.quant_k_perchannel), ("V", run_v, oq.quant_v_pertoken)):
        q, s32, s16 = run(xt)
        rq, rs = ref(x)
        assert_bits(q, rq, f"{tag} {name} codes")
        assert_bits(s32, rs, f"{tag} {name} fp32 scale")
        assert_bits(s16, oq.to_f16(rs), f"{tag} {name} fp16 scale")


def test_golden_edge_cases(golden):
    g = golden("quant_golden.npz")
    names = sorted({k.split("/")[0] for k in g.files})
    for name in names:
        dt = str(g[f"{name}/dtype"])
        x = oq.unpack(g[f"{name}/x"], dt)
        xt = dev(x, dt)
        for tag, run in (("k", run_k), ("v", run_v)):
            q, s32, s16 = run(xt)
            assert_bits(q, g[f"{name}/{tag}_codes"], f"{name} {tag} codes")
            assert_bits(s32, g[f"{name}/{tag}_scale"], f"{name} {tag} scale")
            assert_bits(s16, g[f"{name}/{tag}_scale_f16"], f"{name} {tag} scale f16")


@pytest.mark.parametrize("shape,dt", [
    ((1, 8, 512, 128), "bf16"),      # config 0 shape
    ((2, 3, 1000, 128), "bf16"),     # several chunks, ragged tail
    ((1, 2, 1, 128), "bf16"),        # S = 1
    ((1, 2, 77, 64), "bf16"),
    ((1, 2, 33, 256), "bf16"),
    ((3, 2, 129, 128), "f16"),
    ((1, 2, 65, 128), "f32"),
    ((2, 4, 8192, 128), "bf16"),     # 64 chunks per slab, one group
    ((1, 1, 131072, 128), "bf16"),   # 1024 chunks of one slab: every block shares it
    ((1, 1, 40000, 256), "f32"),
    ((32, 8, 256, 128), "bf16"),     # 256 slabs of 2 chunks: one block range spans slabs
    ((16, 8, 300, 64), "f16"),       # ragged 3-chunk slabs
    ((4, 8, 16384, 128), "bf16"),    # 4 MB slabs: several groups, A / B phases interleave
    ((3, 5, 37000, 128), "bf16"),    # 15 slabs of 9.5 MB, ragged last chunk
    ((2, 3, 5000, 64), "f32"),       # f32 rows of 256 bytes, ragged last chunk
    ((1, 2, 100, 256), "f32"),       # rows of 64 16-byte vectors: a warp covers half a row
    ((64, 8, 1000, 128), "f16"),     # 512 small slabs
])
def test_random_vs_oracle(shape, dt):
    rng = np.random.default_rng(hash(shape) % 2**32)
    x = oin.outlier_k(rng, *shape, dtype=dt)
    check_case(x, dt, tag=str(shape))


def test_strided_input_hf_layout():
    """Qwen3 hands the cache [B, H, S, D] views of [B, S, H, D] storage."""
    rng = np.random.default_rng(3)
    B, S, H, D = 2, 300, 8, 128
    x_bshd = oin.outlier_k(rng, B, S, H, D)
    xt = dev(x_bshd, "bf16").transpose(1, 2)
    assert not xt.is_contiguous()
    check_case(np.ascontiguousarray(x_bshd.transpose(0, 2, 1, 3)), "bf16", xt=xt, tag="strided")


def test_write_into_strided_destination():
    rng = np.random.default_rng(4)
    x = oin.normal(rng, (2, 4, 100, 128))
    xt = dev(x, "bf16")
    cap = torch.full((2, 4, 512, 128), 55, dtype=torch.int8, device="cuda")
    vsc = torch.zeros((2, 4, 512, 1), dtype=torch.float16, device="cuda")
    kernels.quant_v_pertoken(xt, out=cap[:, :, 200:300], scale_out=vsc[:, :, 200:300])
    rq, rs = oq.quant_v_pertoken(x)
    c = cap.cpu().numpy()
    np.testing.assert_array_equal(c[:, :, 200:300], rq)
    assert np.all(c[:, :, :200] == 55) and np.all(c[:, :, 300:] == 55)
    np.testing.assert_array_equal(vsc.cpu().numpy()[:, :, 200:300], oq.to_f16(rs))


def test_bulk_write_full_size():
    """Config 4 (B=8, Hkv=8, S=32768, D=128, bf16): oracle on sampled slabs,
    size-independent properties on the whole tensor."""
    B, H, S, D = 8, 8, 32768, 128
    gen = torch.Generator(device="cuda").manual_seed(0)
    k = torch.randn((B, H, S, D), generator=gen, device="cuda", dtype=torch.float32)
    ch = torch.stack([torch.randperm(D, generator=gen, device="cuda")[:4] for _ in range(B * H)])
    gain = torch.ones((B * H, D), device="cuda").scatter_(1, ch, 20.0).view(B, H, 1, D)
    k = (k * gain).to(torch.bfloat16)
    v = torch.randn((B, H, S, D), generator=gen, device="cuda").to(torch.bfloat16)
    for x, fn, dim in ((k, kernels.quant_k_perchannel, 2), (v, kernels.quant_v_pertoken, 3)):
        q, s32 = fn(x, scale_dtype=torch.float32)
        # property 1: scale == IEEE(amax / 127) everywhere
        amax = x.float().abs().amax(dim=dim, keepdim=True).clamp(min=1e-8)
        sref = amax / torch.full((), 127.0, device="cuda")
        assert torch.equal(s32.view(sref.shape), sref)
        # property 2: codes == rint(IEEE(x / scale)) everywhere (elementwise device divide)
        cref = torch.round(x.float() / sref).clamp(-127, 127).to(torch.int8)
        assert torch.equal(q, cref)
        # property 3: the element holding amax codes to +-127 in every row / column
        assert int(q.abs().amax(dim=dim).min()) == 127
        # oracle on sampled slabs
        for b, h in ((0, 0), (3, 5), (7, 7)):
            xs = x[b:b + 1, h:h + 1].float().cpu().numpy()
            rq, rs = oq.quantize_int8(xs, (dim,))
            np.testing.assert_array_equal(q[b:b + 1, h:h + 1].cpu().numpy(), rq)
            np.testing.assert_array_equal(s32[b:b + 1, h:h + 1].cpu().numpy().reshape(rs.shape), rs)
        del q, s32, cref, amax, sref
    assert kernels.read_status("quant_k") == 0


def test_dequant_matches_reference_read_path():
    rng = np.random.default_rng(6)
    x = oin.outlier_k(rng, 2, 2, 70, 128)
    q, s = oq.quant_k_perchannel(x)
    s16 = oq.to_f16(s)
    qt = torch.from_numpy(q).cuda()
    st = torch.from_numpy(s16).cuda()
    out = kernels.dequant(qt, st, torch.bfloat16, per_channel=True)
    ref = oq.cast(q.astype(np.float32) * s16.astype(np.float32), "bf16")
    np.testing.assert_array_equal(out.float().cpu().numpy(), ref)
    qv, sv = oq.quant_v_pertoken(x)
    out = kernels.dequant(torch.from_numpy(qv).cuda(), torch.from_numpy(sv).cuda(), torch.float32,
                          per_channel=False)
    np.testing.assert_array_equal(out.cpu().numpy(), qv.astype(np.float32) * sv)
