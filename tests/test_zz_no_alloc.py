"""The decode entry point for callers that cannot allocate device memory.

Some callers of the library cannot allocate GPU memory themselves: a plugin
running inside another engine's decode loop, or a binding whose language
runtime owns the whole device heap, can pass the tensors it holds but cannot
call cudaMalloc for a workspace.  ``hq_decode_int8_noalloc`` serves them with
a static 8 MiB scratch array inside the library.  This test calls it through
the C ABI twice in a row and checks both results against the regular
``hq_decode_int8`` (caller workspace) within the decode tests' tolerance, and
checks that a request larger than the static scratch is refused before any
launch.  The file name sorts last so a ``-x`` run has run every other test
before this one.
"""
import math

import numpy as np
import pytest
import torch

from halftone_quantizedkvcache_b200 import _lib, kernels
from oracle import inputs as oin

pytestmark = pytest.mark.gpu


def _noalloc(q, k8, ks, v8, vs, out, sm_scale, partial_out=None):
    B, Hq, D = q.shape
    _, Hkv, S, _ = k8.shape
    return _lib.lib().hq_decode_int8_noalloc(
        q.data_ptr(), _lib.DTYPE_BF16, _lib.strides(q.stride(), 3), k8.data_ptr(), v8.data_ptr(),
        _lib.strides(k8.stride()[:3], 3), ks.data_ptr(), vs.data_ptr(), _lib.DTYPE_F32,
        _lib.strides((ks.stride(0), ks.stride(1), ks.stride(3)), 3),
        _lib.strides(vs.stride()[:3], 3), B, Hq, Hkv, S, D, sm_scale, 0,
        out.data_ptr() if out is not None else None,
        _lib.strides(out.stride(), 3) if out is not None else None,
        partial_out.data_ptr() if partial_out is not None else None,
        torch.cuda.current_stream().cuda_stream)


def _random_cache(B, Hq, Hkv, S, D=128, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((B, Hq, D), generator=g, device="cuda").bfloat16()
    k8 = torch.randint(-127, 128, (B, Hkv, S, D), generator=g, device="cuda", dtype=torch.int8)
    v8 = torch.randint(-127, 128, (B, Hkv, S, D), generator=g, device="cuda", dtype=torch.int8)
    ks = torch.rand((B, Hkv, 1, D), generator=g, device="cuda") * 0.1
    vs = torch.rand((B, Hkv, S, 1), generator=g, device="cuda") * 0.02
    return q, k8, ks, v8, vs


def test_noalloc_matches_workspace_entry_point():
    c = oin.decode_case(2024, 2, 16, 8, 5000, 128)
    dev = torch.device("cuda")
    q = torch.from_numpy(c["q"]).bfloat16().to(dev)
    k8, v8 = torch.from_numpy(c["k_i8"]).to(dev), torch.from_numpy(c["v_i8"]).to(dev)
    ks, vs = torch.from_numpy(c["k_sc"]).to(dev), torch.from_numpy(c["v_sc"]).to(dev)
    sm = 1.0 / math.sqrt(128)
    ref = kernels.int8_decode_attn(q, k8, ks, v8, vs, 2, sm_scale=sm).float().cpu().numpy()
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        assert _noalloc(q, k8, ks, v8, vs, out, sm) == 0
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=1e-3, rtol=2.0 ** -7)


def test_noalloc_refuses_oversized_request():
    # enough sequences that the split partials exceed the 8 MiB static scratch
    Hq, Hkv, S, D = 64, 8, 65536, 128
    B = 1
    while _lib.lib().hq_decode_workspace_bytes(B, Hq, Hkv, S, D) <= 8 * 2 ** 20:
        B *= 2
    assert B <= 4096
    dummy = torch.empty(256, dtype=torch.uint8, device="cuda")
    p = dummy.data_ptr()
    st3 = _lib.strides((Hq * D, D, 1), 3)
    rc = _lib.lib().hq_decode_int8_noalloc(
        p, _lib.DTYPE_BF16, st3, p, p, _lib.strides((Hkv * S * D, S * D, D), 3), p, p,
        _lib.DTYPE_F32, _lib.strides((Hkv * D, D, 1), 3), _lib.strides((Hkv * S, S, 1), 3), B, Hq,
        Hkv, S, D, 0.1, 0, p, st3, None, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ERR_WORKSPACE


@pytest.mark.parametrize("case", ["just_under_limit", "four_heads_per_kv_head", "one_kv_head"])
def test_noalloc_equals_workspace_entry_point_at_extremes(case):
    """Extremes of the static scratch: the largest batch whose workspace still
    fits in 8 MiB (the scratch's last bytes in use); four q heads per kv head at
    S = 32768 (37 split partial rows per head, the short merge); one kv head at
    S = 32768 (256 splits, the long merge).  Same kernel and plan as
    hq_decode_int8, so the outputs are identical."""
    D = 128
    if case == "just_under_limit":
        Hq, Hkv, S, B = 16, 8, 200, 1
        while _lib.lib().hq_decode_workspace_bytes(B + 1, Hq, Hkv, S, D) <= 8 * 2 ** 20:
            B += 1
        assert _lib.lib().hq_decode_workspace_bytes(B, Hq, Hkv, S, D) > 8 * 2 ** 20 - 16384
    elif case == "four_heads_per_kv_head":
        Hq, Hkv, S, B = 32, 8, 32768, 1
    else:
        Hq, Hkv, S, B = 4, 1, 32768, 1
    q, k8, ks, v8, vs = _random_cache(B, Hq, Hkv, S, D, seed=7)
    sm = 1.0 / math.sqrt(D)
    ref = kernels.int8_decode_attn(q, k8, ks, v8, vs, Hq // Hkv, sm_scale=sm)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        assert _noalloc(q, k8, ks, v8, vs, out, sm) == 0
        torch.cuda.synchronize()
        assert torch.equal(out, ref)


def test_noalloc_partial_out_equals_workspace_entry_point():
    """The (m, l, o) partial output path, twice in a row, against hq_decode_int8's."""
    B, Hq, Hkv, S, D = 3, 16, 8, 9000, 128
    q, k8, ks, v8, vs = _random_cache(B, Hq, Hkv, S, D, seed=11)
    sm = 1.0 / math.sqrt(D)
    ref = torch.empty((B, Hq, D + 2), dtype=torch.float32, device="cuda")
    kernels.int8_decode_attn(q, k8, ks, v8, vs, Hq // Hkv, sm_scale=sm, partial_out=ref)
    for _ in range(2):
        part = torch.full_like(ref, float("nan"))
        assert _noalloc(q, k8, ks, v8, vs, None, sm, partial_out=part) == 0
        torch.cuda.synchronize()
        assert torch.equal(part, ref)


def test_noalloc_argument_errors_enqueue_nothing():
    """Invalid counts are argument errors, refused before any work is enqueued."""
    p = 0
    st3 = _lib.strides((16 * 128, 128, 1), 3)
    kv3 = _lib.strides((8 * 64 * 128, 64 * 128, 128), 3)
    for B, Hq, Hkv, S in ((-1, 16, 8, 64), (1, 0, 8, 64), (1, 16, 0, 64), (1, 16, 8, -1)):
        rc = _lib.lib().hq_decode_int8_noalloc(
            p, _lib.DTYPE_BF16, st3, p, p, kv3, p, p, _lib.DTYPE_F32, st3, st3, B, Hq, Hkv, S, 128,
            0.1, 0, p, st3, None, torch.cuda.current_stream().cuda_stream)
        assert rc == _lib.ERR_INVALID_ARGUMENT, (B, Hq, Hkv, S, rc)
