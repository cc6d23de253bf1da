"""The C-ABI library loads on a host without a GPU and exports every entry
point that include/halftone_b200.h declares; host-only calls behave."""
import ctypes
import os
import re

import pytest

from halftone_quantizedkvcache_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "halftone_b200.h")


def declared():
    text = open(HEADER).read()
    return re.findall(r"^HQ_API\s+[\w\s\*]+?\b(hq_\w+)\s*\(", text, flags=re.M)


def test_header_declares_entry_points():
    names = declared()
    assert len(names) == len(set(names)) >= 12
    assert set(names) == set(_lib.SIGNATURES), "ctypes table and header disagree"


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared():
        assert hasattr(lib, name), name


def test_status_strings_and_version():
    assert _lib.lib().hq_version().decode().count(".") == 2
    for code in (0, -1, -2, -3, -4):
        assert _lib.status_string(code)
    assert "unknown" in _lib.status_string(-99)


def test_workspace_queries():
    L = _lib.lib()
    assert L.hq_quant_k_workspace_bytes(8, 8, 128) >= 8 * 8 * 128 * 4
    assert L.hq_decode_workspace_bytes(1, 16, 8, 32768, 128) > 0
    assert L.hq_decode_workspace_bytes(1, 16, 8, 32768, 64) == 0   # head_dim not compiled in
    assert L.hq_decode_workspace_bytes(1, 16, 0, 32768, 128) == 0


def test_argument_errors_return_before_any_launch():
    L = _lib.lib()
    st4 = _lib.strides((0, 0, 0, 1), 4)
    st3 = _lib.strides((0, 0, 1), 3)
    # null pointers
    assert L.hq_quant_v_pertoken(None, 1, st4, 1, 1, 1, 128, None, st4, None, None, None, None) == -1
    assert L.hq_quant_k_perchannel(None, 1, st4, 1, 1, 1, 128, None, st4, None, None, None, 0,
                                   None) == -1
    # unsupported dtype code
    assert L.hq_quant_v_pertoken(16, 9, st4, 1, 1, 1, 128, 16, st4, None, None, None, None) == -2
    # S = 0 is rejected (the reference's amax over an empty axis raises)
    assert L.hq_quant_v_pertoken(16, 1, st4, 1, 1, 0, 128, 16, st4, None, None, None, None) == -1
    # decode: head_dim other than 128, group size not a divisor
    kv = _lib.strides((0, 0, 128), 3)
    args = [16, 1, st3, 16, 16, kv, 16, 16, 0, st3, st3, 1, 16, 8, 64, 64, 0.1, 0, 16, st3, None,
            256, 1 << 20, None]
    assert L.hq_decode_int8(*args) == -2
    args[12], args[13], args[15] = 12, 8, 128
    assert L.hq_decode_int8(*args) == -2
    # missing / misaligned workspace
    args[12] = 16
    args[21] = None
    assert L.hq_decode_int8(*args) == -3
    args[21] = 260
    assert L.hq_decode_int8(*args) == -3


def test_ops_refuse_cpu_tensors():
    torch = pytest.importorskip("torch")
    from halftone_quantizedkvcache_b200 import kernels
    x = torch.zeros(1, 2, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="no CPU path"):
        kernels.quant_v_pertoken(x)
    with pytest.raises(ValueError, match="no CPU path"):
        kernels.quant_k_perchannel(x)
    q = torch.zeros(16, 1, 128, dtype=torch.bfloat16)
    k = torch.zeros(8, 4, 128, dtype=torch.int8)
    s = torch.zeros(8, 1, 128, dtype=torch.float16)
    with pytest.raises(ValueError, match="no CPU path"):
        kernels.int8_decode_attn(q, k, s, k, s, 2)


def test_missing_library_fails_loudly(monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libhalftone_b200.so")
    with pytest.raises(RuntimeError, match="missing"):
        _lib.lib()


def test_peer_buffer_layout():
    """gen [B*Hkv] u32 padded to 256 bytes | part [2][world][B*Hq][D+4] u64 words."""
    L = _lib.lib()
    a256 = lambda n: (n + 255) // 256 * 256  # noqa: E731
    for world, B, Hq, Hkv in ((1, 1, 16, 8), (2, 1, 16, 8), (8, 4, 32, 8), (3, 5, 8, 8)):
        want = a256(4 * B * Hkv) + 8 * 2 * world * B * Hq * 132
        assert L.hq_peer_buffer_bytes(world, B, Hq, Hkv) == want
    assert L.hq_peer_buffer_bytes(0, 1, 16, 8) == 0
    assert L.hq_peer_buffer_bytes(9, 1, 16, 8) == 0
    assert L.hq_peer_buffer_bytes(2, 0, 16, 8) == 0


def test_peer_argument_errors_return_before_any_launch():
    L = _lib.lib()
    st3 = _lib.strides((0, 0, 1), 3)
    kv = _lib.strides((0, 0, 128), 3)
    bufs = (ctypes.c_void_p * 8)(*([256] * 8))
    base = [16, 1, st3, 16, 16, kv, 16, 16, 0, st3, st3, 1, 16, 8, 64, 128, 0.1, 0, 16, st3,
            256, 1 << 20]
    for world, rank in ((0, 0), (9, 0), (2, 2), (2, -1)):
        assert L.hq_decode_int8_peer(*base, bufs, world, rank, None) == -1
    assert L.hq_decode_int8_peer(*base, None, 2, 0, None) == -1
    bad = (ctypes.c_void_p * 2)(256, 320)              # second buffer not 256-byte aligned
    assert L.hq_decode_int8_peer(*base, bad, 2, 0, None) == -1
    no_out = list(base)
    no_out[18] = None
    assert L.hq_decode_int8_peer(*no_out, bufs, 2, 0, None) == -1
    assert L.hq_peer_alloc(0, ctypes.byref(ctypes.c_void_p()), (ctypes.c_char * 64)()) == -1
    assert L.hq_peer_open(None, ctypes.byref(ctypes.c_void_p())) == -1
