"""ctypes binding of ``libhalftone_b200.so`` (C ABI: ``include/halftone_b200.h``).

The shared library is built in-tree by ``halftone_quantizedkvcache_b200.csrc.build``
(nvcc, sm_100a).  There is no fallback: if the library is missing or cannot be
loaded, every op raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import functools
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhalftone_b200.so")

DTYPE_F32, DTYPE_BF16, DTYPE_F16, DTYPE_I8 = 0, 1, 2, 3
OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_DEVICE_TIMEOUT = 0, -1, -2, -3, -4

_i64_4 = ctypes.c_int64 * 4
_i64_3 = ctypes.c_int64 * 3
_P = ctypes.c_void_p
_I = ctypes.c_int
_Z = ctypes.c_size_t
_F = ctypes.c_float
_A4 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes), in the order of include/halftone_b200.h
SIGNATURES = {
    "hq_status_string": (ctypes.c_char_p, [_I]),
    "hq_version": (ctypes.c_char_p, []),
    "hq_quant_k_workspace_bytes": (_Z, [_I, _I, _I]),
    "hq_quant_k_perchannel": (_I, [_P, _I, _A4, _I, _I, _I, _I, _P, _A4, _P, _P, _P, _Z, _P]),
    "hq_quant_v_pertoken": (_I, [_P, _I, _A4, _I, _I, _I, _I, _P, _A4, _P, _P, _A4, _P]),
    "hq_append_kv": (_I, [_P, _P, _I, _A4, _A4, _I, _I, _I, _I, _P, _A4, _P, _A4, _P, _P, _A4, _P]),
    "hq_quant_k_static": (_I, [_P, _I, _A4, _I, _I, _I, _I, _P, _I, _A4, _P, _A4, _P]),
    "hq_append_kv_static": (_I, [_P, _P, _I, _A4, _A4, _I, _I, _I, _I, _P, _I, _A4, _P, _A4, _P,
                                 _A4, _P, _P, _A4, _P]),
    "hq_column_absmax": (_I, [_P, _I, _A4, _I, _I, _I, _I, _P, _P]),
    "hq_k_scale_from_amax": (_I, [_P, _I, _P, _P, _P]),
    "hq_dequant": (_I, [_P, _A4, _I, _I, _I, _I, _P, _I, _A4, _I, _P, _I, _A4, _P]),
    "hq_decode_workspace_bytes": (_Z, [_I, _I, _I, _I, _I]),
    "hq_decode_int8": (_I, [_P, _I, _A4, _P, _P, _A4, _P, _P, _I, _A4, _A4, _I, _I, _I, _I, _I,
                            _F, _I, _P, _A4, _P, _P, _Z, _P]),
    "hq_decode_int8_ex": (_I, [_P, _I, _A4, _P, _P, _A4, _P, _P, _I, _A4, _A4, _I, _I, _I, _I, _I,
                               _F, _I, _P, _A4, _P, _P, _Z, ctypes.c_uint, _P]),
    "hq_prefill_int8": (_I, [_P, _I, _A4, _P, _P, _A4, _P, _P, _I, _A4, _A4, _I, _I, _I, _I, _I, _I,
                             _F, _I, _P, _A4, _P, _P]),
    "hq_decode_dense": (_I, [_P, _A4, _P, _P, _I, _A4, _I, _I, _I, _I, _I, _F, _I, _P, _A4, _P, _P,
                             _Z, _P]),
    "hq_decode_dense_fma": (_I, [_P, _A4, _P, _P, _I, _A4, _I, _I, _I, _I, _I, _F, _I, _P, _A4, _P,
                                 _P, _Z, _P]),
    "hq_decode_combine": (_I, [_P, _I, ctypes.c_int64, _I, _I, _I, _P, _I, _A4, _P]),
    "hq_decode_int8_noalloc": (_I, [_P, _I, _A4, _P, _P, _A4, _P, _P, _I, _A4, _A4, _I, _I, _I, _I,
                                    _I, _F, _I, _P, _A4, _P, _P]),
    "hq_append_kv_at": (_I, [_P, _P, _I, _A4, _A4, _I, _I, _I, _I, _P, _A4, _P, _A4, _P, _P, _A4,
                             _I, _P, _P]),
    "hq_decode_int8_len": (_I, [_P, _I, _A4, _P, _P, _A4, _P, _P, _I, _A4, _A4, _I, _I, _I, _I, _P,
                                _I, _I, _F, _I, _P, _A4, _P, _Z, _P]),
    "hq_decode_append_int8_len": (_I, [_P, _I, _A4, _P, _P, _A4, _A4, _P, _P, _A4, _P, _P, _I, _A4,
                                       _A4, _I, _I, _I, _I, _P, _I, _I, _F, _I, _P, _A4, _P, _Z,
                                       _P]),
    "hq_peer_buffer_bytes": (_Z, [_I, _I, _I, _I]),
    "hq_peer_alloc": (_I, [_Z, ctypes.POINTER(ctypes.c_void_p), _P]),
    "hq_peer_open": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "hq_peer_close": (_I, [_P]),
    "hq_peer_free": (_I, [_P]),
    "hq_decode_int8_peer": (_I, [_P, _I, _A4, _P, _P, _A4, _P, _P, _I, _A4, _A4, _I, _I, _I, _I, _I,
                                 _F, _I, _P, _A4, _P, _Z, ctypes.POINTER(ctypes.c_void_p), _I, _I,
                                 _P]),
    "hq_kblock_write": (_I, [_P, _P, _I, _A4, _A4, _I, _I, _I, _I, _I, _I, _P, _A4, _P, _A4, _P,
                             _A4, _P, _A4, _P, _P, _A4, _I, _P]),
    "hq_kblock_decode_workspace_bytes": (_Z, [_I, _I, _I, _I, _I]),
    "hq_kblock_decode": (_I, [_P, _I, _A4, _P, _A4, _P, _A4, _P, _A4, _P, _I, _A4, _I, _I, _I, _I,
                              _I, _I, _F, _P, _A4, _P, _Z, _P]),
    "hq_kblock_write_at": (_I, [_P, _P, _I, _A4, _A4, _I, _I, _I, _I, _P, _A4, _P, _A4, _P, _A4,
                                _P, _A4, _P, _P, _A4, _I, _P, _P]),
    "hq_kblock_decode_len": (_I, [_P, _I, _A4, _P, _A4, _P, _A4, _P, _A4, _P, _I, _A4, _I, _I, _I,
                                  _I, _P, _I, _I, _I, _F, _P, _A4, _P, _Z, _P]),
    "hq_kblock_dequant": (_I, [_P, _A4, _P, _A4, _I, _I, _I, _I, _I, _P, _I, _A4, _P]),
    "hq_read_status": (_I, [_P, _P]),
    "hq_set_plan_sms": (_I, [_I, _I]),
}

_lib = None
_lock = threading.Lock()


class HalftoneError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, what: str, status: int):
        self.status = status
        super().__init__(f"{what} failed: {status_string(status)} (status {status})")


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with "
                    "`python -m halftone_quantizedkvcache_b200.csrc.build` (needs nvcc)")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def status_string(status: int) -> str:
    return lib().hq_status_string(int(status)).decode()


def check(status: int, what: str) -> None:
    if status != OK:
        raise HalftoneError(what, status)


@functools.lru_cache(maxsize=8192)
def _strides_cached(seq: tuple, n: int) -> ctypes.Array:
    arr = (_i64_4 if n == 4 else _i64_3)()
    for i, v in enumerate(seq):
        arr[i] = int(v)
    return arr


def strides(seq, n) -> ctypes.Array:
    """Element strides as a C ``int64_t[n]`` (shared per value: the library only reads them)."""
    return _strides_cached(seq if type(seq) is tuple else tuple(seq), n)
