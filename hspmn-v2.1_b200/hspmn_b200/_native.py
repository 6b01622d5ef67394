"""ctypes binding of libhspmn_sm100.so (C ABI in include/hspmn_sm100.h).

The library is loaded from this package directory only; there is no other
implementation to fall back to, so every entry point raises when the library
is missing or the device is not a B200.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_NAME = "libhspmn_sm100.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

HSPMN_F32, HSPMN_F16, HSPMN_BF16 = 0, 1, 2
DEVERR_POSITION, DEVERR_UNSORTED, DEVERR_TIMEOUT = 1, 2, 4

# name -> (restype, argtypes)
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_int = ctypes.c_int
_SIGNATURES = {
    "hspmn_version": (_int, []),
    "hspmn_strerror": (ctypes.c_char_p, [_int]),
    "hspmn_router_topk": (_int, [_vp, _int, _i64, _vp, _int, _int, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _vp]),
    "hspmn_gate_logits": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp]),
    "hspmn_gather_rows": (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "hspmn_scatter_rows": (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "hspmn_sqdk_fwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp,
                              _i64, _i64, _i64, _i64, _i64, _i64, _int, ctypes.c_float,
                              _vp, ctypes.c_size_t, _vp]),
    "hspmn_sqdk_workspace_size": (_i64, [_i64, _i64, _i64, _i64, _i64, _i64]),
    "hspmn_sqdk_fwd_noalloc": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp,
                                      _i64, _i64, _i64, _i64, _i64, _i64, _int, ctypes.c_float, _vp]),
    "hspmn_sqdk_fwd_lse": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _i64,
                                  _i64, _i64, _i64, _i64, _i64, _i64, _int, ctypes.c_float,
                                  _vp, ctypes.c_size_t, _vp]),
    "hspmn_sqdk_bwd_workspace_size": (_i64, [_i64, _i64, _i64, _i64]),
    "hspmn_sqdk_bwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                              _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _int,
                              ctypes.c_float, _vp, ctypes.c_size_t, _vp]),
    "hspmn_rope_gather_rows": (_int, [_vp, _i64, _i64, _int, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64,
                                      _i64, _i64, _i64, _i64, _i64, _int, _vp]),
    "hspmn_rope_rows": (_int, [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64,
                               _i64, _int, _vp]),
    "hspmn_scatter_add_rows": (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                                      _int, _vp]),
    "hspmn_device_errors": (_int, [ctypes.POINTER(ctypes.c_uint), _int, _vp]),
}
EXPORTED = tuple(_SIGNATURES)

_lib = None
_lock = threading.Lock()


class HSPMNNativeError(RuntimeError):
    """A library entry point returned a non-zero status."""


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_NAME} is not built (expected at {LIB_PATH}); run "
                    "`python hspmn-v2.1_b200/build_native.py` on a machine with the CUDA toolkit")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def strerror(status: int) -> str:
    return lib().hspmn_strerror(int(status)).decode()


def check(status: int, what: str) -> None:
    if status != 0:
        raise HSPMNNativeError(f"{what} failed: {strerror(status)} (status {status})")


def device_errors(stream: int = 0, clear: bool = True) -> int:
    """Synchronise ``stream`` and return the device flag word (DEVERR_* bits)."""
    bits = ctypes.c_uint(0)
    check(lib().hspmn_device_errors(ctypes.byref(bits), int(clear), ctypes.c_void_p(stream)),
          "hspmn_device_errors")
    return int(bits.value)


def i64_array(vals):
    arr = (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])
    return arr
