"""ctypes binding of ``libgdn_b200.so`` (the C ABI in ``include/gdn_b200.h``).

The library is built in-tree by ``python -m gdn_kernel_b200.build``.  There is
no fallback: if the library is missing or fails to load, every entry point
raises, so a run can never silently measure or check anything but the CUDA
kernels.
"""

from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libgdn_b200.so")
TVM_DECODE_PATH = os.path.join(_PKG, "libgdn_b200_tvm_decode.so")
TVM_PREFILL_PATH = os.path.join(_PKG, "libgdn_b200_tvm_prefill.so")

GDN_B200_OK = 0
GDN_B200_ERR_INVALID_ARGUMENT = 1
GDN_B200_ERR_CUDA = 2

STATUS_TMA_TIMEOUT = 1
STATUS_MMA_TIMEOUT = 2
STATUS_BAD_SEQLENS = 4
STATUS_BAD_INDEX = 8
STATUS_SELFTEST_WAIT = 16

# Every symbol the header declares, with its ctypes signature.
_P = ctypes.c_void_p
_SIGNATURES = {
    "gdn_b200_decode": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_double, _P, _P,
                                       ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_int32, _P]),
    "gdn_b200_decode_pool": (ctypes.c_int, [_P, _P, _P, _P, _P, ctypes.c_int32, _P, _P,
                                            ctypes.c_int32, _P, _P, _P, _P, _P, ctypes.c_double,
                                            _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P]),
    "gdn_b200_prefill": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_int32,
                                        ctypes.c_double, _P, _P, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P]),
    "gdn_b200_prefill_fused": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_int32,
                                              ctypes.c_double, _P, _P, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, _P]),
    "gdn_b200_prefill_workspace_size": (ctypes.c_uint64, [ctypes.c_int64, ctypes.c_int64,
                                                         ctypes.c_int32]),
    "gdn_b200_prefill_ws": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_int32,
                                           ctypes.c_double, _P, _P, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                           ctypes.c_int32, _P, ctypes.c_uint64, _P]),
    "gdn_b200_prefill_static": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P,
                                               ctypes.c_int32, ctypes.c_double, _P, _P,
                                               ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                               ctypes.c_int32, ctypes.c_int32, _P]),
    "gdn_b200_prefill_prepare": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, ctypes.c_int32,
                                                ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                                ctypes.c_int32, ctypes.c_int32, _P,
                                                ctypes.c_uint64, _P]),
    "gdn_b200_prefill_recur": (ctypes.c_int, [_P, _P, _P, ctypes.c_double, _P, _P,
                                              ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_int32, _P, ctypes.c_uint64,
                                              _P]),
    "gdn_b200_state_affine": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int64, _P]),
    "gdn_b200_current_device": (ctypes.c_int32, []),
    "gdn_b200_device_status": (ctypes.c_int, [ctypes.c_int32, ctypes.POINTER(ctypes.c_uint32),
                                              ctypes.c_int32]),
    "gdn_b200_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_uint64, _P]),
    "gdn_b200_selftest_prefill_abort": (ctypes.c_int, [ctypes.c_uint64, _P, _P, _P, _P, _P,
                                                       ctypes.c_int64, ctypes.c_int64,
                                                       ctypes.c_int32, ctypes.c_int32,
                                                       ctypes.c_int32, _P, ctypes.c_uint64, _P]),
    "gdn_b200_last_error": (ctypes.c_char_p, []),
    "gdn_b200_abi_version": (ctypes.c_int32, []),
}

_lock = threading.Lock()
_lib = None


class GdnError(RuntimeError):
    """A CUDA-side failure reported by the library."""


def load() -> ctypes.CDLL:
    """Load the library once; raise if it is absent (no fallback path exists)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m gdn_kernel_b200.build`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int) -> None:
    if rc == GDN_B200_OK:
        return
    msg = load().gdn_b200_last_error().decode()
    if rc == GDN_B200_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise GdnError(msg)


def device_status(device: int, clear: bool = True) -> int:
    """Synchronise ``device`` and read (optionally clear) the kernels' status bits."""
    out = ctypes.c_uint32(0)
    check(load().gdn_b200_device_status(int(device), ctypes.byref(out), 1 if clear else 0))
    return int(out.value)
