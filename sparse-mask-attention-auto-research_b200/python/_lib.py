"""ctypes binding of libsma.so (declared in include/sma_capi.h).

The library is loaded on first use.  There is deliberately no fallback: if
libsma.so is missing or cannot be loaded, every entry point raises
RuntimeError instead of silently computing something else.
"""

import ctypes
import os
import threading

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("SMA_LIBRARY", os.path.join(_PKG_ROOT, "libsma.so"))

# Status codes (include/sma_capi.h).
SMA_OK = 0
SMA_ERR_ARG = 1
SMA_ERR_DTYPE = 2
SMA_ERR_UNSUPPORTED_D = 3
SMA_ERR_LAUNCH = 4
SMA_ERR_TIMEOUT = 5
SMA_ERR_UNSUPPORTED_N = 6
SMA_ERR_CUDA = 7

SMA_DTYPE_FP16 = 0
SMA_DTYPE_BF16 = 1
SMA_MAX_SEQ_LEN = 65536
SMA_MAX_SEQ_LEN_OCCUPANCY = 8192

# Every symbol include/sma_capi.h declares, with (restype, argtypes).
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
SIGNATURES = {
    "sma_pack_mask": (ctypes.c_int, [_vp, _vp, _i64, _i64, _i64, _vp]),
    "sma_attn_fwd": (
        ctypes.c_int,
        [ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_float, _vp],
    ),
    "sma_attn_fwd_mask": (
        ctypes.c_int,
        [ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_float, _vp],
    ),
    "sma_pack_mask_occupancy": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "sma_attn_fwd_occupancy": (
        ctypes.c_int,
        [ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_float, _vp],
    ),
    "sma_attn_bwd": (
        ctypes.c_int,
        [ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
         ctypes.c_float, _vp],
    ),
    "sma_attn_bwd_noalloc": (
        ctypes.c_int,
        [ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_float, _vp],
    ),
    "sma_device_status": (ctypes.c_int, [_vp, ctypes.c_int]),
    "sma_set_wait_timeout_ns": (ctypes.c_int, [ctypes.c_uint64]),
    "sma_debug_wait_probe": (ctypes.c_int, [ctypes.c_uint64, _vp]),
    "sma_last_error": (ctypes.c_char_p, []),
    "sma_abi_version": (ctypes.c_int, []),
}

_lock = threading.Lock()
_lib = None


class SmaError(RuntimeError):
    """A libsma.so entry point returned a non-zero status."""

    def __init__(self, code, message):
        super().__init__(f"[sma status {code}] {message}")
        self.code = code


def load():
    """Load libsma.so once and return the ctypes handle."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libsma.so not found at {LIB_PATH}; build it with "
                "`python sparse-mask-attention-auto-research_b200/build.py` (there is no CPU fallback)"
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(code):
    """Raise SmaError for a non-zero status."""
    if code != SMA_OK:
        msg = load().sma_last_error()
        raise SmaError(code, msg.decode() if msg else "unknown error")
