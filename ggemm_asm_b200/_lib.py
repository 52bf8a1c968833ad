"""ctypes binding of libggemm_vark.so (the C ABI in include/ggemm_vark.h).

Loading fails loudly: there is no Python or CPU fallback for the product path. If the
library is missing, build it with ``python -m ggemm_asm_b200.build``.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libggemm_vark.so"

# Status codes (GGEMM_VARK_*), mirrored from the header.
OK = 0
EINVAL_PTR = 1
EINVAL_SHAPE = 2
EINVAL_STRIDE = 3
EINVAL_ARG = 4
ENO_DEVICE = 5
ECUDA = 6
ELAYOUT = 7
ETOO_LARGE = 8

DEV_BAD_OFFS = 0x1
DEV_TIMEOUT = 0x2

# Status block words (GGEMM_VARK_STATUS_WORD_*).
STATUS_WORD_BITS = 0
STATUS_WORD_SITE = 1
STATUS_WORD_LHS_ROWS = 4
STATUS_WORD_RHS_ROWS = 5

PATH_AUTO = 0
PATH_TCGEN05 = 1
PATH_SIMT = 2
PATH_TCGEN05_1SM = 3

# Every function the header declares, with its ctypes signature.
_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
SIGNATURES = {
    "ggemm_vark_fp8_wgrad": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                                            _i32, _i32, _i32, _i32, _i32, _vp]),
    "ggemm_vark_fp8_wgrad_ex": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                                               _i32, _i32, _i32, _i32, _i32, _i64, _i32, _i32,
                                               _vp, _u64, _vp]),
    "ggemm_vark_fp8_wgrad_noalloc": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32,
                                                    _i32, _i32, _i32, _i32, _i32, _i32, _i64,
                                                    _i32, _vp, _vp]),
    "ggemm_vark_grouped_fp8_fwd": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                                                  _i32, _i32, _i32, _i32, _i32, _vp]),
    "ggemm_vark_grouped_fp8_fwd_ex": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32,
                                                     _i32, _i32, _i32, _i32, _i32, _i32, _i64,
                                                     _i32, _i32, _i32, _vp, _u64, _vp]),
    "ggemm_vark_quantize_workspace_bytes": (ctypes.c_size_t, [_i32]),
    "ggemm_vark_quantize_fp8": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
                                               _i32, _i64, _vp, _vp, _u64, _vp]),
    "ggemm_vark_read_status": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.POINTER(ctypes.c_uint32)]),
    "ggemm_vark_read_status_stream": (ctypes.c_int, [_vp, ctypes.c_int,
                                                     ctypes.POINTER(ctypes.c_uint32), _i32, _vp]),
    "ggemm_vark_device_bytes": (ctypes.c_int, [_i32, ctypes.POINTER(ctypes.c_uint64)]),
    "ggemm_vark_tc_supported": (ctypes.c_int, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32,
                                               _i32]),
    "ggemm_vark_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "ggemm_vark_last_cuda_error": (ctypes.c_int, []),
    "ggemm_vark_version": (ctypes.c_int, []),
}

_lock = threading.Lock()
_lib = None


class VarkError(RuntimeError):
    """A GGEMM_VARK_E* status returned by the C ABI."""

    def __init__(self, code: int, what: str):
        self.code = code
        msg = f"{what}: GGEMM_VARK error {code} ({strerror(code)})"
        if code == ECUDA:
            msg += f", cudaError {lib().ggemm_vark_last_cuda_error()}"
        super().__init__(msg)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: the CUDA library is not built "
                    "(run `python -m ggemm_asm_b200.build`)")
            cdll = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(cdll, name)
                fn.restype = res
                fn.argtypes = args
            _lib = cdll
    return _lib


def strerror(code: int) -> str:
    return lib().ggemm_vark_strerror(code).decode()


def check(code: int, what: str) -> None:
    if code != OK:
        raise VarkError(code, what)


def read_status(status_ptr: int | None = None, clear: bool = False) -> int:
    """Synchronously read the device status bits (DEV_*) of a status block (None = library's)."""
    bits = ctypes.c_uint32(0)
    check(lib().ggemm_vark_read_status(status_ptr, 1 if clear else 0, ctypes.byref(bits)),
          "ggemm_vark_read_status")
    return int(bits.value)


def read_status_words(status_ptr: int | None = None, nwords: int = 8, clear: bool = False,
                      stream: int | None = None) -> list[int]:
    """The first `nwords` words of a status block, read in the order of `stream` (None = the
    legacy default stream); only that stream is waited for."""
    words = (ctypes.c_uint32 * 8)()
    check(lib().ggemm_vark_read_status_stream(status_ptr, 1 if clear else 0, words, nwords,
                                              stream),
          "ggemm_vark_read_status_stream")
    return [int(words[i]) for i in range(nwords)]


def device_bytes(device: int) -> int:
    """Device memory the library has allocated on `device` (its status block, once set up)."""
    n = ctypes.c_uint64(0)
    check(lib().ggemm_vark_device_bytes(device, ctypes.byref(n)), "ggemm_vark_device_bytes")
    return int(n.value)
