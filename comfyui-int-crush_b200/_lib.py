"""ctypes binding of ``libintcrush_b200.so`` (the C ABI in include/intcrush_b200.h).

The shared library is built in place by ``build.py`` and loaded from this
directory.  There is no fallback: if the library is missing or fails to load,
``lib()`` raises, and every op of ``_b200_runtime`` raises with it.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("INTCRUSH_LIB") or os.path.join(_HERE, "libintcrush_b200.so")

IC_OK = 0
IC_ERR_ARG = 1
IC_ERR_UNSUPPORTED = 2
IC_ERR_CUDA = 3

IC_DTYPE_F16 = 0
IC_DTYPE_BF16 = 1
IC_DTYPE_F32 = 2

IC_W_INT8 = 0
IC_W_INT4 = 1
IC_W_INT4R = 2

IC_DEV_ERR_TIMEOUT = 1

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float

# name -> argument types (all return int status except where noted)
SIGNATURES: dict[str, list] = {
    "ic_version": [],
    "ic_last_error": [],
    "ic_read_device_error": [_I, ctypes.POINTER(_I)],
    "ic_prep_quant": [_P, _I, _L, _L, _L, _P, _I, _L, _P, _P, _P, _L, _P, _P, _P, _P],
    "ic_prep_quant_norm": [_P, _I, _L, _L, _L, _I, _P, _P, _F, _P, _I, _L, _P, _P, _L, _P, _P, _P, _P],
    "ic_dynamic_quantize": [_P, _I, _L, _L, _L, _P, _L, _P, _P],
    "ic_gemm_a8": [_P, _L, _L, _L, _P, _I, _L, _L, _P, _L, _L, _P, _P, _I, _P, _P, _P, _I, _L, _P],
    "ic_gemm_a8_splitk": [_P, _L, _L, _L, _P, _I, _L, _L, _P, _L, _L, _P, _P, _I, _P, _P, _P, _I, _L, _I, _P, _L, _P],
    "ic_gemm_a8_splitk_noalloc": [_P, _L, _L, _L, _P, _I, _L, _L, _P, _L, _L, _P, _P, _I, _P, _P, _P, _I, _L, _I, _P],
    "ic_gemm_a8_ex": [_P, _L, _L, _L, _P, _I, _L, _L, _P, _L, _L, _P, _P, _I, _P, _P, _I, _P, _I, _L, _P, _I, _L, _I,
                      _P, _L, _P],
    "ic_quantize_weight": [_P, _L, _L, _L, _I, _P, _L, _P, _P],
    "ic_lokr_add": [_P, _I, _L, _L, _P, _L, _L, _P, _L, _L, _P, _L, _L, _F, _P, _L, _P],
    "ic_gemm_a8_int8out": [_P, _L, _L, _L, _P, _I, _L, _L, _P, _L, _L, _P, _P, _I, _I, _P, _L, _P, _P, _L, _P],
    "ic_gemm_w4a16": [_P, _I, _L, _L, _L, _P, _L, _L, _I, _P, _I, _L, _L, _P, _I, _P, _P, _L, _F, _P, _L, _P],
    "ic_gemm_w4a16_splitk": [_P, _I, _L, _L, _L, _P, _L, _L, _I, _P, _I, _L, _L, _P, _I, _P, _P, _L, _F, _P, _L,
                             _I, _P, _L, _P],
    "ic_repack_int4": [_P, _L, _L, _L, _P, _L, _I, _P],
    "ic_lowrank_down": [_P, _L, _L, _L, _P, _L, _P, _P],
    "ic_lowrank_down_ex": [_P, _I, _L, _L, _L, _P, _L, _P, _P],
    "ic_lowrank_add": [_P, _L, _L, _L, _P, _P, _L, _F, _P],
    "ic_lowrank_add_ex": [_P, _I, _L, _L, _L, _P, _P, _L, _F, _P],
    "ic_unpack_int4_to_int8": [_P, _L, _L, _L, _P, _P],
    "ic_selftest_wait_timeout": [_L, _P],
    "ic_unpack_int4_to_f16": [_P, _L, _L, _L, _P, _I, _L, _L, _P, _P],
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class IntCrushError(RuntimeError):
    """A non-zero status from the C ABI."""


def lib() -> ctypes.CDLL:
    """Load (once) and return the library.  Raises OSError when it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise OSError(
                    f"{LIB_PATH} is missing: build it with `python build.py` "
                    "in the package directory (nvcc, sm_100a)")
            L = ctypes.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = ctypes.c_char_p if name == "ic_last_error" else ctypes.c_int
            _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != IC_OK:
        msg = lib().ic_last_error().decode(errors="replace")
        kind = {IC_ERR_ARG: "bad argument", IC_ERR_UNSUPPORTED: "unsupported",
                IC_ERR_CUDA: "CUDA error"}.get(status, f"status {status}")
        if status == IC_ERR_ARG:
            raise ValueError(f"{what}: {kind}: {msg}")
        raise IntCrushError(f"{what}: {kind}: {msg}")


def read_device_error(clear: bool = True) -> int:
    """Device error word (1 = a bounded wait timed out).  Synchronises."""
    code = ctypes.c_int(0)
    check(lib().ic_read_device_error(1 if clear else 0, ctypes.byref(code)), "ic_read_device_error")
    return code.value
