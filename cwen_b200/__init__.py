"""ctypes binding of the cwen B200 engine (include/cwen_cuda.h).

The engine is native: CUDA kernels for sm_100a and a C host side, all in
cwen_b200/libcwen_cuda.so.  This module only loads that library and declares
its C ABI for tests and bench.py; there is no Python or CPU fallback, and
`lib()` raises if the library is missing.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libcwen_cuda.so"

CWEN_T_F32, CWEN_T_Q4_0, CWEN_T_Q8_0 = 0, 2, 8


class Dims(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "n_embd", "n_ff", "n_vocab", "n_layer", "n_head", "n_head_kv", "head_dim", "n_rot",
        "ssm_n_kh", "ssm_n_vh", "ssm_d", "conv_k", "full_interval", "has_mtp")]


class CwenError(RuntimeError):
    pass


_lib = None

# name -> (restype, argtypes)
_SIGS = {
    "cwen_cuda_last_error": (C.c_char_p, []),
    "cwen_cuda_init": (C.c_int, [C.c_int, C.c_int, C.c_int]),
    "cwen_cuda_shutdown": (None, []),
    "cwen_cuda_weight_upload": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "cwen_cuda_gemvb": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "cwen_cuda_gemvb_host": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int]),
    "cwen_cuda_profile": (C.c_int, [C.c_int]),
    "cwen_cuda_profile_read": (C.c_int, [C.POINTER(C.c_double), C.POINTER(C.c_double),
                                         C.POINTER(C.c_longlong), C.POINTER(C.c_longlong)]),
}


def lib() -> C.CDLL:
    """Load libcwen_cuda.so (build it with `python cwen_b200/build.py`)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise CwenError(f"{LIB_PATH} is missing: the engine is CUDA-only, build it first")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int, what: str = "cwen") -> None:
    if rc != 0:
        raise CwenError(f"{what}: rc={rc}: {lib().cwen_cuda_last_error().decode()}")


def ptr(a) -> C.c_void_p:
    """Address of a numpy array's data (or a torch tensor's device data)."""
    if hasattr(a, "data_ptr"):
        return C.c_void_p(a.data_ptr())
    return a.ctypes.data_as(C.c_void_p)
