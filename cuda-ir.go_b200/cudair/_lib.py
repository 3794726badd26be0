"""Loads libcudair_b200.so (built in-tree by cuda-ir.go_b200/build.py) and
declares the ctypes signature of every entry point of include/cudair_b200.h.

There is no fallback: if the library is missing, importing the wrapper fails
with an error naming the build command.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcudair_b200.so")
CUBIN_PATH = os.path.join(HERE, "cudair_kernels.cubin")
HEADER_PATH = os.path.join(os.path.dirname(os.path.dirname(HERE)), "include", "cudair_b200.h")

_lib = None

c_int, c_u32, c_u64, c_i64, c_size, c_vp = (ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64,
                                           ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_u32p = ctypes.POINTER(ctypes.c_uint32)

SIGNATURES = {
    "cudair_last_error": (ctypes.c_char_p, []),
    "cudair_version": (ctypes.c_char_p, []),
    "cudair_encode_tiled": (c_int, [c_vp, c_u32, c_u32, c_u64, _u64p, _u64p, c_u32, _u32p, c_u32,
                                    _u32p, c_u32, c_u32, c_u32, c_u32, c_u32, c_u32]),
    "cudair_module_load": (c_int, [c_vp, c_size, ctypes.POINTER(c_vp)]),
    "cudair_module_unload": (c_int, [c_vp]),
    "cudair_module_function": (c_int, [c_vp, ctypes.c_char_p, ctypes.POINTER(c_vp)]),
    "cudair_launch_ex": (c_int, [c_vp, _u32p, _u32p, c_u32, c_vp, _u32p, c_int, c_int,
                                 ctypes.POINTER(c_vp)]),
    "cudair_ctx_synchronize": (c_int, []),
    "cudair_matmul16": (c_int, [c_vp, c_vp, c_vp, ctypes.c_int32, c_vp]),
    "cudair_gemm_f16f32": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                   c_vp]),
    "cudair_gemm_f16f32_noalloc": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64,
                                           c_i64, c_vp]),
    "cudair_gemm_f16f32_host": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                        c_vp, c_vp, c_vp, c_i64, c_vp]),
    "cudair_matmul16_host": (c_int, [c_vp, c_vp, c_vp, ctypes.c_int32, c_vp, c_vp, c_vp, c_vp]),
    "cudair_vecadd_host": (c_int, [c_vp, c_vp, c_vp, ctypes.c_int32, c_vp, c_vp, c_vp, ctypes.c_int32,
                                   c_vp]),
    "cudair_gemm": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                            c_u32, c_vp]),
    "cudair_set_gemm_variant": (c_int, [c_int]),
    "cudair_set_gemm_pdl": (c_int, [c_int]),
    "cudair_vecadd": (c_int, [c_vp, c_vp, c_vp, ctypes.c_int32, c_vp]),
    "cudair_saxpy": (c_int, [ctypes.c_float, c_vp, c_vp, ctypes.c_int32, c_vp]),
    "cudair_square": (c_int, [c_vp, ctypes.c_int32, c_vp]),
    "cudair_reduce_f32": (c_int, [c_vp, c_vp, ctypes.c_int32, c_vp]),
    "cudair_fill": (c_int, [c_vp, c_u32, c_u32, c_i64, c_u64, c_i64, ctypes.c_double, ctypes.c_double,
                            c_vp]),
    "cudair_wait_status": (c_int, [_u32p, c_int]),
    "cudair_wait_timeout_selftest": (c_int, [c_u64, c_vp]),
    "cudair_ipc_export": (c_int, [c_vp, c_vp, _u64p]),
    "cudair_ipc_open": (c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "cudair_ipc_close": (c_int, [c_vp]),
    "cudair_peer_copy": (c_int, [c_vp, c_vp, c_size, c_vp]),
}

# Error codes of include/cudair_b200.h.
OK, ERR_INVALID, ERR_DRIVER, ERR_CUDA, ERR_TIMEOUT, ERR_UNSUPPORTED = range(6)


class CudairError(RuntimeError):
    """A failed C-ABI call: .code is the CUDAIR_ERR_* value."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def header_functions() -> list[str]:
    """Names of the functions include/cudair_b200.h declares."""
    text = open(HEADER_PATH).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cudair_[a-z0-9_]+)\s*\(", text)))


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python cuda-ir.go_b200/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().cudair_last_error().decode()


def check(rc: int) -> None:
    if rc != OK:
        raise CudairError(rc, last_error())
