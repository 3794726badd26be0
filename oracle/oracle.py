"""ctypes front end of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker or the timed CPU baseline.  The
product path (the CUDA library under cuda-ir.go_b200/) never imports it.

Each function names the reference test whose CPU model oracle.c restates:
  f32_to_f16      float32ToHalf, advanced_test.go:597-623
  matmul16/gemm   the i-j-k float32 loop, advanced_test.go:466-475
  vecadd          out = a + b, main_test.go:51
  reduce_f32      math.Min/Max fold per warp, advanced_test.go:572-579
  saxpy/square    examples/vecadd/run/main.go:62-76
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64 = ctypes.c_int64


def build() -> str:
    """Compiles oracle.c with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(
            os.path.join(_HERE, "oracle.c")
        ):
            build()
        L = ctypes.CDLL(_SO)
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        L.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        L.oracle_f16_to_f32.restype = ctypes.c_float
        L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_f32_to_f16_array.argtypes = [_f32p, _u16p, _i64]
        L.oracle_f16_to_f32_array.argtypes = [_u16p, _f32p, _i64]
        gemm_args = [_i64, _i64, _i64, _f32p, _i64, _f32p, _i64, _f32p, _i64,
                     _f32p, _i64, _i64, _i64, ctypes.c_int]
        L.oracle_gemm_ijk.argtypes = gemm_args
        L.oracle_gemm_ikj.argtypes = gemm_args
        L.oracle_matmul16.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int32]
        L.oracle_vecadd.argtypes = [_f32p, _f32p, _f32p, _i64, ctypes.c_int]
        L.oracle_reduce_f32.argtypes = [_f32p, _f32p, ctypes.c_int32]
        L.oracle_saxpy.argtypes = [ctypes.c_float, _f32p, _f32p, _i64]
        L.oracle_square.argtypes = [_f32p, _i64]
        L.oracle_stream_word.restype = ctypes.c_uint64
        L.oracle_stream_word.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.oracle_fill_uniform.argtypes = [_f32p, _i64, ctypes.c_uint64, _i64,
                                          ctypes.c_float, ctypes.c_float]
        L.oracle_fill_normal.argtypes = [_f32p, _i64, ctypes.c_uint64, _i64,
                                         ctypes.c_double, ctypes.c_double]
        L.oracle_error_norms.argtypes = [_f32p, _f32p, _i64, _f64p]
        L.oracle_num_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(t)


def num_threads() -> int:
    return int(lib().oracle_num_threads())


# ---- fp16 ------------------------------------------------------------------

def f32_to_f16(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 bits (uint16), float32ToHalf of advanced_test.go:597-623."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_f16_array(_p(x, _f32p), _p(out, _u16p), x.size)
    return out


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().oracle_f16_to_f32_array(_p(h, _u16p), _p(out, _f32p), h.size)
    return out


# ---- GEMM ------------------------------------------------------------------

def gemm_ijk(af, bf, c, rows=None, threads=1) -> np.ndarray:
    """c + af.bf by the reference's i-j-k float32 loop (advanced_test.go:466-475).

    af: M x K, bf: K x N, c: M x N float32 (fp16-rounded operands widened to
    float32).  rows=(r0, r1) computes only those rows.
    """
    af = np.ascontiguousarray(af, dtype=np.float32)
    bf = np.ascontiguousarray(bf, dtype=np.float32)
    c = np.ascontiguousarray(c, dtype=np.float32)
    M, K = af.shape
    K2, N = bf.shape
    assert K == K2 and c.shape == (M, N)
    r0, r1 = rows if rows is not None else (0, M)
    out = np.empty((r1 - r0, N), dtype=np.float32)
    lib().oracle_gemm_ijk(M, N, K, _p(af, _f32p), K, _p(bf, _f32p), N,
                          _p(c, _f32p), N, _p(out, _f32p), N, r0, r1, threads)
    return out


def gemm_ikj(af, bf, c, rows=None, threads=None) -> np.ndarray:
    """c + af.bf in float32, i-k-j order (tolerance reference for big sizes)."""
    af = np.ascontiguousarray(af, dtype=np.float32)
    bf = np.ascontiguousarray(bf, dtype=np.float32)
    c = np.ascontiguousarray(c, dtype=np.float32)
    M, K = af.shape
    K2, N = bf.shape
    assert K == K2 and c.shape == (M, N)
    r0, r1 = rows if rows is not None else (0, M)
    out = np.empty((r1 - r0, N), dtype=np.float32)
    lib().oracle_gemm_ikj(M, N, K, _p(af, _f32p), K, _p(bf, _f32p), N,
                          _p(c, _f32p), N, _p(out, _f32p), N, r0, r1,
                          threads or num_threads())
    return out


def matmul16(af, bf, c) -> np.ndarray:
    """The square n x n model of TestHopper/MatMul16."""
    af = np.ascontiguousarray(af, dtype=np.float32)
    n = af.shape[0]
    bf = np.ascontiguousarray(bf, dtype=np.float32)
    c = np.ascontiguousarray(c, dtype=np.float32)
    out = np.empty((n, n), dtype=np.float32)
    lib().oracle_matmul16(_p(af, _f32p), _p(bf, _f32p), _p(c, _f32p),
                          _p(out, _f32p), n)
    return out


# ---- VecAdd / ReduceF32 ----------------------------------------------------

def vecadd(a, b, threads=1) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    out = np.empty_like(a)
    lib().oracle_vecadd(_p(a, _f32p), _p(b, _f32p), _p(out, _f32p), a.size, threads)
    return out


def saxpy(alpha: float, x, y) -> np.ndarray:
    """alpha*x + y, rounded after the product and after the sum
    (the check of examples/vecadd/run/main.go:62-68)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.array(y, dtype=np.float32, copy=True)
    lib().oracle_saxpy(alpha, _p(x, _f32p), _p(out, _f32p), x.size)
    return out


def square(x) -> np.ndarray:
    """x*x (the check of examples/vecadd/run/main.go:70-76)."""
    out = np.array(x, dtype=np.float32, copy=True)
    lib().oracle_square(_p(out, _f32p), out.size)
    return out


def reduce_f32(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(2 * (x.size // 32), dtype=np.float32)
    lib().oracle_reduce_f32(_p(x, _f32p), _p(out, _f32p), x.size)
    return out


# ---- generators --------------------------------------------------------------

def stream_word(seed: int, i: int) -> int:
    return int(lib().oracle_stream_word(seed, i))


def uniform(n: int, seed: int, lo=-1.0, hi=1.0, offset=0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().oracle_fill_uniform(_p(out, _f32p), n, seed, offset, lo, hi)
    return out


def normal(n: int, seed: int, mean=0.0, std=1.0, offset=0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().oracle_fill_normal(_p(out, _f32p), n, seed, offset, mean, std)
    return out


def error_norms(got, want):
    """(relative Frobenius, max abs, non-finite count) of got vs want."""
    got = np.ascontiguousarray(got, dtype=np.float32).ravel()
    want = np.ascontiguousarray(want, dtype=np.float32).ravel()
    assert got.size == want.size
    res = np.zeros(3, dtype=np.float64)
    lib().oracle_error_norms(_p(got, _f32p), _p(want, _f32p), got.size,
                             _p(res, _f64p))
    return float(res[0]), float(res[1]), int(res[2])


def gemm_tolerance(K: int, amax: float, bmax: float):
    """The north-star bounds: rel-Frobenius <= 1e-3 and
    max |err| <= 5e-3 * sqrt(K) * max|a| * max|b|."""
    return 1e-3, 5e-3 * np.sqrt(K) * amax * bmax


# ---- the reference tests' known-answer inputs -------------------------------

def matmul16_kat(n: int = 64):
    """TestHopper/MatMul16 data (advanced_test.go:457-465):
    af = (i+2j)%7-3, bf = (3i+j)%5-2, c = j-i."""
    i = np.arange(n).reshape(n, 1)
    j = np.arange(n).reshape(1, n)
    af = ((i + 2 * j) % 7 - 3).astype(np.float32)
    bf = ((3 * i + j) % 5 - 2).astype(np.float32)
    c = (j - i).astype(np.float32)
    return af, bf, c


def vecadd_kat(n: int = 1 << 20):
    """TestVecAdd data (main_test.go:26-31): a = 0.5 i, b = 1000 - i (float32)."""
    i = np.arange(n, dtype=np.float32)
    return (i * np.float32(0.5)).astype(np.float32), (np.float32(1000) - i).astype(np.float32)


def reduce_kat(n: int = 1024):
    """TestBlackwell data (advanced_test.go:564-568): float32(sin(i))."""
    return np.sin(np.arange(n, dtype=np.float64)).astype(np.float32)
