"""Launchers of the tuned sm_100a kernels over the C ABI, taking torch CUDA
tensors (device memory and streams come from torch; the arithmetic is the
library's).  Each call is asynchronous on the given stream (default: torch's
current stream).
"""
from __future__ import annotations

import ctypes

from ._lib import CudairError, check, lib


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _need(t, dtype, name):
    import torch
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise CudairError(1, f"cudair: {name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise CudairError(1, f"cudair: {name} must be {dtype}, got {t.dtype}")
    # The library launches on the current device; a tensor of another GPU
    # would be read across NVLink by the kernels (or fail to launch).
    cur = torch.cuda.current_device()
    if t.device.index != cur:
        raise CudairError(1, f"cudair: {name} is on {t.device}, the current device is cuda:{cur}")


def matmul16(a, b, c, stream=None) -> None:
    """c += a @ b for n x n row-major fp16 a, b and fp32 c (MatMul16's operands)."""
    import torch
    _need(a, torch.float16, "a")
    _need(b, torch.float16, "b")
    _need(c, torch.float32, "c")
    n = a.shape[0]
    if not (a.shape == b.shape == c.shape == (n, n)) or not (
            a.is_contiguous() and b.is_contiguous() and c.is_contiguous()):
        raise CudairError(1, "cudair: MatMul16: a, b, c must be contiguous n x n")
    check(lib().cudair_matmul16(a.data_ptr(), b.data_ptr(), c.data_ptr(), n, _stream(stream)))


def gemm(a, b, c, stream=None) -> None:
    """c += a @ b: a (M x K) and b (K x N) fp16, c (M x N) fp32, row-major with
    unit inner stride."""
    import torch
    _need(a, torch.float16, "a")
    _need(b, torch.float16, "b")
    _need(c, torch.float32, "c")
    M, K = a.shape
    K2, N = b.shape
    if K2 != K or tuple(c.shape) != (M, N):
        raise CudairError(1, f"cudair: gemm: shapes {tuple(a.shape)} {tuple(b.shape)} {tuple(c.shape)}")
    for t, nm in ((a, "a"), (b, "b"), (c, "c")):
        if t.stride(1) != 1:
            raise CudairError(1, f"cudair: gemm: {nm} needs unit inner stride")
    check(lib().cudair_gemm_f16f32(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K,
                                   a.stride(0), b.stride(0), c.stride(0), _stream(stream)))


GEMM_BF16, GEMM_B_T, GEMM_OVERWRITE, GEMM_C_F16 = 0x1, 0x2, 0x4, 0x8


def gemm_ex(a, b, c, bias=None, b_trans=False, overwrite=False, stream=None) -> None:
    """The tensor-package GEMM family on the tcgen05 kernels (cudair_gemm):
    c (+)= a @ B with B = b, or b.T when b_trans (b is N x K).  a and b are
    both fp16 or both bf16; c is fp32 (accumulated into, or written when
    overwrite) or fp16 (written: needs overwrite); bias (fp32 M x N) gives
    c = a @ B + bias."""
    import torch
    if a.dtype not in (torch.float16, torch.bfloat16) or b.dtype != a.dtype:
        raise CudairError(1, "cudair: gemm_ex: a and b must be both float16 or both bfloat16")
    for t, nm in ((a, "a"), (b, "b"), (c, "c")):
        _need(t, t.dtype, nm)
        if t.stride(1) != 1:
            raise CudairError(1, f"cudair: gemm_ex: {nm} needs unit inner stride")
    if c.dtype not in (torch.float32, torch.float16):
        raise CudairError(1, "cudair: gemm_ex: c must be float32 or float16")
    M, K = a.shape
    N = b.shape[0] if b_trans else b.shape[1]
    if (b.shape[1] if b_trans else b.shape[0]) != K or tuple(c.shape) != (M, N):
        raise CudairError(1, f"cudair: gemm_ex: shapes {tuple(a.shape)} {tuple(b.shape)} {tuple(c.shape)}")
    flags = (GEMM_BF16 if a.dtype == torch.bfloat16 else 0) | (GEMM_B_T if b_trans else 0) | \
        (GEMM_OVERWRITE if overwrite else 0) | (GEMM_C_F16 if c.dtype == torch.float16 else 0)
    bias_ptr, ldbias = None, 0
    if bias is not None:
        _need(bias, torch.float32, "bias")
        if tuple(bias.shape) != (M, N) or bias.stride(1) != 1:
            raise CudairError(1, "cudair: gemm_ex: bias must be M x N with unit inner stride")
        bias_ptr, ldbias = bias.data_ptr(), bias.stride(0)
    check(lib().cudair_gemm(a.data_ptr(), b.data_ptr(), c.data_ptr(), bias_ptr, M, N, K, a.stride(0),
                            b.stride(0), c.stride(0), ldbias, flags, _stream(stream)))


def gemm_host(a_h, b_h, c_h, a_d, b_d, c_d, rows_per_block=0, stream=None) -> None:
    """c_h += a_h @ b_h from host (CPU) tensors, through the caller's device
    buffers a_d, b_d, c_d (dense, same shapes): copies in, GEMM and copy out
    pipelined over tiles of C (rows_per_block > 0: full-width row blocks of
    that height; 0: automatic).  b_h = None: b_d already holds B.
    Asynchronous on `stream`; c_h holds the result once the stream is
    synchronised.  Pinned host tensors let the copies overlap."""
    import torch
    for t, dt, nm in ((a_h, torch.float16, "a_h"), (b_h, torch.float16, "b_h"),
                      (c_h, torch.float32, "c_h")):
        if t is None and nm == "b_h":
            continue  # B already in b_d
        if not isinstance(t, torch.Tensor) or t.is_cuda or t.dtype != dt or t.stride(1) != 1:
            raise CudairError(1, f"cudair: gemm_host: {nm} must be a host {dt} tensor, unit inner stride")
    for t, dt, nm in ((a_d, torch.float16, "a_d"), (b_d, torch.float16, "b_d"),
                      (c_d, torch.float32, "c_d")):
        _need(t, dt, nm)
        if not t.is_contiguous():
            raise CudairError(1, f"cudair: gemm_host: {nm} must be contiguous")
    M, K = a_h.shape
    K2, N = b_d.shape
    if K2 != K or tuple(c_h.shape) != (M, N) or tuple(a_d.shape) != (M, K) or \
            tuple(c_d.shape) != (M, N) or (b_h is not None and tuple(b_h.shape) != (K, N)):
        raise CudairError(1, "cudair: gemm_host: shapes do not match")
    check(lib().cudair_gemm_f16f32_host(
        a_h.data_ptr(), None if b_h is None else b_h.data_ptr(), c_h.data_ptr(), M, N, K,
        a_h.stride(0), N if b_h is None else b_h.stride(0),
        c_h.stride(0), a_d.data_ptr(), b_d.data_ptr(), c_d.data_ptr(), rows_per_block,
        _stream(stream)))


def _host_tensor(t, dtype, name):
    import torch
    if not isinstance(t, torch.Tensor) or t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise CudairError(1, f"cudair: {name} must be a contiguous host {dtype} tensor")


def vecadd_host(a_h, b_h, out_h, a_d, b_d, out_d, chunk=0, stream=None) -> None:
    """out_h = a_h + b_h from host (CPU) fp32 vectors through the caller's
    device buffers (cudair_vecadd_host): copies in, VecAdd and copies out
    pipelined over chunks.  Asynchronous on `stream`; pinned host tensors let
    the copies overlap."""
    import torch
    for t, nm in ((a_h, "a_h"), (b_h, "b_h"), (out_h, "out_h")):
        _host_tensor(t, torch.float32, nm)
    for t, nm in ((a_d, "a_d"), (b_d, "b_d"), (out_d, "out_d")):
        _need(t, torch.float32, nm)
    n = out_h.numel()
    if any(t.numel() != n for t in (a_h, b_h, a_d, b_d, out_d)):
        raise CudairError(1, "cudair: vecadd_host: length mismatch")
    check(lib().cudair_vecadd_host(a_h.data_ptr(), b_h.data_ptr(), out_h.data_ptr(), n, a_d.data_ptr(),
                                   b_d.data_ptr(), out_d.data_ptr(), chunk, _stream(stream)))


def matmul16_host(a_h, b_h, c_h, a_d, b_d, c_d, stream=None) -> None:
    """c_h += a_h @ b_h for n x n host tensors (MatMul16's operands) through
    the caller's device buffers (cudair_matmul16_host).  Asynchronous on
    `stream`."""
    import torch
    _host_tensor(a_h, torch.float16, "a_h")
    _host_tensor(b_h, torch.float16, "b_h")
    _host_tensor(c_h, torch.float32, "c_h")
    _need(a_d, torch.float16, "a_d")
    _need(b_d, torch.float16, "b_d")
    _need(c_d, torch.float32, "c_d")
    n = c_h.shape[0]
    if any(tuple(t.shape) != (n, n) for t in (a_h, b_h, c_h, a_d, b_d, c_d)):
        raise CudairError(1, "cudair: matmul16_host: every operand must be n x n")
    check(lib().cudair_matmul16_host(a_h.data_ptr(), b_h.data_ptr(), c_h.data_ptr(), n, a_d.data_ptr(),
                                     b_d.data_ptr(), c_d.data_ptr(), _stream(stream)))


def set_gemm_variant(variant: int) -> None:
    """0 = automatic, 1 = single-CTA 128x256 tiles, 2 = CTA-pair 256x256 tiles,
    3 = few-row kernel (M <= 128), 4 = CTA-pair 256x512 tiles, 5 = small-problem
    kernel (K <= 512), 6 = few-row kernel with k-chunks handed out at run time
    (M <= 64)."""
    check(lib().cudair_set_gemm_variant(variant))


def set_gemm_pdl(mode: int) -> None:
    """Programmatic dependent launch of the few-row GEMM: 0 off, 1 on, 2 on
    with B (weights, not written by the preceding kernel) requested early."""
    check(lib().cudair_set_gemm_pdl(mode))


def vecadd(a, b, out, stream=None) -> None:
    """out = a + b over fp32 vectors (VecAdd's operands)."""
    import torch
    for t, nm in ((a, "a"), (b, "b"), (out, "out")):
        _need(t, torch.float32, nm)
    n = out.numel()
    if a.numel() != n or b.numel() != n:
        raise CudairError(1, "cudair: VecAdd: length mismatch")
    check(lib().cudair_vecadd(a.data_ptr(), b.data_ptr(), out.data_ptr(), n, _stream(stream)))


def saxpy(alpha, x, y, stream=None) -> None:
    """y = alpha * x + y over fp32 vectors (Saxpy's operands)."""
    import torch
    _need(x, torch.float32, "x")
    _need(y, torch.float32, "y")
    if x.numel() != y.numel():
        raise CudairError(1, "cudair: Saxpy: length mismatch")
    check(lib().cudair_saxpy(float(alpha), x.data_ptr(), y.data_ptr(), y.numel(), _stream(stream)))


def square(x, stream=None) -> None:
    """x = x * x in place over an fp32 vector (Square's operand)."""
    import torch
    _need(x, torch.float32, "x")
    check(lib().cudair_square(x.data_ptr(), x.numel(), _stream(stream)))


def reduce_f32(x, out, stream=None) -> None:
    """out[2w], out[2w+1] = min, max of warp w's 32 values (ReduceF32)."""
    import torch
    _need(x, torch.float32, "in")
    _need(out, torch.float32, "out")
    check(lib().cudair_reduce_f32(x.data_ptr(), out.data_ptr(), x.numel(), _stream(stream)))


FILL_F32, FILL_F16 = 0, 1
FILL_UNIFORM, FILL_NORMAL = 0, 1


def _fill(t, dist, seed, p0, p1, offset, stream):
    import torch
    if t.dtype not in (torch.float32, torch.float16):
        raise CudairError(1, f"cudair: fill: tensor must be float32 or float16, got {t.dtype}")
    _need(t, t.dtype, "out")
    if not t.is_contiguous():
        raise CudairError(1, "cudair: fill: tensor must be contiguous")
    check(lib().cudair_fill(t.data_ptr(), FILL_F16 if t.dtype == torch.float16 else FILL_F32, dist,
                            t.numel(), seed, offset, float(p0), float(p1), _stream(stream)))


def fill_uniform(t, seed: int, lo=-1.0, hi=1.0, offset: int = 0, stream=None) -> None:
    """Fills t (contiguous fp32 or fp16) with elements offset.. of the seeded
    U(lo, hi) stream (cudair_fill), bit for bit the CPU oracle's values."""
    _fill(t, FILL_UNIFORM, seed, lo, hi, offset, stream)


def fill_normal(t, seed: int, mean=0.0, std=1.0, offset: int = 0, stream=None) -> None:
    """Fills t (contiguous fp32 or fp16) with elements offset.. of the seeded
    N(mean, std) stream (cudair_fill), bit for bit the CPU oracle's values."""
    _fill(t, FILL_NORMAL, seed, mean, std, offset, stream)


def wait_status(clear: bool = True) -> int:
    """Synchronises and returns the bounded-wait status word (0 = no wait gave
    up); raises CudairError(ERR_TIMEOUT) when a bit is set."""
    v = ctypes.c_uint32()
    rc = lib().cudair_wait_status(ctypes.byref(v), 1 if clear else 0)
    if rc != 0:
        err = CudairError(rc, lib().cudair_last_error().decode())
        err.status = v.value
        raise err
    return v.value


def wait_timeout_selftest(limit_ns: int, stream=None) -> None:
    check(lib().cudair_wait_timeout_selftest(limit_ns, _stream(stream)))
