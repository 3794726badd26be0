"""The library runs in the device's primary context (the one gocudrv and the
CUDA runtime use): a call made while another context is current is refused
with CUDAIR_ERR_UNSUPPORTED before anything is launched, and calls work
again once the primary context is current."""
import ctypes

import pytest

pytestmark = pytest.mark.gpu


def test_a_non_primary_context_is_refused(dev, cudair):
    import torch
    from cudair import kernels
    x = torch.ones(1024, device=dev)
    out = torch.empty_like(x)
    kernels.vecadd(x, x, out)  # the library's per-device state, in the primary context
    torch.cuda.synchronize()
    cu = ctypes.CDLL("libcuda.so.1")
    ctx = ctypes.c_void_p()
    assert cu.cuCtxCreate_v2(ctypes.byref(ctx), 0, 0) == 0  # created and made current
    try:
        L = cudair.lib()
        rc = L.cudair_vecadd(x.data_ptr(), x.data_ptr(), out.data_ptr(), 1024, None)
        assert rc == 5 and "primary context" in cudair.last_error(), cudair.last_error()
        rc = L.cudair_gemm_f16f32_noalloc(256, 256, 256, 16, 128, 64, 64, 128, 128, None)
        assert rc == 5 and "primary context" in cudair.last_error(), cudair.last_error()
    finally:
        popped = ctypes.c_void_p()
        assert cu.cuCtxPopCurrent_v2(ctypes.byref(popped)) == 0
        assert cu.cuCtxDestroy_v2(ctx) == 0
    out.zero_()
    kernels.vecadd(x, x, out)
    torch.cuda.synchronize()
    assert bool((out == 2).all())
