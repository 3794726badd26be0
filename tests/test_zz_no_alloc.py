"""cudair_gemm_f16f32_noalloc: the few-row GEMM for callers that must not
allocate device memory (their device memory belongs to another allocator,
or allocating after start-up is forbidden because cudaMalloc can synchronise
the device).  Its scratch space is a fixed array inside the library, so the
test checks, through the C ABI:
  * two calls in a row each match the allocating entry point
    cudair_gemm_f16f32 within the GEMM tolerance (the second call runs on the
    array the first one left behind);
  * after a first call on the device (the start-up call, which under lazy
    module loading is when the array is reserved), those two calls change
    neither the device's free memory (cudaMemGetInfo) nor the bytes torch's
    caching allocator holds;
  * requests beyond the array's limits are refused.

This file is collected last so that a failure here never hides another test.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _call(cudair, fn, da, db, dc):
    import torch
    M, K = da.shape
    N = db.shape[1]
    stream = torch.cuda.current_stream().cuda_stream
    rc = getattr(cudair.lib(), fn)(da.data_ptr(), db.data_ptr(), dc.data_ptr(), M, N, K,
                                   da.stride(0), db.stride(0), dc.stride(0), stream)
    assert rc == 0, cudair.last_error()


@pytest.mark.parametrize("M,N,K", [(16, 14336, 4096), (40, 2056, 1000)])
def test_noalloc_matches_allocating_entry_twice(dev, cudair, oracle, M, N, K):
    import torch
    from cudair import kernels
    a16 = oracle.f32_to_f16(oracle.normal(M * K, 81, 0.0, 1.0))
    b16 = oracle.f32_to_f16(oracle.normal(K * N, 82, 0.0, 0.02))
    c = oracle.uniform(M * N, 83).reshape(M, N)
    c_h = torch.from_numpy(c)
    da = torch.from_numpy(a16.view(np.int16)).to(dev).view(torch.float16).reshape(M, K)
    db = torch.from_numpy(b16.view(np.int16)).to(dev).view(torch.float16).reshape(K, N)
    dc = torch.empty(M, N, device=dev)
    kernels.set_gemm_variant(0)
    dc.copy_(c_h)
    _call(cudair, "cudair_gemm_f16f32", da, db, dc)
    torch.cuda.synchronize()
    want = dc.cpu().numpy()
    af = oracle.f16_to_f32(a16)
    bf = oracle.f16_to_f32(b16)
    tol_rel, tol_max = oracle.gemm_tolerance(K, np.abs(af).max(), np.abs(bf).max())

    # The start-up call: loads the library's image on this device if nothing
    # did before, and looks up the array's address.
    dc.copy_(c_h)
    _call(cudair, "cudair_gemm_f16f32_noalloc", da, db, dc)
    torch.cuda.synchronize()

    free_before, _ = torch.cuda.mem_get_info()
    held_before = torch.cuda.memory_reserved()
    results = []
    for _ in range(2):
        dc.copy_(c_h)
        _call(cudair, "cudair_gemm_f16f32_noalloc", da, db, dc)
        torch.cuda.synchronize()
        results.append(dc.cpu().numpy())
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, (free_before, free_after)
    assert torch.cuda.memory_reserved() == held_before
    for got in results:
        rel, mx, bad = oracle.error_norms(got, want)
        assert bad == 0 and rel <= tol_rel and mx <= tol_max, (rel, mx)
    assert kernels.wait_status(clear=True) == 0


def test_noalloc_rejects_sizes_beyond_its_scratch(dev, cudair):
    L = cudair.lib()
    rc = L.cudair_gemm_f16f32_noalloc(16, 16, 16, 65, 128, 64, 64, 128, 128, None)
    assert rc == 1 and "exceeds the maximum of 64 rows" in cudair.last_error()
    rc = L.cudair_gemm_f16f32_noalloc(16, 16, 16, 16, 524288 + 8, 64, 64, 524288 + 8, 524288 + 8, None)
    assert rc == 1 and "exceeds the maximum of 524288 columns" in cudair.last_error()
