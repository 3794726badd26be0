"""cudair_gemm_f16f32_noalloc: the few-row GEMM for callers that must not
allocate device memory (their device memory belongs to another allocator,
or allocating after start-up is forbidden because cudaMalloc can synchronise
the device).  Its scratch space is a fixed array inside the library, so the
test checks, through the C ABI, that two calls in a row each match the
allocating entry point cudair_gemm_f16f32 within the GEMM tolerance (the
second call runs on the array the first one left behind), and that requests
beyond the array's limits are refused.

This file is collected last so that a failure here never hides another test.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gemm(cudair, fn, da, db, c_init, dev):
    import torch
    M, K = da.shape
    N = db.shape[1]
    dc = torch.from_numpy(c_init.copy()).to(dev)
    stream = torch.cuda.current_stream().cuda_stream
    rc = getattr(cudair.lib(), fn)(da.data_ptr(), db.data_ptr(), dc.data_ptr(), M, N, K,
                                   da.stride(0), db.stride(0), dc.stride(0), stream)
    assert rc == 0, cudair.last_error()
    torch.cuda.synchronize()
    return dc.cpu().numpy()


@pytest.mark.parametrize("M,N,K", [(16, 14336, 4096), (40, 2056, 1000)])
def test_noalloc_matches_allocating_entry_twice(dev, cudair, oracle, M, N, K):
    import torch
    from cudair import kernels
    a16 = oracle.f32_to_f16(oracle.normal(M * K, 81, 0.0, 1.0))
    b16 = oracle.f32_to_f16(oracle.normal(K * N, 82, 0.0, 0.02))
    c = oracle.uniform(M * N, 83).reshape(M, N)
    da = torch.from_numpy(a16.view(np.int16)).to(dev).view(torch.float16).reshape(M, K)
    db = torch.from_numpy(b16.view(np.int16)).to(dev).view(torch.float16).reshape(K, N)
    kernels.set_gemm_variant(0)
    want = _gemm(cudair, "cudair_gemm_f16f32", da, db, c, dev)
    af = oracle.f16_to_f32(a16)
    bf = oracle.f16_to_f32(b16)
    tol_rel, tol_max = oracle.gemm_tolerance(K, np.abs(af).max(), np.abs(bf).max())
    for _ in range(2):
        got = _gemm(cudair, "cudair_gemm_f16f32_noalloc", da, db, c, dev)
        rel, mx, bad = oracle.error_norms(got, want)
        assert bad == 0 and rel <= tol_rel and mx <= tol_max, (rel, mx)
    assert kernels.wait_status(clear=True) == 0


def test_noalloc_rejects_sizes_beyond_its_scratch(dev, cudair):
    L = cudair.lib()
    rc = L.cudair_gemm_f16f32_noalloc(16, 16, 16, 65, 128, 64, 64, 128, 128, None)
    assert rc == 1 and "exceeds the maximum of 64 rows" in cudair.last_error()
    rc = L.cudair_gemm_f16f32_noalloc(16, 16, 16, 16, 524288 + 8, 64, 64, 524288 + 8, 524288 + 8, None)
    assert rc == 1 and "exceeds the maximum of 524288 columns" in cudair.last_error()
