"""Programmatic dependent launch of the few-row GEMM (cudair_set_gemm_pdl):
chains of GEMMs and other kernels on one stream give the same exact results
in every mode.  A GEMM that reads A written by the kernel before it, or adds
into C that the GEMM before it wrote, sees that data; so does a chain
replayed from a CUDA graph."""
import numpy as np
import pytest

from test_matmul16_gpu import kat

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[0, 1, 2], ids=["plain", "pdl", "pdl-b-early"])
def pdl(request, dev, cudair):
    from cudair import kernels
    kernels.set_gemm_pdl(request.param)
    yield request.param
    kernels.set_gemm_pdl(0)


def _ops(M, N, K, dev, seed):
    import torch
    rng = np.random.default_rng(seed)
    a = rng.integers(-3, 4, size=(M, K)).astype(np.float32)
    b = rng.integers(-2, 3, size=(K, N)).astype(np.float32)
    return a, b, torch.from_numpy(a).to(dev).half(), torch.from_numpy(b).to(dev).half()


def test_pdl_chain_sees_preceding_writes(dev, cudair, pdl):
    import torch
    from cudair import kernels
    M, N, K = 16, 4096, 1024
    a1, b1, da1, db1 = _ops(M, N, K, dev, 1)
    a2, b2, _, db2 = _ops(M, N, K, dev, 2)
    _, b3, _, db3 = _ops(M, N, K, dev, 3)
    c0 = np.arange(M * N, dtype=np.float32).reshape(M, N) % 97 - 48
    dc = torch.from_numpy(c0).to(dev)
    da2 = torch.zeros(M, K, dtype=torch.float16, device=dev)
    src2 = torch.from_numpy(a2).to(dev).half()
    torch.cuda.synchronize()
    big = torch.randn(2048, 2048, device=dev)
    for _ in range(3):
        big = big @ big  # keeps the stream busy so the chain is queued behind it
    kernels.gemm(da1, db1, dc)   # C += A1 B1
    da2.copy_(src2)              # a torch kernel writes A2
    kernels.gemm(da2, db2, dc)   # reads the new A2, adds into C from the first GEMM
    kernels.gemm(da2, db3, dc)   # back to back with the previous GEMM
    torch.cuda.synchronize()
    want = c0.astype(np.int64) + a1.astype(np.int64) @ b1.astype(np.int64) \
        + a2.astype(np.int64) @ b2.astype(np.int64) + a2.astype(np.int64) @ b3.astype(np.int64)
    assert np.array_equal(dc.cpu().numpy(), want.astype(np.float32))


@pytest.mark.parametrize("M,N,K", [(16, 14336, 4096), (64, 1000, 520), (3, 2056, 8192)])
def test_pdl_long_chain_accumulates(dev, cudair, pdl, M, N, K):
    import torch
    from cudair import kernels
    af, bf, c, want1 = kat(M, N, K)
    da = torch.from_numpy(af).to(dev).half()
    db = torch.from_numpy(bf).to(dev).half()
    dc = torch.from_numpy(c).to(dev)
    reps = 12
    for _ in range(reps):
        kernels.gemm(da, db, dc)
    torch.cuda.synchronize()
    prod = (want1.astype(np.float64) - c)
    assert np.array_equal(dc.cpu().numpy(), (c + reps * prod).astype(np.float32))


def test_pdl_chain_in_cuda_graph(dev, cudair, pdl):
    import torch
    from cudair import kernels
    M, N, K = 16, 4096, 2048
    af, bf, c, want1 = kat(M, N, K)
    da = torch.from_numpy(af).to(dev).half()
    dbs = [torch.from_numpy(bf).to(dev).half() for _ in range(3)]
    dc = torch.from_numpy(c).to(dev)
    kernels.gemm(da, dbs[0], dc)  # first use outside capture (workspace, attributes)
    torch.cuda.synchronize()
    dc.copy_(torch.from_numpy(c))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=torch.cuda.Stream(device=dev)):
        for i in range(9):
            kernels.gemm(da, dbs[i % 3], dc)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    prod = want1.astype(np.float64) - c
    assert np.array_equal(dc.cpu().numpy(), (c + 18 * prod).astype(np.float32))


@pytest.mark.parametrize("variant", [1, 2, 4], ids=["single", "pair", "pairwide"])
def test_pdl_square_kernel_chain(dev, cudair, pdl, variant):
    # The square-tile kernels under programmatic dependent launch: a chain
    # that reads an A just written by a torch kernel and adds into a C just
    # written by the preceding GEMM, exact in every mode.
    import torch
    from cudair import kernels
    M, N, K = 512, 1024, 256
    a1, b1, da1, db1 = _ops(M, N, K, dev, 21)
    a2, b2, _, db2 = _ops(M, N, K, dev, 22)
    c0 = (np.arange(M * N, dtype=np.float32).reshape(M, N) % 89) - 44
    dc = torch.from_numpy(c0).to(dev)
    da2 = torch.zeros(M, K, dtype=torch.float16, device=dev)
    src2 = torch.from_numpy(a2).to(dev).half()
    torch.cuda.synchronize()
    kernels.set_gemm_variant(variant)
    try:
        big = torch.randn(2048, 2048, device=dev)
        for _ in range(3):
            big = big @ big
        for _ in range(3):
            kernels.gemm(da1, db1, dc)
        da2.copy_(src2)
        kernels.gemm(da2, db2, dc)
        kernels.gemm(da2, db2, dc)
        torch.cuda.synchronize()
    finally:
        kernels.set_gemm_variant(0)
    p1 = a1.astype(np.int64) @ b1.astype(np.int64)
    p2 = a2.astype(np.int64) @ b2.astype(np.int64)
    want = (c0.astype(np.int64) + 3 * p1 + 2 * p2).astype(np.float32)
    assert np.array_equal(dc.cpu().numpy(), want)
