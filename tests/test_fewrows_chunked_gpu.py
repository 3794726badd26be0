"""The chunked few-row GEMM (variant 6) on the B200: C = A.B + C for M <= 64
with each 128-column tile cut into fixed k-chunks that the SMs take at run
time from a ticket counter, and each tile summed by its last chunk in chunk
order.

Exact on the TestHopper generator's integer operands (advanced_test.go:459-463),
bit-identical between runs, within the oracle tolerance on seeded data, and
correct over chains of launches (the ticket is reset by each launch's last
CTA and read by the next only after its dependency wait).
"""
import functools
import os

import numpy as np
import pytest

from test_matmul16_gpu import _dev, _seeded_normal_f16, kat

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def chunked(dev, cudair):
    from cudair import kernels
    kernels.wait_status(clear=True)
    kernels.set_gemm_variant(6)
    yield
    kernels.set_gemm_variant(0)
    kernels.set_gemm_pdl(0)
    os.environ.pop("CUDAIR_FEWROWS_CHUNKS", None)
    assert kernels.wait_status(clear=True) == 0


@functools.lru_cache(maxsize=None)
def _kat32(N, K):
    # Row i of the generator does not depend on M, so the 32-row answer
    # serves every M <= 32.
    return kat(32, N, K)


@pytest.mark.parametrize("chunks", [None, 1, 3, 8, 64])
@pytest.mark.parametrize("M", [1, 5, 16, 17, 32])
@pytest.mark.parametrize("N,K", [(14336, 4096), (9416, 1000), (18816, 136), (1001, 520), (128, 64),
                                 (300, 4104)])
def test_chunked_exact(dev, cudair, M, N, K, chunks):
    # Every chunk count from one chunk per tile (no partial sums) to one per
    # k-block, ragged N and K, twice in a row from the same C (bit-identical:
    # which CTA ran which chunk does not matter), and C's padding untouched.
    import torch
    from cudair import kernels
    if chunks is not None:
        os.environ["CUDAIR_FEWROWS_CHUNKS"] = str(chunks)
    af, bf, c, want = _kat32(N, K)
    af, c, want = af[:M], c[:M], want[:M]
    da = _dev(af, dev, torch.float16)
    B = torch.zeros(K, (N + 7) // 8 * 8, dtype=torch.float16, device=dev)
    B[:, :N] = _dev(bf, dev, torch.float16)
    db = B[:, :N]
    ldc = N + 4
    for _ in range(2):
        C = torch.full((M, ldc), -9.0, dtype=torch.float32, device=dev)
        C[:, :N] = _dev(c, dev, torch.float32)
        kernels.gemm(da, db, C[:, :N])
        got = C.cpu().numpy()
        bad = np.argwhere(got[:, :N] != want)
        assert bad.size == 0, (len(bad), tuple(bad[0]))
        assert np.all(got[:, N:] == -9.0)


@functools.lru_cache(maxsize=None)
def _kat64(N, K):
    return kat(64, N, K)


@pytest.mark.parametrize("chunks", [None, 3, 64])
@pytest.mark.parametrize("M", [33, 48, 64])
@pytest.mark.parametrize("N,K", [(14336, 4096), (1001, 520), (300, 4104), (128, 64)])
def test_chunked_exact_wide(dev, cudair, M, N, K, chunks):
    # 33 to 64 rows: the accumulator stays in TMEM and is read 16 rows at a
    # time where it is needed.  Exact, twice from the same C, padding untouched.
    import torch
    from cudair import kernels
    if chunks is not None:
        os.environ["CUDAIR_FEWROWS_CHUNKS"] = str(chunks)
    af, bf, c, want = _kat64(N, K)
    af, c, want = af[:M], c[:M], want[:M]
    da = _dev(af, dev, torch.float16)
    B = torch.zeros(K, (N + 7) // 8 * 8, dtype=torch.float16, device=dev)
    B[:, :N] = _dev(bf, dev, torch.float16)
    ldc = N + 4
    for _ in range(2):
        C = torch.full((M, ldc), -9.0, dtype=torch.float32, device=dev)
        C[:, :N] = _dev(c, dev, torch.float32)
        kernels.gemm(da, B[:, :N], C[:, :N])
        got = C.cpu().numpy()
        bad = np.argwhere(got[:, :N] != want)
        assert bad.size == 0, (len(bad), tuple(bad[0]))
        assert np.all(got[:, N:] == -9.0)


@pytest.mark.parametrize("M", [16, 64])
@pytest.mark.parametrize("pdl", [0, 1, 2])
def test_chunked_chain_of_launches(dev, cudair, pdl, M):
    # Twenty launches back to back on one stream, with programmatic dependent
    # launch off, on, and on with B requested early: each launch must find the
    # ticket reset by the one before.  Integer data: C + 20 A.B exactly.
    import torch
    from cudair import kernels
    kernels.set_gemm_pdl(pdl)
    N, K = 14336, 4096
    af, bf, c, want = _kat64(N, K)
    af, c, want = af[:M], c[:M], want[:M]
    da, db = _dev(af, dev, torch.float16), _dev(bf, dev, torch.float16)
    dc = _dev(c, dev, torch.float32)
    for _ in range(20):
        kernels.gemm(da, db, dc)
    prod = want.astype(np.int64) - c.astype(np.int64)
    assert np.array_equal(dc.cpu().numpy(), (c.astype(np.int64) + 20 * prod).astype(np.float32))


@pytest.mark.parametrize("M", [16, 64])
def test_chunked_decode_shape_seeded(dev, cudair, oracle, M):
    # M x 14336 x 4096: A ~ N(0,1), B ~ N(0,0.02), C ~ U(-1,1), against the
    # oracle within tolerance, and the same bits on a second run.
    import torch
    from cudair import kernels
    N, K = 14336, 4096
    a16, af = _seeded_normal_f16(oracle, M * K, 9, 1.0)
    b16, bf = _seeded_normal_f16(oracle, K * N, 10, 0.02)
    c = oracle.uniform(M * N, 63).reshape(M, N)
    da = torch.from_numpy(a16.view(np.int16)).to(dev).view(torch.float16).reshape(M, K)
    db = torch.from_numpy(b16.view(np.int16)).to(dev).view(torch.float16).reshape(K, N)
    outs = []
    for _ in range(2):
        dc = torch.from_numpy(c.copy()).to(dev)
        kernels.gemm(da, db, dc)
        outs.append(dc.cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    want = oracle.gemm_ikj(af.reshape(M, K), bf.reshape(K, N), c)
    tol_rel, tol_max = oracle.gemm_tolerance(K, np.abs(af).max(), np.abs(bf).max())
    rel, mx, bad = oracle.error_norms(outs[0], want)
    assert bad == 0 and rel <= tol_rel and mx <= tol_max, (rel, mx)


def test_chunked_refuses_other_forms(dev, cudair):
    import torch
    from cudair import kernels
    a = torch.zeros(65, 64, dtype=torch.float16, device=dev)
    b = torch.zeros(64, 128, dtype=torch.float16, device=dev)
    c = torch.zeros(65, 128, dtype=torch.float32, device=dev)
    with pytest.raises(Exception, match="M <= 64"):
        kernels.gemm(a, b, c)
    with pytest.raises(Exception, match="plain form"):
        kernels.gemm_ex(a[:16], b, c[:16], overwrite=True)


@pytest.mark.parametrize("M,N,K", [(16, 128, 4096), (1, 128, 8192), (32, 296, 2048), (7, 256, 1000),
                                   (64, 128, 4096), (48, 256, 2048), (64, 4096, 4096), (40, 2048, 2048)])
def test_automatic_choice_takes_chunked(dev, cudair, oracle, M, N, K):
    # Fewer (128-column x 64-k) units than SMs at M <= 64: the automatic
    # choice cuts K into chunks on the chunked kernel instead of streaming all
    # of K through one SM; with more units at 33 to 64 rows it also takes the
    # chunked kernel.  Exact on the integer generator; on seeded data the
    # same bits as the chunked kernel chosen explicitly (so that kernel ran)
    # and within the oracle's tolerance.
    import torch
    from cudair import kernels
    af, bf, c, want = kat(M, N, K)
    kernels.set_gemm_variant(0)
    dc = _dev(c, dev, torch.float32)
    kernels.gemm(_dev(af, dev, torch.float16), _dev(bf, dev, torch.float16), dc)
    assert np.array_equal(dc.cpu().numpy(), want)

    a16, a32 = _seeded_normal_f16(oracle, M * K, 21, 1.0)
    b16, b32 = _seeded_normal_f16(oracle, K * N, 22, 0.05)
    c = oracle.uniform(M * N, 23).reshape(M, N)
    da = torch.from_numpy(a16.view(np.int16)).to(dev).view(torch.float16).reshape(M, K)
    db = torch.from_numpy(b16.view(np.int16)).to(dev).view(torch.float16).reshape(K, N)
    outs = []
    for variant in (0, 6):
        kernels.set_gemm_variant(variant)
        dc = torch.from_numpy(c.copy()).to(dev)
        kernels.gemm(da, db, dc)
        outs.append(dc.cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    want = oracle.gemm_ikj(a32.reshape(M, K), b32.reshape(K, N), c)
    tol_rel, tol_max = oracle.gemm_tolerance(K, np.abs(a32).max(), np.abs(b32).max())
    rel, mx, bad = oracle.error_norms(outs[0], want)
    assert bad == 0 and rel <= tol_rel and mx <= tol_max, (rel, mx)
