"""cudair_gemm_f16f32_host: the MatMul16 test flow (copy A, B, C in; launch;
copy C back; advanced_test.go:466-483) as one pipelined call from host
buffers.  Exact on the reference's integer generator, identical to the
device-buffer call on seeded data, correct with padded host pitches, ragged
row blocks and pageable host memory, and ordered after earlier work on the
caller's stream."""
import numpy as np
import pytest

from test_matmul16_gpu import _seeded_normal_f16, kat

pytestmark = pytest.mark.gpu


def _pinned(x, dtype):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).pin_memory()


@pytest.mark.parametrize("M,N,K,rpb", [(1000, 520, 200, 256), (300, 1024, 64, 0), (64, 136, 520, 0),
                                       (2048, 256, 1024, 512)])
def test_gemm_host_kat_exact(dev, cudair, M, N, K, rpb):
    import torch
    from cudair import kernels
    af, bf, c, want = kat(M, N, K)
    a_h, b_h, c_h = _pinned(af, torch.float16), _pinned(bf, torch.float16), _pinned(c, torch.float32)
    a_d = torch.empty(M, K, dtype=torch.float16, device=dev)
    b_d = torch.empty(K, N, dtype=torch.float16, device=dev)
    c_d = torch.empty(M, N, dtype=torch.float32, device=dev)
    kernels.gemm_host(a_h, b_h, c_h, a_d, b_d, c_d, rows_per_block=rpb)
    torch.cuda.synchronize()
    assert np.array_equal(c_h.numpy(), want)


def test_gemm_host_padded_pitches_and_pageable(dev, cudair):
    # Host rows longer than the matrices (lda, ldb, ldc > K, N, N); the
    # padding is neither read into the result nor written.  Pageable memory.
    import torch
    from cudair import kernels
    M, N, K = 700, 264, 136
    af, bf, c, want = kat(M, N, K)
    A = torch.full((M, K + 8), 9.0, dtype=torch.float16)
    B = torch.full((K, N + 16), 9.0, dtype=torch.float16)
    C = torch.full((M, N + 3), -2.0, dtype=torch.float32)
    A[:, :K] = torch.from_numpy(af).half()
    B[:, :N] = torch.from_numpy(bf).half()
    C[:, :N] = torch.from_numpy(c)
    a_d = torch.empty(M, K, dtype=torch.float16, device=dev)
    b_d = torch.empty(K, N, dtype=torch.float16, device=dev)
    c_d = torch.empty(M, N, dtype=torch.float32, device=dev)
    kernels.gemm_host(A[:, :K], B[:, :N], C[:, :N], a_d, b_d, c_d, rows_per_block=256)
    torch.cuda.synchronize()
    got = C.numpy()
    assert np.array_equal(got[:, :N], want)
    assert np.all(got[:, N:] == -2.0)


def test_gemm_host_matches_device_call(dev, cudair, oracle):
    # Same kernels, same blocks of rows: bit-identical to cudair_gemm_f16f32
    # on device copies of the same operands, and within the GEMM tolerance
    # of the fp32 oracle on sampled rows.
    import torch
    from cudair import kernels
    M, N, K = 2048, 1024, 2048
    a16, af = _seeded_normal_f16(oracle, M * K, 71, 1.0 / np.sqrt(K))
    b16, bf = _seeded_normal_f16(oracle, K * N, 72, 1.0 / np.sqrt(K))
    c = oracle.normal(M * N, 73).reshape(M, N)
    a_h = torch.from_numpy(a16.view(np.int16)).view(torch.float16).reshape(M, K).pin_memory()
    b_h = torch.from_numpy(b16.view(np.int16)).view(torch.float16).reshape(K, N).pin_memory()
    c_h = torch.from_numpy(c.copy()).pin_memory()
    a_d = torch.empty(M, K, dtype=torch.float16, device=dev)
    b_d = torch.empty(K, N, dtype=torch.float16, device=dev)
    c_d = torch.empty(M, N, dtype=torch.float32, device=dev)
    kernels.gemm_host(a_h, b_h, c_h, a_d, b_d, c_d, rows_per_block=512)
    torch.cuda.synchronize()
    ref = torch.from_numpy(c.copy()).to(dev)
    da, db = a_h.to(dev), b_h.to(dev)
    for r0 in range(0, M, 512):
        kernels.gemm(da[r0:r0 + 512], db, ref[r0:r0 + 512])
    torch.cuda.synchronize()
    got = c_h.numpy()
    assert np.array_equal(got.view(np.uint32), ref.cpu().numpy().view(np.uint32))
    tol_rel, tol_max = oracle.gemm_tolerance(K, np.abs(af).max(), np.abs(bf).max())
    af2, bf2 = af.reshape(M, K), bf.reshape(K, N)
    for r in (0, 511, 512, 1500, M - 1):
        want = oracle.gemm_ikj(af2, bf2, c, rows=(r, r + 1))
        rel, mx, bad = oracle.error_norms(got[r:r + 1], want)
        assert bad == 0 and rel <= tol_rel and mx <= tol_max, (r, rel, mx)


def test_gemm_host_waits_for_earlier_work_on_the_stream(dev, cudair):
    # The device buffers are still being written by earlier work on the
    # caller's stream when the call is made: its copies in must wait for it.
    import torch
    from cudair import kernels
    M, N, K = 512, 512, 256
    af, bf, c, want = kat(M, N, K)
    a_h, b_h, c_h = _pinned(af, torch.float16), _pinned(bf, torch.float16), _pinned(c, torch.float32)
    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        a_d = torch.empty(M, K, dtype=torch.float16, device=dev)
        b_d = torch.empty(K, N, dtype=torch.float16, device=dev)
        c_d = torch.empty(M, N, dtype=torch.float32, device=dev)
        big = torch.randn(4096, 4096, device=dev)
        for _ in range(4):
            big = big @ big  # keeps the stream busy
        c_d.fill_(123.0)  # earlier writer of c_d
        kernels.gemm_host(a_h, b_h, c_h, a_d, b_d, c_d, stream=s)
    s.synchronize()
    assert np.array_equal(c_h.numpy(), want)


def test_gemm_host_with_b_already_on_device(dev, cudair):
    # b_host = NULL: B is taken from b_dev (replicated there beforehand), only
    # A and C cross the host link.
    import torch
    from cudair import kernels
    M, N, K = 1000, 520, 200
    af, bf, c, want = kat(M, N, K)
    a_h, c_h = _pinned(af, torch.float16), _pinned(c, torch.float32)
    a_d = torch.empty(M, K, dtype=torch.float16, device=dev)
    b_d = torch.from_numpy(bf).to(dev).half()
    c_d = torch.empty(M, N, dtype=torch.float32, device=dev)
    kernels.gemm_host(a_h, None, c_h, a_d, b_d, c_d, rows_per_block=256)
    torch.cuda.synchronize()
    assert np.array_equal(c_h.numpy(), want)


# With B from the host, N >= 4096 and M >= 1024, the default schedule tiles C
# in both dimensions (about 4 x 4 tiles): B crosses the link one column block
# at a time, A one row block at a time on the first column pass.

@pytest.mark.parametrize("M,N,K", [(1100, 4104, 72), (1024, 4096, 200), (2000, 8192, 16)])
def test_gemm_host_2d_tiles_kat_exact(dev, cudair, M, N, K):
    # Ragged in both dimensions (1100 rows in blocks of 512; 4104 columns in
    # blocks of 1280, the last 264 wide).
    import torch
    from cudair import kernels
    af, bf, c, want = kat(M, N, K)
    a_h, b_h, c_h = _pinned(af, torch.float16), _pinned(bf, torch.float16), _pinned(c, torch.float32)
    a_d = torch.empty(M, K, dtype=torch.float16, device=dev)
    b_d = torch.empty(K, N, dtype=torch.float16, device=dev)
    c_d = torch.empty(M, N, dtype=torch.float32, device=dev)
    kernels.gemm_host(a_h, b_h, c_h, a_d, b_d, c_d)
    torch.cuda.synchronize()
    assert np.array_equal(c_h.numpy(), want)
    # The device copies hold the operands and the result, as after the
    # reference test's copy-in / launch.
    assert np.array_equal(c_d.cpu().numpy(), want)
    assert torch.equal(b_d.cpu(), b_h)


def test_gemm_host_2d_tiles_padded_pitches_and_pageable(dev, cudair):
    import torch
    from cudair import kernels
    M, N, K = 1030, 4360, 136
    af, bf, c, want = kat(M, N, K)
    A = torch.full((M, K + 8), 9.0, dtype=torch.float16)
    B = torch.full((K, N + 16), 9.0, dtype=torch.float16)
    C = torch.full((M, N + 3), -2.0, dtype=torch.float32)
    A[:, :K] = torch.from_numpy(af).half()
    B[:, :N] = torch.from_numpy(bf).half()
    C[:, :N] = torch.from_numpy(c)
    a_d = torch.empty(M, K, dtype=torch.float16, device=dev)
    b_d = torch.empty(K, N, dtype=torch.float16, device=dev)
    c_d = torch.empty(M, N, dtype=torch.float32, device=dev)
    kernels.gemm_host(A[:, :K], B[:, :N], C[:, :N], a_d, b_d, c_d)
    torch.cuda.synchronize()
    got = C.numpy()
    assert np.array_equal(got[:, :N], want)
    assert np.all(got[:, N:] == -2.0)


def test_gemm_host_2d_tiles_match_device_call(dev, cudair, oracle):
    # Seeded data at 4096^3: the tiled host call agrees with one device-buffer
    # GEMM of the whole problem within the GEMM tolerance (each tile is
    # computed by the same kernels over the whole K).
    import torch
    from cudair import kernels
    M = N = K = 4096
    a16, _ = _seeded_normal_f16(oracle, M * K, 81, 1.0 / 64)
    b16, _ = _seeded_normal_f16(oracle, K * N, 82, 1.0 / 64)
    c = oracle.normal(M * N, 83).reshape(M, N)
    a_h = torch.from_numpy(a16.view(np.int16)).view(torch.float16).reshape(M, K).pin_memory()
    b_h = torch.from_numpy(b16.view(np.int16)).view(torch.float16).reshape(K, N).pin_memory()
    c_h = torch.from_numpy(c.copy()).pin_memory()
    a_d = torch.empty(M, K, dtype=torch.float16, device=dev)
    b_d = torch.empty(K, N, dtype=torch.float16, device=dev)
    c_d = torch.empty(M, N, dtype=torch.float32, device=dev)
    kernels.gemm_host(a_h, b_h, c_h, a_d, b_d, c_d)
    torch.cuda.synchronize()
    a2, b2, c2 = a_h.to(dev), b_h.to(dev), torch.from_numpy(c).to(dev)
    kernels.gemm(a2, b2, c2)
    torch.cuda.synchronize()
    got, ref = c_h.to(dev), c2
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel <= 1e-6, rel
