"""MatMul16 on the B200: C = A.B + C with fp16 A, B and fp32 C.

Exact where the reference test is exact (small-integer operands: every
product and partial sum is an integer below 2^24, so any correct fp32
evaluation gives the int64 answer) and within the stated tolerance on seeded
real-valued data:
  relative Frobenius error <= 1e-3 and
  max |error| <= 5e-3 * sqrt(K) * max|a| * max|b|
against the fp32 CPU oracle on the fp16-rounded inputs.
"""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def module(dev, cudair):
    from cudair import host
    m = host.LoadModule(host.KernelsImage())
    yield m
    m.Close()


@pytest.fixture(autouse=True)
def no_wait_timeouts(dev, cudair):
    from cudair import kernels
    kernels.wait_status(clear=True)
    yield
    assert kernels.wait_status(clear=True) == 0


@pytest.fixture(params=[1, 2, 3, 4, 5, 6], ids=["single", "pair", "fewrows", "pairwide", "small", "chunked"])
def variant(request, dev, cudair):
    """Runs a test on each GEMM kernel in turn: single CTA (128x256 tiles),
    CTA pair (256x256), the few-row kernel (M <= 128), the wide CTA pair
    (256x512), the small-problem kernel (K <= 512, one 128x64 tile per CTA)
    and the chunked few-row kernel (M <= 64), then restores the automatic
    choice."""
    from cudair import kernels
    kernels.set_gemm_variant(request.param)
    yield request.param
    kernels.set_gemm_variant(0)


def _applies(variant, M, K=0):
    if variant == 3 and M > 128:
        pytest.skip("the few-row kernel takes M <= 128")
    if variant == 5 and K > 512:
        pytest.skip("the small-problem kernel takes K <= 512")
    if variant == 6 and M > 64:
        pytest.skip("the chunked few-row kernel takes M <= 64")


def kat(M, N, K):
    """The TestHopper generator (advanced_test.go:459-463) on an M x K / K x N
    grid: af = (i+2j)%7-3, bf = (3i+j)%5-2, c = j-i."""
    i = np.arange(M).reshape(M, 1)
    k = np.arange(K).reshape(1, K)
    af = ((i + 2 * k) % 7 - 3)
    kk = np.arange(K).reshape(K, 1)
    j = np.arange(N).reshape(1, N)
    bf = ((3 * kk + j) % 5 - 2)
    c = (j - i)
    want = (af.astype(np.int64) @ bf.astype(np.int64) + c).astype(np.float32)
    return af.astype(np.float32), bf.astype(np.float32), c.astype(np.float32), want


def _dev(x, dev, dtype):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev).to(dtype)


def test_matmul16_reference_launch_kat64(dev, module, oracle, golden_dir):
    # TestHopper/MatMul16: n = 64, grid (n/16, n/16), 32 threads, exact ==.
    import torch
    from cudair import host
    n = 64
    af, bf, c = oracle.matmul16_kat(n)
    want = np.load(os.path.join(golden_dir, "matmul16_kat64.npz"))["want"]
    a16 = oracle.f32_to_f16(af)
    b16 = oracle.f32_to_f16(bf)
    da = torch.from_numpy(a16.view(np.int16)).to(dev)
    db = torch.from_numpy(b16.view(np.int16)).to(dev)
    dc = torch.from_numpy(c).to(dev)
    torch.cuda.synchronize()
    module.Function("MatMul16").LaunchEx(
        host.LaunchConfig(GridX=n // 16, GridY=n // 16, BlockX=32), host.LaunchAttrs(),
        host.ArgBuffer(da), host.ArgBuffer(db), host.ArgBuffer(dc), host.ArgValue(ctypes.c_int32(n)))
    got = dc.cpu().numpy()
    assert np.array_equal(got, want)
    assert np.array_equal(got, oracle.matmul16(af, bf, c))


def test_matmul16_reference_launch_seeded_n256(dev, module, oracle, golden_dir):
    import torch
    from cudair import host
    n = 256
    a16 = oracle.f32_to_f16(oracle.uniform(n * n, 1)).reshape(n, n)
    b16 = oracle.f32_to_f16(oracle.uniform(n * n, 2)).reshape(n, n)
    c = oracle.uniform(n * n, 3).reshape(n, n)
    af, bf = oracle.f16_to_f32(a16), oracle.f16_to_f32(b16)
    dc = torch.from_numpy(c).to(dev)
    da = torch.from_numpy(a16.view(np.int16)).to(dev)
    db = torch.from_numpy(b16.view(np.int16)).to(dev)
    torch.cuda.synchronize()
    module.Function("MatMul16").LaunchEx(
        host.LaunchConfig(GridX=n // 16, GridY=n // 16, BlockX=32), host.LaunchAttrs(),
        host.ArgBuffer(da), host.ArgBuffer(db), host.ArgBuffer(dc), host.ArgValue(ctypes.c_int32(n)))
    got = dc.cpu().numpy()
    want = oracle.matmul16(af, bf, c)
    golden = np.load(os.path.join(golden_dir, "matmul16_n256.npz"))["want"]
    tol_rel, tol_max = oracle.gemm_tolerance(n, np.abs(af).max(), np.abs(bf).max())
    for ref in (want, golden):
        rel, mx, bad = oracle.error_norms(got, ref)
        assert bad == 0 and rel <= tol_rel and mx <= tol_max, (rel, mx)


@pytest.mark.parametrize("n", [64, 256, 512, 1024, 2048])
def test_matmul16_tcgen05_kat_exact(dev, cudair, variant, n):
    import torch
    from cudair import kernels
    _applies(variant, n, n)
    af, bf, c, want = kat(n, n, n)
    da, db, dc = _dev(af, dev, torch.float16), _dev(bf, dev, torch.float16), _dev(c, dev, torch.float32)
    kernels.matmul16(da, db, dc)
    got = dc.cpu().numpy()
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{len(bad)} mismatches, first at {tuple(bad[0])}: {got[tuple(bad[0])]} vs {want[tuple(bad[0])]}"


def test_matmul16_tcgen05_seeded_n256(dev, cudair, oracle, golden_dir):
    import torch
    from cudair import kernels
    n = 256
    a16 = oracle.f32_to_f16(oracle.uniform(n * n, 1)).reshape(n, n)
    b16 = oracle.f32_to_f16(oracle.uniform(n * n, 2)).reshape(n, n)
    c = oracle.uniform(n * n, 3).reshape(n, n)
    af, bf = oracle.f16_to_f32(a16), oracle.f16_to_f32(b16)
    da = torch.from_numpy(a16.view(np.int16)).to(dev).view(torch.float16)
    db = torch.from_numpy(b16.view(np.int16)).to(dev).view(torch.float16)
    dc = torch.from_numpy(c).to(dev)
    kernels.matmul16(da, db, dc)
    got = dc.cpu().numpy()
    want = oracle.matmul16(af, bf, c)
    golden = np.load(os.path.join(golden_dir, "matmul16_n256.npz"))["want"]
    tol_rel, tol_max = oracle.gemm_tolerance(n, np.abs(af).max(), np.abs(bf).max())
    for ref in (want, golden):
        rel, mx, bad = oracle.error_norms(got, ref)
        assert bad == 0 and rel <= tol_rel and mx <= tol_max, (rel, mx)


@pytest.mark.parametrize("M,N,K", [
    (1, 8, 8), (7, 16, 24), (128, 256, 64), (129, 264, 72), (200, 264, 136), (300, 1000, 1000),
    (513, 8, 4096), (16, 14336, 512), (1000, 2056, 520), (257, 136, 64), (384, 384, 8),
    (5, 136, 200), (33, 1000, 1000), (64, 2048, 8), (48, 520, 4104), (17, 128, 64),
    (65, 1000, 1032), (96, 2056, 520), (128, 4096, 2048), (113, 264, 8192),
])
def test_gemm_tcgen05_ragged_kat_exact(dev, cudair, variant, M, N, K):
    import torch
    from cudair import kernels
    _applies(variant, M, K)
    af, bf, c, want = kat(M, N, K)
    da, db, dc = _dev(af, dev, torch.float16), _dev(bf, dev, torch.float16), _dev(c, dev, torch.float32)
    kernels.gemm(da, db, dc)
    got = dc.cpu().numpy()
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{len(bad)} mismatches, first at {tuple(bad[0])}"


@pytest.mark.parametrize("M", [300, 40])
def test_gemm_tcgen05_padded_leading_dims(dev, cudair, variant, M):
    # lda, ldb, ldc larger than the logical widths; untouched padding.
    import torch
    from cudair import kernels
    _applies(variant, M)
    N, K = 520, 200
    af, bf, c, want = kat(M, N, K)
    A = torch.zeros(M, K + 24, dtype=torch.float16, device=dev)
    B = torch.zeros(K, N + 8, dtype=torch.float16, device=dev)
    C = torch.full((M, N + 12), -5.0, dtype=torch.float32, device=dev)
    A[:, :K] = _dev(af, dev, torch.float16)
    B[:, :N] = _dev(bf, dev, torch.float16)
    C[:, :N] = _dev(c, dev, torch.float32)
    kernels.gemm(A[:, :K], B[:, :N], C[:, :N])
    got = C.cpu().numpy()
    assert np.array_equal(got[:, :N], want)
    assert np.all(got[:, N:] == -5.0)


def _seeded_normal_f16(oracle, n, seed, std):
    h = oracle.f32_to_f16(oracle.normal(n, seed, 0.0, std))
    return h, oracle.f16_to_f32(h)


def test_gemm_8192_cube_seeded(dev, cudair, oracle, variant):
    # The 8192^3 configuration: A, B ~ fp16(N(0,1)/sqrt(8192)), C ~ N(0,1).
    import torch
    from cudair import kernels
    n = 8192
    _applies(variant, n, n)
    a16, af = _seeded_normal_f16(oracle, n * n, 6, 1.0 / np.sqrt(n))
    b16, bf = _seeded_normal_f16(oracle, n * n, 7, 1.0 / np.sqrt(n))
    c = oracle.normal(n * n, 8).reshape(n, n)
    af, bf = af.reshape(n, n), bf.reshape(n, n)
    da = torch.from_numpy(a16.view(np.int16)).to(dev).view(torch.float16).reshape(n, n)
    db = torch.from_numpy(b16.view(np.int16)).to(dev).view(torch.float16).reshape(n, n)
    dc = torch.from_numpy(c).to(dev)
    kernels.gemm(da, db, dc)
    torch.cuda.synchronize()
    got = dc.cpu().numpy()
    tol_rel, tol_max = oracle.gemm_tolerance(n, np.abs(af).max(), np.abs(bf).max())
    # (1) whole matrix against an fp32 GPU reference of the same op.
    ref = (da.float() @ db.float()).add_(torch.from_numpy(c).to(dev)).cpu().numpy()
    rel, mx, bad = oracle.error_norms(got, ref)
    assert bad == 0 and rel <= tol_rel and mx <= tol_max, (rel, mx)
    # (2) rows against the CPU oracle (fp32): every 257th row (each 256-row
    # pair tile and 128-row CTA half hit at a different offset) and both
    # sides of the tile boundaries at the start, middle and end.
    edges = [0, 1, 127, 128, 255, 256, 511, 512, n // 2 - 1, n // 2, n - 257, n - 256, n - 129, n - 128,
             n - 2, n - 1]
    rows = np.unique(np.concatenate([np.arange(0, n, 257), edges]))
    want = oracle.gemm_ikj(np.ascontiguousarray(af[rows]), bf, np.ascontiguousarray(c[rows]))
    for i, r in enumerate(rows):
        rel, mx, bad = oracle.error_norms(got[r:r + 1], want[i:i + 1])
        assert bad == 0 and rel <= tol_rel and mx <= tol_max, (r, rel, mx)


def test_gemm_skinny_decode_shape(dev, cudair, oracle):
    # M=16, N=14336, K=4096: A ~ N(0,1), B ~ N(0,0.02), C = 0.
    import torch
    from cudair import kernels
    M, N, K = 16, 14336, 4096
    a16, af = _seeded_normal_f16(oracle, M * K, 9, 1.0)
    b16, bf = _seeded_normal_f16(oracle, K * N, 10, 0.02)
    af, bf = af.reshape(M, K), bf.reshape(K, N)
    c = np.zeros((M, N), dtype=np.float32)
    da = torch.from_numpy(a16.view(np.int16)).to(dev).view(torch.float16).reshape(M, K)
    db = torch.from_numpy(b16.view(np.int16)).to(dev).view(torch.float16).reshape(K, N)
    dc = torch.zeros(M, N, dtype=torch.float32, device=dev)
    kernels.gemm(da, db, dc)
    got = dc.cpu().numpy()
    want = oracle.gemm_ikj(af, bf, c)
    tol_rel, tol_max = oracle.gemm_tolerance(K, np.abs(af).max(), np.abs(bf).max())
    rel, mx, bad = oracle.error_norms(got, want)
    assert bad == 0 and rel <= tol_rel and mx <= tol_max, (rel, mx)


@pytest.mark.parametrize("M", [256, 16])
def test_gemm_repeated_calls_accumulate(dev, cudair, variant, M):
    # C = A.B + C is not idempotent: two calls add the product twice.
    import torch
    from cudair import kernels
    _applies(variant, M)
    N, K = 512, 320
    af, bf, c, want1 = kat(M, N, K)
    da, db, dc = _dev(af, dev, torch.float16), _dev(bf, dev, torch.float16), _dev(c, dev, torch.float32)
    kernels.gemm(da, db, dc)
    kernels.gemm(da, db, dc)
    want2 = want1 + (want1 - c)
    assert np.array_equal(dc.cpu().numpy(), want2)


@pytest.mark.parametrize("M,N,K", [(16, 14336, 4096), (3, 4096, 12288), (64, 1024, 520),
                                   (128, 8192, 2048), (100, 1000, 4104)])
def test_fewrows_deterministic_and_within_tolerance(dev, cudair, oracle, M, N, K):
    # The split-K fix-up sums partials in a fixed order: two runs from the
    # same C give identical bits, and both match the oracle within tolerance.
    import torch
    from cudair import kernels
    a16, af = _seeded_normal_f16(oracle, M * K, 61, 1.0)
    b16, bf = _seeded_normal_f16(oracle, K * N, 62, 0.02)
    c = oracle.uniform(M * N, 63).reshape(M, N)
    da = torch.from_numpy(a16.view(np.int16)).to(dev).view(torch.float16).reshape(M, K)
    db = torch.from_numpy(b16.view(np.int16)).to(dev).view(torch.float16).reshape(K, N)
    outs = []
    kernels.set_gemm_variant(3)  # the few-row kernel, whatever the automatic choice
    try:
        for _ in range(2):
            dc = torch.from_numpy(c.copy()).to(dev)
            kernels.gemm(da, db, dc)
            outs.append(dc.cpu().numpy())
    finally:
        kernels.set_gemm_variant(0)
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    want = oracle.gemm_ikj(af.reshape(M, K), bf.reshape(K, N), c)
    tol_rel, tol_max = oracle.gemm_tolerance(K, np.abs(af).max(), np.abs(bf).max())
    rel, mx, bad = oracle.error_norms(outs[0], want)
    assert bad == 0 and rel <= tol_rel and mx <= tol_max, (rel, mx)


@pytest.mark.parametrize("c_offset,ldc_pad", [(0, 2), (1, 0), (3, 5)], ids=["odd-n", "c+4B", "c+12B-odd-ldc"])
def test_gemm_c_layouts(dev, cudair, variant, c_offset, ldc_pad):
    # C views the reduce-add epilogue must clip (N not a multiple of 4) or
    # cannot describe (a base or row pitch not on 16 bytes: scalar path).
    # Elements of C outside the view keep their value.
    import torch
    from cudair import kernels
    M = 40 if variant == 3 else (24 if variant == 6 else 300)
    N, K = 101, 136
    af, bf, c, want = kat(M, N, K)
    A = _dev(af, dev, torch.float16)
    B = torch.zeros(K, 104, dtype=torch.float16, device=dev)
    B[:, :N] = _dev(bf, dev, torch.float16)
    ldc = N + ldc_pad
    flat = torch.full((c_offset + M * ldc + 8,), -7.0, dtype=torch.float32, device=dev)
    C = flat[c_offset:c_offset + M * ldc].view(M, ldc)[:, :N]
    C.copy_(_dev(c, dev, torch.float32))
    kernels.gemm(A, B[:, :N], C)
    got = flat.cpu().numpy()
    body = got[c_offset:c_offset + M * ldc].reshape(M, ldc)
    assert np.array_equal(body[:, :N], want)
    assert np.all(body[:, N:] == -7.0)
    assert np.all(got[:c_offset] == -7.0) and np.all(got[c_offset + M * ldc:] == -7.0)


@pytest.mark.parametrize("variant_id", [0, 4], ids=["auto", "pairwide"])
def test_gemm_c_beyond_2p31_elements(dev, cudair, variant_id):
    # C with more than 2^31 elements (65600 x 32776 fp32 = 8.6 GB): no 32-bit
    # index overflows in the tiles, the tensor-map coordinates or the
    # epilogue.  Integer operands (exact); rows around the 2^31-element
    # boundary, the ragged last tile and the last row are checked against
    # int64 products.
    import torch
    from cudair import kernels
    M, N, K = 65600, 32776, 64
    i = torch.arange(M, device=dev, dtype=torch.int32).view(M, 1)
    k = torch.arange(K, device=dev, dtype=torch.int32).view(1, K)
    a = ((i + 2 * k) % 7 - 3).half()
    kk = torch.arange(K, device=dev, dtype=torch.int32).view(K, 1)
    j = torch.arange(N, device=dev, dtype=torch.int32).view(1, N)
    b = ((3 * kk + j) % 5 - 2).half()
    c = (j - i).float()  # c[i][j] = j - i, as the reference's generator
    kernels.set_gemm_variant(variant_id)
    try:
        kernels.gemm(a, b, c)
        torch.cuda.synchronize()
    finally:
        kernels.set_gemm_variant(0)
    boundary = (1 << 31) // N
    rows = sorted({0, 1, boundary - 1, boundary, boundary + 1, M - 65, M - 64, M - 2, M - 1})
    bf = b.cpu().numpy().astype(np.int64)
    for r in rows:
        ar = a[r].cpu().numpy().astype(np.int64)
        want = ar @ bf + (np.arange(N, dtype=np.int64) - r)
        got = c[r].cpu().numpy()
        assert np.array_equal(got, want.astype(np.float32)), r
    del a, b, c
    torch.cuda.empty_cache()


@pytest.mark.parametrize("M", [1, 16, 40, 64])
@pytest.mark.parametrize("kb", [2, 3, 4, 5, 6, 8, 16])
def test_fewrows_contributors_per_tile(dev, cudair, M, kb):
    # With fewer 64-wide k-blocks than SMs, every k-block has its own CTA, so
    # each 128-column tile has exactly kb contributors; their parts must all
    # be summed, whichever contributor finishes last.  Exact (integer data),
    # twice in a row from the same C (bit-identical, timing-independent).
    # N = 1001 in a C of pitch 1004: 16-byte aligned rows with a ragged last
    # tile (the fix-up's staged copies of C end in a partial 16-byte piece).
    import torch
    from cudair import kernels
    kernels.set_gemm_variant(3)  # the few-row kernel, whatever the automatic choice
    try:
        for N, ldc in ((128, 128), (264, 264), (1001, 1004)):
            K = 64 * kb
            af, bf, c, want = kat(M, N, K)
            da = _dev(af, dev, torch.float16)
            B = torch.zeros(K, (N + 7) // 8 * 8, dtype=torch.float16, device=dev)
            B[:, :N] = _dev(bf, dev, torch.float16)
            for _ in range(2):
                C = torch.full((M, ldc), -9.0, dtype=torch.float32, device=dev)
                C[:, :N] = _dev(c, dev, torch.float32)
                kernels.gemm(da, B[:, :N], C[:, :N])
                got = C.cpu().numpy()
                assert np.array_equal(got[:, :N], want), (N, K)
                assert np.all(got[:, N:] == -9.0)
    finally:
        kernels.set_gemm_variant(0)


@pytest.mark.parametrize("M", [1, 5, 16, 40, 64])
@pytest.mark.parametrize("N,K", [(14336, 4096), (9416, 1000), (18816, 136), (12000, 64), (10000, 4104)])
def test_fewrows_fewer_tiles_than_sms(dev, cudair, M, N, K):
    # The few-row kernel on shapes with fewer 128-column tiles than SMs, so
    # that some CTAs' ranges lie inside one tile and a tile can have two
    # contributors finishing together: the decode shape, ragged N and K, K of
    # a single k-block, N with 74 to 147 tiles.  Exact (integer data), twice
    # in a row from the same C (bit-identical), and C's padding columns
    # untouched.
    import torch
    from cudair import kernels
    kernels.set_gemm_variant(3)
    try:
        af, bf, c, want = kat(M, N, K)
        da = _dev(af, dev, torch.float16)
        db = _dev(bf, dev, torch.float16)
        ldc = N + 4
        for _ in range(2):
            C = torch.full((M, ldc), -9.0, dtype=torch.float32, device=dev)
            C[:, :N] = _dev(c, dev, torch.float32)
            kernels.gemm(da, db, C[:, :N])
            got = C.cpu().numpy()
            bad = np.argwhere(got[:, :N] != want)
            assert bad.size == 0, (N, K, len(bad), tuple(bad[0]))
            assert np.all(got[:, N:] == -9.0)
    finally:
        kernels.set_gemm_variant(0)
