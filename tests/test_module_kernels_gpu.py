"""The rest of the module's reference-named kernels on the B200, loaded and
launched the way the reference's tests do, with the same known answers:

  TestHopper (advanced_test.go:355-548): Cluster, MBarrier, TMA, Elect,
      GridDep, StMatrix
  TestTensorMap (hostapi_test.go:472-623): TensorTile2D, OutOfBounds
  TestLaunchEx (hostapi_test.go:360-466): RuntimeClusterDims,
      ProgrammaticDependentLaunch, Cooperative
  examples/vecadd/run/main.go:62-76: Saxpy, Square
  TestTensor (tensor_test.go:23-326): MmaF16, MmaF16Bias, MmaF16Trans,
      MmaF16Half, MmaBF16, MmaTF32, MmaTF32Trans, MmaS8, MmaU8,
      LdMatrixRegs, MmaLdMatrix, WmmaBF16, WmmaBF16Trans, WmmaTF32, WmmaS8,
      WmmaU8
  TestAdvanced/Wmma (advanced_test.go:25-80): Wmma, WmmaTrans
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BLOCKS, BS = 8, 256


@pytest.fixture(scope="module")
def mod(dev, cudair):
    from cudair import host
    m = host.LoadModule(host.KernelsImage())
    yield m
    m.Close()


def up(dev, arr):
    import torch
    return torch.from_numpy(np.ascontiguousarray(arr)).to(dev)


def launch(mod, name, cfg, *args, attrs=None):
    from cudair import host
    import torch
    torch.cuda.synchronize()
    mod.Function(name).LaunchEx(cfg, attrs or host.LaunchAttrs(), *args)


def cfg1d(n, bs):
    from cudair import host
    return host.LaunchConfig1D(n, bs)


# ---- TestHopper ----------------------------------------------------------------

def test_cluster_exchange(dev, mod):
    from cudair import host
    dout = up(dev, np.zeros(BLOCKS * BS, np.int32))
    dinfo = up(dev, np.zeros(BLOCKS, np.int32))
    launch(mod, "ClusterExchange", cfg1d(BLOCKS * BS, BS), host.ArgBuffer(dout), host.ArgBuffer(dinfo))
    out, info = dout.cpu().numpy(), dinfo.cpu().numpy()
    i = np.arange(BLOCKS * BS)
    b, tid = i // BS, i % BS
    assert np.array_equal(out, (b ^ 1) * 1000 + tid)
    bb = np.arange(BLOCKS)
    assert np.array_equal(info, bb % 2 + 10 * 2 + 100 * (bb // 2) + 1000 * BLOCKS // 2)


def test_mbarrier_sum(dev, mod):
    from cudair import host
    x = (np.arange(BLOCKS * BS) % 7).astype(np.int32)
    dout = up(dev, np.zeros(BLOCKS, np.int32))
    din = up(dev, x)
    launch(mod, "MBarrierSum", cfg1d(BLOCKS * BS, BS), host.ArgBuffer(din), host.ArgBuffer(dout))
    assert np.array_equal(dout.cpu().numpy(), x.reshape(BLOCKS, BS).sum(axis=1).astype(np.int32))


def test_tma_double(dev, mod):
    from cudair import host
    x = (np.arange(BLOCKS * BS) * 3 - 100).astype(np.int32)
    dout = up(dev, np.zeros(BLOCKS * BS, np.int32))
    din = up(dev, x)
    launch(mod, "TmaDouble", cfg1d(BLOCKS * BS, BS), host.ArgBuffer(din), host.ArgBuffer(dout),
           host.ArgValue(ctypes.c_int32(BLOCKS * BS)))
    assert np.array_equal(dout.cpu().numpy(), 2 * x)


def test_elect(dev, mod):
    from cudair import host
    dl = up(dev, np.zeros(BLOCKS * BS, np.int32))
    de = up(dev, np.zeros(BLOCKS * BS, np.int32))
    launch(mod, "Elect", cfg1d(BLOCKS * BS, BS), host.ArgBuffer(dl), host.ArgBuffer(de))
    leader, elected = dl.cpu().numpy().reshape(-1, 32), de.cpu().numpy().reshape(-1, 32)
    for w in range(leader.shape[0]):
        assert np.all(leader[w] == leader[w, 0])
        assert elected[w].sum() == 1 and elected[w, leader[w, 0]] == 1


def test_grid_dep(dev, mod):
    from cudair import host
    dout = up(dev, np.zeros(BLOCKS * BS, np.int32))
    launch(mod, "GridDep", cfg1d(BLOCKS * BS, BS), host.ArgBuffer(dout))
    assert np.array_equal(dout.cpu().numpy(), np.arange(BLOCKS * BS, dtype=np.int32))


def test_stmatrix_round_trip(dev, mod, oracle):
    from cudair import host
    inp = oracle.f32_to_f16(np.arange(1, 4 * 64 + 1, dtype=np.float32))
    dout = up(dev, np.zeros(11 * 64, np.uint16).view(np.int16))
    din = up(dev, inp.view(np.int16))
    launch(mod, "StMatrixRoundTrip", cfg1d(32, 32), host.ArgBuffer(din),
           host.ArgBuffer(dout))
    out = dout.cpu().numpy().view(np.uint16)
    assert np.array_equal(out[:256], inp)
    for off, mats in ((4 * 64, 4), (8 * 64, 2), (10 * 64, 1)):
        for m in range(mats):
            got = out[off + m * 64: off + (m + 1) * 64].reshape(8, 8)
            want = inp[m * 64:(m + 1) * 64].reshape(8, 8).T
            assert np.array_equal(got, want), (off, m)


# ---- TestTensorMap -------------------------------------------------------------

def _tile_double(dev, mod, w, h, grid, oob_fill):
    import torch
    from cudair import host
    src = (np.arange(w * h, dtype=np.float32) + 1) if oob_fill else \
        (np.arange(w, dtype=np.float32)[None, :] + 1000 * np.arange(h, dtype=np.float32)[:, None]).ravel()
    dsrc = up(dev, src.astype(np.float32))
    ddst = up(dev, np.zeros(w * h, np.float32))
    desc = host.TiledTensor(DataType=host.TensorMapFloat32, GlobalDim=[w, h], GlobalStrides=[w * 4],
                            BoxDim=[32, 32], OOBFill=host.OOBFillNaN if oob_fill else host.OOBFillNone)
    smap, dmap = host.EncodeTiled(dsrc, desc), host.EncodeTiled(ddst, desc)
    # The descriptors live in global memory, 128 bytes each.
    dsmap = torch.frombuffer(bytearray(smap.Bytes()), dtype=torch.uint8).to(dev)
    ddmap = torch.frombuffer(bytearray(dmap.Bytes()), dtype=torch.uint8).to(dev)
    launch(mod, "TensorTileDouble", host.LaunchConfig(GridX=grid[0], GridY=grid[1], BlockX=128),
           host.ArgBuffer(dsmap), host.ArgBuffer(ddmap))
    return src, ddst.cpu().numpy()


def test_tensor_tile_2d(dev, mod):
    src, got = _tile_double(dev, mod, 96, 64, (3, 2), False)
    assert np.array_equal(got, 2 * src)


def test_tensor_tile_out_of_bounds(dev, mod):
    # 40 x 40 in 32 x 32 tiles: the edge tiles hang off and are clamped.
    src, got = _tile_double(dev, mod, 40, 40, (2, 2), True)
    assert np.array_equal(got, 2 * src)


def test_encode_rejects_bad_descriptors_on_device(dev, cudair):
    import torch
    from cudair import host
    d = torch.zeros(64 * 64, dtype=torch.float32, device=dev)
    base = dict(DataType=host.TensorMapFloat32, GlobalDim=[64, 64], GlobalStrides=[64 * 4], BoxDim=[32, 32])
    host.EncodeTiled(d, host.TiledTensor(**base))
    for mut in (dict(GlobalStrides=[64 * 4 + 4]), dict(BoxDim=[512, 32]), dict(GlobalStrides=[256, 256]),
                dict(BoxDim=[32])):
        with pytest.raises(cudair.CudairError):
            host.EncodeTiled(d, host.TiledTensor(**{**base, **mut}))
    di = torch.zeros(64 * 64, dtype=torch.int32, device=dev)
    with pytest.raises(cudair.CudairError):
        host.EncodeTiled(di, host.TiledTensor(**{**base, "DataType": host.TensorMapFloat16}))


# ---- TestLaunchEx ---------------------------------------------------------------

@pytest.mark.parametrize("cluster", [1, 2, 4])
def test_runtime_cluster_dims(dev, mod, cluster):
    from cudair import host
    dout = up(dev, np.zeros(BLOCKS, np.int32))
    launch(mod, "ClusterRankRuntime", host.LaunchConfig(GridX=BLOCKS, BlockX=32), host.ArgBuffer(dout),
           attrs=host.LaunchAttrs(ClusterDim=(cluster, 1, 1)))
    b = np.arange(BLOCKS)
    assert np.array_equal(dout.cpu().numpy(), b % cluster + 100 * cluster)


def test_programmatic_dependent_launch(dev, mod):
    from cudair import host
    dout = up(dev, np.zeros(256, np.int32))
    launch(mod, "GridDep", cfg1d(256, 64), host.ArgBuffer(dout),
           attrs=host.LaunchAttrs(ProgrammaticStreamSerialization=True))
    assert np.array_equal(dout.cpu().numpy(), np.arange(256, dtype=np.int32))


def test_cooperative_attribute(dev, mod):
    from cudair import host
    dout = up(dev, np.zeros(64, np.int32))
    launch(mod, "GridDep", cfg1d(64, 64), host.ArgBuffer(dout), attrs=host.LaunchAttrs(Cooperative=True))
    assert np.array_equal(dout.cpu().numpy(), np.arange(64, dtype=np.int32))


# ---- vecadd run program ------------------------------------------------------------

def test_vecadd_saxpy_square_run(dev, mod, oracle):
    # examples/vecadd/run/main.go: VecAdd, then Saxpy (64 blocks, grid-stride)
    # on its output, then Square in place on a.
    from cudair import host
    n = 1 << 20
    a, b = oracle.vecadd_kat(n)
    da, db, dout = up(dev, a), up(dev, b), up(dev, np.zeros(n, np.float32))
    launch(mod, "VecAdd", cfg1d(n, 256), host.ArgBuffer(da), host.ArgBuffer(db), host.ArgBuffer(dout),
           host.ArgValue(ctypes.c_int32(n)))
    out = dout.cpu().numpy()
    assert np.array_equal(out, oracle.vecadd(a, b))
    launch(mod, "Saxpy", cfg1d(64 * 256, 256), host.ArgValue(ctypes.c_float(2.0)), host.ArgBuffer(da),
           host.ArgBuffer(dout), host.ArgValue(ctypes.c_int32(n)))
    assert np.array_equal(dout.cpu().numpy(), oracle.saxpy(2.0, a, out))
    launch(mod, "Square", cfg1d(n, 256), host.ArgBuffer(da), host.ArgValue(ctypes.c_int32(n)))
    assert np.array_equal(da.cpu().numpy(), oracle.square(a))


def test_saxpy_unfused_on_awkward_alpha(dev, mod, oracle):
    # With alpha = 1/3 a fused multiply-add would differ from the CPU check in
    # the last bit for many elements; the kernel rounds the product first.
    from cudair import host
    n = 100003
    x, y = oracle.uniform(n, 71), oracle.uniform(n, 72)
    dx, dy = up(dev, x), up(dev, y)
    alpha = np.float32(1.0) / np.float32(3.0)
    launch(mod, "Saxpy", cfg1d(n, 256), host.ArgValue(ctypes.c_float(alpha)), host.ArgBuffer(dx),
           host.ArgBuffer(dy), host.ArgValue(ctypes.c_int32(n)))
    assert np.array_equal(dy.cpu().numpy(), oracle.saxpy(float(alpha), x, y))


# ---- TestTensor: the mma.sync m16n8k16 family (tensor_test.go:23-145) -----------

def _elem(n, wi, wj, wij, m):
    i = np.arange(n).reshape(n, 1)
    j = np.arange(n).reshape(1, n)
    return (wi * i + wj * j + wij * i * j) % m


def _bf16_bits(x):
    # small integers: bfloat16 holds them exactly, the top half of the f32 bits
    return (np.asarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


@pytest.fixture(scope="module")
def tensor_kat():
    n = 64
    af = (_elem(n, 7, 13, 3, 5) - 2).astype(np.float32)
    bf = (_elem(n, 11, 5, 7, 5) - 2).astype(np.float32)
    bias = (_elem(n, 3, 7, 5, 11) - 5).astype(np.float32)
    want = (af.astype(np.int64) @ bf.astype(np.int64)).astype(np.float32)
    return n, af, bf, bias, want


def _mma_cfg(n):
    return cfg1d((n // 16) * (n // 8) * 32, 128)


def test_mma_f16_family(dev, mod, oracle, tensor_kat):
    from cudair import host
    n, af, bf, bias, want = tensor_kat
    ah = up(dev, oracle.f32_to_f16(af).view(np.int16))
    bh = up(dev, oracle.f32_to_f16(bf).view(np.int16))
    bth = up(dev, oracle.f32_to_f16(np.ascontiguousarray(bf.T)).view(np.int16))
    n32 = host.ArgValue(ctypes.c_int32(n))
    dc = up(dev, np.zeros((n, n), np.float32))
    launch(mod, "MmaF16", _mma_cfg(n), host.ArgBuffer(ah), host.ArgBuffer(bh), host.ArgBuffer(dc), n32)
    assert np.array_equal(dc.cpu().numpy(), want)
    dc2 = up(dev, np.zeros((n, n), np.float32))
    dbias = up(dev, bias)
    launch(mod, "MmaF16Bias", _mma_cfg(n), host.ArgBuffer(ah), host.ArgBuffer(bh),
           host.ArgBuffer(dbias), host.ArgBuffer(dc2), n32)
    assert np.array_equal(dc2.cpu().numpy(), want + bias)
    dc3 = up(dev, np.zeros((n, n), np.float32))
    launch(mod, "MmaF16Trans", _mma_cfg(n), host.ArgBuffer(ah), host.ArgBuffer(bth), host.ArgBuffer(dc3), n32)
    assert np.array_equal(dc3.cpu().numpy(), want)


def test_mma_f16_half_accumulator(dev, mod, oracle, tensor_kat):
    from cudair import host
    n, af, bf, _, want = tensor_kat
    dc = up(dev, np.zeros((n, n), np.int16))
    ah = up(dev, oracle.f32_to_f16(af).view(np.int16))
    bh = up(dev, oracle.f32_to_f16(bf).view(np.int16))
    launch(mod, "MmaF16Half", _mma_cfg(n), host.ArgBuffer(ah), host.ArgBuffer(bh), host.ArgBuffer(dc),
           host.ArgValue(ctypes.c_int32(n)))
    # |want| <= 256, so the fp16 accumulator is exact too
    got = oracle.f16_to_f32(dc.cpu().numpy().view(np.uint16))
    assert np.array_equal(got, want)


def test_mma_bf16(dev, mod, tensor_kat):
    from cudair import host
    n, af, bf, _, want = tensor_kat
    dc = up(dev, np.zeros((n, n), np.float32))
    ab = up(dev, _bf16_bits(af).view(np.int16))
    bb = up(dev, _bf16_bits(bf).view(np.int16))
    launch(mod, "MmaBF16", _mma_cfg(n), host.ArgBuffer(ab), host.ArgBuffer(bb), host.ArgBuffer(dc),
           host.ArgValue(ctypes.c_int32(n)))
    assert np.array_equal(dc.cpu().numpy(), want)


# ---- TestTensor: tf32, int8, ldmatrix and wmma (tensor_test.go:147-326) -------

def _wmma_cfg(n):
    return cfg1d((n // 16) * (n // 16) * 32, 128)


def _int8_kat(n):
    # tensor_test.go:161-169 and 293-305: signed operands are the float KAT's
    # values, unsigned ones other elem() patterns, bt the transpose of bu
    au = _elem(n, 7, 13, 3, 5).astype(np.uint8)
    bu = _elem(n, 11, 5, 7, 3).astype(np.uint8)
    bias_i = (_elem(n, 3, 7, 5, 11) - 5).astype(np.int32)
    return au, bu, np.ascontiguousarray(bu.T), bias_i


def test_mma_tf32(dev, mod, tensor_kat):
    from cudair import host
    n, af, bf, _, want = tensor_kat
    da, db, dbt = up(dev, af), up(dev, bf), up(dev, np.ascontiguousarray(bf.T))
    n32 = host.ArgValue(ctypes.c_int32(n))
    dc = up(dev, np.zeros((n, n), np.float32))
    launch(mod, "MmaTF32", _mma_cfg(n), host.ArgBuffer(da), host.ArgBuffer(db), host.ArgBuffer(dc), n32)
    assert np.array_equal(dc.cpu().numpy(), want)
    dc2 = up(dev, np.zeros((n, n), np.float32))
    launch(mod, "MmaTF32Trans", _mma_cfg(n), host.ArgBuffer(da), host.ArgBuffer(dbt), host.ArgBuffer(dc2), n32)
    assert np.array_equal(dc2.cpu().numpy(), want)


def test_mma_tf32_rounds_inputs(dev, mod):
    # cvt.rna keeps 10 mantissa bits, ties away from zero: 1 + 2^-11 (a tie)
    # becomes 1 + 2^-10 and 1 + 2^-12 becomes 1, so one 16 x 8 tile of A = that
    # value, B = identity shows the rounding the reference asks for.
    from cudair import host
    n = 16
    a = np.zeros((n, n), np.float32)
    a[:, 0] = 1 + 2.0 ** -11
    a[:, 1] = 1 + 2.0 ** -12
    a[:, 2] = -(1 + 2.0 ** -11)
    b = np.eye(n, dtype=np.float32)
    dc = up(dev, np.zeros((n, n), np.float32))
    launch(mod, "MmaTF32", _mma_cfg(n), host.ArgBuffer(up(dev, a)), host.ArgBuffer(up(dev, b)),
           host.ArgBuffer(dc), host.ArgValue(ctypes.c_int32(n)))
    got = dc.cpu().numpy()
    assert np.all(got[:, 0] == np.float32(1 + 2.0 ** -10))
    assert np.all(got[:, 1] == np.float32(1.0))
    assert np.all(got[:, 2] == np.float32(-(1 + 2.0 ** -10)))
    assert np.all(got[:, 3:] == 0)


def test_mma_int8(dev, mod, tensor_kat):
    from cudair import host
    n, af, bf, _, _ = tensor_kat
    a_s, b_s = af.astype(np.int8), bf.astype(np.int8)
    au, bu, but, _ = _int8_kat(n)
    want_s = a_s.astype(np.int64) @ b_s.astype(np.int64)
    want_u = au.astype(np.int64) @ bu.astype(np.int64)
    n32 = host.ArgValue(ctypes.c_int32(n))
    dc = up(dev, np.zeros((n, n), np.int32))
    launch(mod, "MmaS8", _mma_cfg(n), host.ArgBuffer(up(dev, a_s)), host.ArgBuffer(up(dev, b_s)),
           host.ArgBuffer(dc), n32)
    assert np.array_equal(dc.cpu().numpy(), want_s)
    dc2 = up(dev, np.zeros((n, n), np.int32))
    launch(mod, "MmaU8", _mma_cfg(n), host.ArgBuffer(up(dev, au)), host.ArgBuffer(up(dev, but)),
           host.ArgBuffer(dc2), n32)
    assert np.array_equal(dc2.cpu().numpy(), want_u)


def test_mma_int8_full_range(dev, mod):
    # every byte value, n = 128 (four k steps of 32): the s8 product, and the
    # u8 one whose sums stay far below the .satfinite limit
    from cudair import host
    n = 128
    rng = np.random.default_rng(5)
    a = rng.integers(0, 256, (n, n), dtype=np.uint8)
    b = rng.integers(0, 256, (n, n), dtype=np.uint8)
    n32 = host.ArgValue(ctypes.c_int32(n))
    dc = up(dev, np.zeros((n, n), np.int32))
    launch(mod, "MmaS8", _mma_cfg(n), host.ArgBuffer(up(dev, a.view(np.int8))),
           host.ArgBuffer(up(dev, b.view(np.int8))), host.ArgBuffer(dc), n32)
    assert np.array_equal(dc.cpu().numpy(), a.view(np.int8).astype(np.int64) @ b.view(np.int8).astype(np.int64))
    dc2 = up(dev, np.zeros((n, n), np.int32))
    launch(mod, "MmaU8", _mma_cfg(n), host.ArgBuffer(up(dev, a)), host.ArgBuffer(up(dev, np.ascontiguousarray(b.T))),
           host.ArgBuffer(dc2), n32)
    assert np.array_equal(dc2.cpu().numpy(), a.astype(np.int64) @ b.astype(np.int64))


def test_ldmatrix_registers(dev, mod, oracle):
    # tensor_test.go:192-228: four 8 x 8 matrices of distinct halves; lane
    # g*4+s holds (g, 2s), (g, 2s+1) of matrix i in register i (x4), the
    # transposed pair in .trans, matrices 0-1 in x2 and matrix 0 in x1
    from cudair import host
    vals = oracle.f32_to_f16(np.arange(1, 4 * 64 + 1, dtype=np.float32)).astype(np.uint32)
    dout = up(dev, np.zeros(4 * 32 * 4, np.int32))
    launch(mod, "LdMatrixRegs", cfg1d(32, 32), host.ArgBuffer(up(dev, vals.astype(np.uint16).view(np.int16))),
           host.ArgBuffer(dout))
    out = dout.cpu().numpy().view(np.uint32)
    mats = vals.reshape(4, 8, 8)
    lane = np.arange(32)
    g, s = lane // 4, lane % 4
    for i in range(4):
        m = mats[i]
        assert np.array_equal(out[lane * 4 + i], m[g, 2 * s] | (m[g, 2 * s + 1] << 16))
        assert np.array_equal(out[128 + lane * 4 + i], m[2 * s, g] | (m[2 * s + 1, g] << 16))
    for i in range(2):
        m = mats[i]
        assert np.array_equal(out[256 + lane * 2 + i], m[g, 2 * s] | (m[g, 2 * s + 1] << 16))
    assert np.array_equal(out[384 + lane], mats[0][g, 2 * s] | (mats[0][g, 2 * s + 1] << 16))


def test_mma_ldmatrix(dev, mod, oracle):
    # tensor_test.go:230-261
    from cudair import host
    i16 = np.arange(16).reshape(16, 1)
    j16, j8 = np.arange(16).reshape(1, 16), np.arange(8).reshape(1, 8)
    a16 = ((5 * i16 + 11 * j16 + 3 * i16 * j16) % 7 - 3).astype(np.float32)
    b16 = ((13 * i16 + 7 * j8 + 5 * i16 * j8) % 5 - 2).astype(np.float32)
    want = (a16.astype(np.int64) @ b16.astype(np.int64)).astype(np.float32)
    dc = up(dev, np.zeros((16, 8), np.float32))
    launch(mod, "MmaLdMatrix", cfg1d(32, 32), host.ArgBuffer(up(dev, oracle.f32_to_f16(a16).view(np.int16))),
           host.ArgBuffer(up(dev, oracle.f32_to_f16(b16).view(np.int16))), host.ArgBuffer(dc))
    assert np.array_equal(dc.cpu().numpy(), want)


def test_wmma_bf16(dev, mod, tensor_kat):
    from cudair import host
    n, af, bf, bias, want = tensor_kat
    da = up(dev, _bf16_bits(af).view(np.int16))
    db = up(dev, _bf16_bits(bf).view(np.int16))
    dbt = up(dev, _bf16_bits(np.ascontiguousarray(bf.T)).view(np.int16))
    n32 = host.ArgValue(ctypes.c_int32(n))
    dc = up(dev, np.zeros((n, n), np.float32))
    launch(mod, "WmmaBF16", _wmma_cfg(n), host.ArgBuffer(da), host.ArgBuffer(db), host.ArgBuffer(up(dev, bias)),
           host.ArgBuffer(dc), n32)
    assert np.array_equal(dc.cpu().numpy(), want + bias)
    dc2 = up(dev, np.zeros((n, n), np.float32))
    launch(mod, "WmmaBF16Trans", _wmma_cfg(n), host.ArgBuffer(da), host.ArgBuffer(dbt), host.ArgBuffer(dc2), n32)
    assert np.array_equal(dc2.cpu().numpy(), want)


def test_wmma_tf32(dev, mod, tensor_kat):
    from cudair import host
    n, af, bf, _, want = tensor_kat
    dc = up(dev, np.zeros((n, n), np.float32))
    launch(mod, "WmmaTF32", _wmma_cfg(n), host.ArgBuffer(up(dev, af)), host.ArgBuffer(up(dev, bf)),
           host.ArgBuffer(dc), host.ArgValue(ctypes.c_int32(n)))
    assert np.array_equal(dc.cpu().numpy(), want)


@pytest.mark.parametrize("n", [64, 48])
def test_wmma_int8(dev, mod, n):
    # n = 48: an odd number of 16-byte k steps and odd column tiles, the
    # cases whose tiles sit only 16 bytes apart in global memory
    from cudair import host
    af = (_elem(n, 7, 13, 3, 5) - 2).astype(np.int8)
    bf = (_elem(n, 11, 5, 7, 5) - 2).astype(np.int8)
    au, bu, but, bias_i = _int8_kat(n)
    want_s = af.astype(np.int64) @ bf.astype(np.int64)
    want_u = bias_i + au.astype(np.int64) @ bu.astype(np.int64)
    n32 = host.ArgValue(ctypes.c_int32(n))
    dc = up(dev, np.zeros((n, n), np.int32))
    launch(mod, "WmmaS8", _wmma_cfg(n), host.ArgBuffer(up(dev, af)), host.ArgBuffer(up(dev, bf)),
           host.ArgBuffer(dc), n32)
    assert np.array_equal(dc.cpu().numpy(), want_s)
    dc2 = up(dev, np.zeros((n, n), np.int32))
    launch(mod, "WmmaU8", _wmma_cfg(n), host.ArgBuffer(up(dev, au)), host.ArgBuffer(up(dev, but)),
           host.ArgBuffer(up(dev, bias_i)), host.ArgBuffer(dc2), n32)
    assert np.array_equal(dc2.cpu().numpy(), want_u)


def test_tensor_kernels_refuse_bad_shapes(dev, mod):
    # n not a multiple of 16, or of the int8 mma's k step of 32: the kernels
    # return without writing.  The buffers hold 64 x 64, so a kernel that
    # went ahead would still stay inside them.
    from cudair import host
    import torch
    a = up(dev, np.ones((64, 64), np.int8))
    dc = up(dev, np.full((64, 64), 7, np.int32))
    for name, cfg, n in (("MmaS8", _mma_cfg(64), 48), ("MmaU8", _mma_cfg(64), 40),
                         ("WmmaS8", _wmma_cfg(64), 40)):
        launch(mod, name, cfg, host.ArgBuffer(a), host.ArgBuffer(a), host.ArgBuffer(dc),
               host.ArgValue(ctypes.c_int32(n)))
    torch.cuda.synchronize()
    assert np.all(dc.cpu().numpy() == 7)


# ---- TestAdvanced/Wmma (advanced_test.go:25-80) ----------------------------------

def test_wmma_f16(dev, mod, oracle):
    from cudair import host
    n = 64
    i = np.arange(n).reshape(n, 1)
    j = np.arange(n).reshape(1, n)
    af = ((i + j) % 5 - 2).astype(np.float32)
    bf = ((i * j) % 3).astype(np.float32)
    bias = (i - j).astype(np.float32)
    prod = (af.astype(np.int64) @ bf.astype(np.int64)).astype(np.float32)
    da = up(dev, oracle.f32_to_f16(af).view(np.int16))
    db = up(dev, oracle.f32_to_f16(bf).view(np.int16))
    dbt = up(dev, oracle.f32_to_f16(np.ascontiguousarray(bf.T)).view(np.int16))
    n32 = host.ArgValue(ctypes.c_int32(n))
    dc = up(dev, np.zeros((n, n), np.float32))
    launch(mod, "Wmma", _wmma_cfg(n), host.ArgBuffer(da), host.ArgBuffer(db), host.ArgBuffer(up(dev, bias)),
           host.ArgBuffer(dc), n32)
    assert np.array_equal(dc.cpu().numpy(), prod + bias)
    # WmmaTrans: B given transposed, no bias, C stored column-major
    dc2 = up(dev, np.zeros((n, n), np.float32))
    launch(mod, "WmmaTrans", _wmma_cfg(n), host.ArgBuffer(da), host.ArgBuffer(dbt), host.ArgBuffer(dc2), n32)
    assert np.array_equal(dc2.cpu().numpy().T, prod)
