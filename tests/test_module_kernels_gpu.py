"""The rest of the module's reference-named kernels on the B200, loaded and
launched the way the reference's tests do, with the same known answers:

  TestHopper (advanced_test.go:355-548): Cluster, MBarrier, TMA, Elect,
      GridDep, StMatrix
  TestTensorMap (hostapi_test.go:472-623): TensorTile2D, OutOfBounds
  TestLaunchEx (hostapi_test.go:360-466): RuntimeClusterDims,
      ProgrammaticDependentLaunch, Cooperative
  examples/vecadd/run/main.go:62-76: Saxpy, Square
  TestTensor (tensor_test.go:23-145): MmaF16, MmaF16Bias, MmaF16Trans,
      MmaF16Half, MmaBF16
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
