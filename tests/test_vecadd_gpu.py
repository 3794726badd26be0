"""VecAdd on the B200: bit-exact against the oracle and the golden fixture,
through the loaded module (the reference's launch, main_test.go:19-61) and
through the C-ABI launcher, with ragged lengths and misaligned pointers."""
import ctypes
import hashlib
import json
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


def _bits_equal(got, want):
    return np.array_equal(np.asarray(got).view(np.uint32), np.asarray(want).view(np.uint32))


def test_vecadd_reference_launch_kat(dev, module, oracle, golden_dir):
    # TestVecAdd: n = 2^20, a = 0.5 i, b = 1000 - i, LaunchConfig1D(n, 256).
    import torch
    from cudair import host
    g = json.load(open(os.path.join(golden_dir, "vecadd_kat.json")))
    n = g["n"]
    a, b = oracle.vecadd_kat(n)
    da, db = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    dout = torch.zeros(n, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    k = module.Function("VecAdd")
    k.LaunchEx(host.LaunchConfig1D(n, 256), host.LaunchAttrs(),
               host.ArgBuffer(da), host.ArgBuffer(db), host.ArgBuffer(dout),
               host.ArgValue(ctypes.c_int32(n)))
    out = dout.cpu().numpy()
    assert hashlib.sha256(out.tobytes()).hexdigest() == g["sha256"]
    assert _bits_equal(out, oracle.vecadd(a, b))


def test_vecadd_launcher_kat(dev, cudair, oracle, golden_dir):
    import torch
    from cudair import kernels
    g = json.load(open(os.path.join(golden_dir, "vecadd_kat.json")))
    a, b = oracle.vecadd_kat(g["n"])
    da, db = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    dout = torch.empty_like(da)
    kernels.vecadd(da, db, dout)
    out = dout.cpu().numpy()
    assert hashlib.sha256(out.tobytes()).hexdigest() == g["sha256"]


def test_vecadd_full_size_seeded(dev, cudair, oracle):
    # The benchmark configuration: n = 2^28, a, b ~ U(-1, 1) (seeds 4, 5).
    import torch
    from cudair import kernels
    n = 1 << 28
    a, b = oracle.uniform(n, 4), oracle.uniform(n, 5)
    want = oracle.vecadd(a, b, threads=oracle.num_threads())
    da, db = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    dout = torch.empty_like(da)
    kernels.vecadd(da, db, dout)
    out = dout.cpu().numpy()
    del da, db, dout
    torch.cuda.empty_cache()
    assert _bits_equal(out, want)


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 7, 255, 256, 257, 1023, 4097, 65537, 1000003])
@pytest.mark.parametrize("offsets", [(0, 0, 0), (1, 1, 1), (3, 3, 3), (1, 2, 3), (0, 1, 0)])
def test_vecadd_ragged_and_misaligned(dev, cudair, oracle, n, offsets):
    import torch
    from cudair import kernels
    rng = np.random.default_rng(n * 31 + sum(offsets))
    a = rng.standard_normal(n + 8).astype(np.float32)
    b = rng.standard_normal(n + 8).astype(np.float32)
    da, db = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    dout = torch.full((n + 8,), 7.0, dtype=torch.float32, device=dev)
    oa, ob, oo = offsets
    kernels.vecadd(da[oa:oa + n], db[ob:ob + n], dout[oo:oo + n])
    out = dout.cpu().numpy()
    want = oracle.vecadd(a[oa:oa + n], b[ob:ob + n])
    assert _bits_equal(out[oo:oo + n], want)
    # Nothing outside [oo, oo + n) was written.
    assert np.all(out[:oo] == 7.0) and np.all(out[oo + n:] == 7.0)


@pytest.mark.parametrize("n", [1, 33, 256 * 5 + 3])
def test_vecadd_reference_launch_ragged(dev, module, oracle, n):
    import torch
    from cudair import host
    a = np.arange(n, dtype=np.float32) * np.float32(0.25)
    b = np.float32(3) - np.arange(n, dtype=np.float32)
    da, db = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    dout = torch.zeros(n + 4, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    module.Function("VecAdd").LaunchEx(
        host.LaunchConfig1D(n, 256), host.LaunchAttrs(), host.ArgBuffer(da), host.ArgBuffer(db),
        host.ArgBuffer(dout), host.ArgValue(ctypes.c_int32(n)))
    out = dout.cpu().numpy()
    assert _bits_equal(out[:n], oracle.vecadd(a, b)) and np.all(out[n:] == 0)


def test_vecadd_special_values(dev, cudair, oracle):
    import torch
    from cudair import kernels
    rng = np.random.default_rng(3)
    bits = rng.integers(0, 2 ** 32, 1 << 16, dtype=np.uint64).astype(np.uint32)
    a = bits.view(np.float32).copy()
    b = np.roll(a, 1).copy()
    a[:8] = [np.inf, -np.inf, np.inf, 0.0, -0.0, 3.4e38, 1e-45, np.nan]
    b[:8] = [-np.inf, 1.0, np.inf, -0.0, -0.0, 3.4e38, -1e-45, 1.0]
    da, db = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    dout = torch.empty_like(da)
    kernels.vecadd(da, db, dout)
    out = dout.cpu().numpy()
    want = oracle.vecadd(a, b)
    same = (out.view(np.uint32) == want.view(np.uint32)) | (np.isnan(out) & np.isnan(want))
    assert same.all()


def test_vecadd_zero_length_is_noop(dev, cudair):
    assert cudair.lib().cudair_vecadd(None, None, None, 0, None) == 0
