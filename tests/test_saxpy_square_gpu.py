"""Saxpy and Square (vecadd.go:13-28) through their tuned launchers:
bit-exact with the oracle's float32 loops (product and sum rounded
separately) on ragged lengths, every misalignment the launchers take, special
values, and the full 2^28-element size; nothing outside the vectors is
written.  The module entries under the reference's launches are covered with
the run program's checks in test_module_kernels_gpu.py."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits_equal(x, y):
    return np.array_equal(np.asarray(x, np.float32).view(np.uint32), np.asarray(y, np.float32).view(np.uint32))


@pytest.mark.parametrize("n", [1, 3, 4, 5, 255, 257, 4097, 65537, 1000003])
@pytest.mark.parametrize("offsets", [(0, 0), (1, 1), (3, 3), (1, 2), (0, 3)])
def test_saxpy_ragged_and_misaligned(dev, cudair, oracle, n, offsets):
    import torch
    from cudair import kernels
    rng = np.random.default_rng(n * 7 + sum(offsets))
    x = rng.standard_normal(n + 8).astype(np.float32)
    y = rng.standard_normal(n + 8).astype(np.float32)
    alpha = np.float32(1.0) / np.float32(3.0)
    ox, oy = offsets
    dx, dy = torch.from_numpy(x).to(dev), torch.from_numpy(y).to(dev)
    kernels.saxpy(alpha, dx[ox:ox + n], dy[oy:oy + n])
    out = dy.cpu().numpy()
    assert _bits_equal(out[oy:oy + n], oracle.saxpy(float(alpha), x[ox:ox + n], y[oy:oy + n]))
    assert _bits_equal(out[:oy], y[:oy]) and _bits_equal(out[oy + n:], y[oy + n:])


@pytest.mark.parametrize("n", [1, 2, 5, 257, 65537, 1000003])
@pytest.mark.parametrize("offset", [0, 1, 2, 3])
def test_square_ragged_and_misaligned(dev, cudair, oracle, n, offset):
    import torch
    from cudair import kernels
    rng = np.random.default_rng(n + offset)
    x = (rng.standard_normal(n + 8) * 100).astype(np.float32)
    dx = torch.from_numpy(x).to(dev)
    kernels.square(dx[offset:offset + n])
    out = dx.cpu().numpy()
    assert _bits_equal(out[offset:offset + n], oracle.square(x[offset:offset + n]))
    assert _bits_equal(out[:offset], x[:offset]) and _bits_equal(out[offset + n:], x[offset + n:])


def test_special_values(dev, cudair, oracle):
    import torch
    from cudair import kernels
    v = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 3.4e38, -3.4e38, 1e20, 7.0, -2.5],
                 dtype=np.float32)
    x = np.tile(v, 40)
    y = np.roll(x, 3).copy()
    dx, dy = torch.from_numpy(x).to(dev), torch.from_numpy(y).to(dev)
    kernels.saxpy(2.0, dx, dy)
    kernels.square(dx)
    # Bit-exact, except that a NaN matches any NaN (payloads differ by platform).
    for got, want in ((dy.cpu().numpy(), oracle.saxpy(2.0, x, y)), (dx.cpu().numpy(), oracle.square(x))):
        same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
        assert same.all()


def test_full_size(dev, cudair, oracle):
    import torch
    from cudair import kernels
    n = 1 << 28
    x, y = oracle.uniform(n, 14), oracle.uniform(n, 15)
    dx, dy = torch.from_numpy(x).to(dev), torch.from_numpy(y).to(dev)
    kernels.saxpy(0.75, dx, dy)
    kernels.square(dx)
    got_y, got_x = dy.cpu().numpy(), dx.cpu().numpy()
    del dx, dy
    torch.cuda.empty_cache()
    assert _bits_equal(got_y, oracle.saxpy(0.75, x, y))
    assert _bits_equal(got_x, oracle.square(x))


def test_zero_length_and_validation(dev, cudair):
    L = cudair.lib()
    assert L.cudair_saxpy(1.0, None, None, 0, None) == 0
    assert L.cudair_square(None, 0, None) == 0
    assert L.cudair_saxpy(1.0, None, None, -1, None) == 1
    assert L.cudair_square(None, 4, None) == 1 and "nil pointer" in cudair.last_error()
