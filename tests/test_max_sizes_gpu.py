"""The streaming kernels at the largest length their int32 `n` allows
(VecAdd, Saxpy and Square at 2^31 - 1 elements, 8 GiB per vector; ReduceF32
at the largest multiple of 32): no 32-bit index overflows in the chunk
loops, the vector body or the scalar tail.  Operands are closed-form (small
integers and halves, exact in fp32), generated and checked on the GPU in
chunks, so nothing of the 8 GiB vectors crosses the host link."""
import pytest

pytestmark = pytest.mark.gpu

N_MAX = (1 << 31) - 1
CHUNK = 1 << 28


def _pattern(i, mod, scale, offset):
    return ((i % mod).float() * scale + offset)


def _chunks(n, chunk=CHUNK):
    for lo in range(0, n, chunk):
        yield lo, min(n, lo + chunk)


def _fill(t, mod, scale, offset, dev):
    import torch
    for lo, hi in _chunks(t.numel()):
        i = torch.arange(lo, hi, device=dev, dtype=torch.int64)
        t[lo:hi] = _pattern(i, mod, scale, offset)


def _check(t, fn, dev):
    import torch
    for lo, hi in _chunks(t.numel()):
        i = torch.arange(lo, hi, device=dev, dtype=torch.int64)
        want = fn(i)
        bad = (t[lo:hi] != want).nonzero()
        assert bad.numel() == 0, f"first mismatch at {lo + int(bad[0])}"


def test_vecadd_saxpy_square_at_int32_max(dev, cudair):
    import torch
    from cudair import kernels
    a = torch.empty(N_MAX, device=dev)
    b = torch.empty(N_MAX, device=dev)
    out = torch.empty(N_MAX, device=dev)
    _fill(a, 1000, 0.5, -250.0, dev)
    _fill(b, 777, 1.0, 3.0, dev)
    kernels.vecadd(a, b, out)
    _check(out, lambda i: _pattern(i, 1000, 0.5, -250.0) + _pattern(i, 777, 1.0, 3.0), dev)
    kernels.saxpy(2.0, a, b)  # b = 2 a + b
    _check(b, lambda i: 2.0 * _pattern(i, 1000, 0.5, -250.0) + _pattern(i, 777, 1.0, 3.0), dev)
    kernels.square(a)
    _check(a, lambda i: _pattern(i, 1000, 0.5, -250.0) ** 2, dev)
    del a, b, out
    torch.cuda.empty_cache()


def test_reduce_f32_at_int32_max(dev, cudair):
    import torch
    from cudair import kernels
    n = N_MAX // 32 * 32
    x = torch.empty(n, device=dev)
    _fill(x, 4099, 1.0, -2000.0, dev)
    out = torch.empty(n // 16, device=dev)
    kernels.reduce_f32(x, out)
    # Per warp w: min and max of x[32 w .. 32 w + 31], from the same closed form.
    w = torch.arange(n // 32, device=dev, dtype=torch.int64)
    got_min, got_max = out[0::2], out[1::2]
    for lo, hi in _chunks(n // 32, 1 << 22):  # 2^22 warps: a 1 GiB index block at a time
        ww = w[lo:hi].view(-1, 1)
        vals = _pattern(ww * 32 + torch.arange(32, device=dev).view(1, 32), 4099, 1.0, -2000.0)
        assert torch.equal(got_min[lo:hi], vals.min(dim=1).values)
        assert torch.equal(got_max[lo:hi], vals.max(dim=1).values)
    del x, out
    torch.cuda.empty_cache()
