"""cudair_fill: the seeded streams generated on the device are bit for bit the
oracle's (uniform and Box-Muller normal, fp32 and fp16, at offsets), so the
benchmark's operands are the ones the parity checks regenerate on the CPU."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev_fill(kind, n, seed, p0, p1, offset, half, dev):
    import torch
    from cudair import kernels
    t = torch.empty(n, dtype=torch.float16 if half else torch.float32, device=dev)
    fn = kernels.fill_uniform if kind == "uniform" else kernels.fill_normal
    fn(t, seed, p0, p1, offset=offset)
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _oracle(oracle, kind, n, seed, p0, p1, offset, half):
    x = (oracle.uniform if kind == "uniform" else oracle.normal)(n, seed, p0, p1, offset=offset)
    return oracle.f32_to_f16(x) if half else x


@pytest.mark.parametrize("kind,p0,p1", [("uniform", -1.0, 1.0), ("uniform", 0.25, 3.5),
                                        ("normal", 0.0, 1.0), ("normal", 0.0, 1.0 / np.sqrt(8192.0)),
                                        ("normal", 0.5, 0.02)])
@pytest.mark.parametrize("half", [False, True])
@pytest.mark.parametrize("n,offset", [(1, 0), (1000003, 0), (65537, 123456789)])
def test_fill_matches_oracle_bit_for_bit(dev, oracle, kind, p0, p1, half, n, offset):
    for seed in (4, 12):
        got = _dev_fill(kind, n, seed, p0, p1, offset, half, dev)
        want = _oracle(oracle, kind, n, seed, p0, p1, offset, half)
        got_bits = got.view(np.uint16 if half else np.uint32)
        want_bits = want.view(np.uint16) if half else want.view(np.uint32)
        bad = np.flatnonzero(got_bits != want_bits)
        assert bad.size == 0, (kind, seed, half, bad[:5], got[bad[:5]], want[bad[:5]])


def test_fill_full_benchmark_operand(dev, oracle):
    # B of the 8192^3 GEMM: fp16(N(0, 1/sqrt(8192))), seed 7, all 2^26 values.
    n = 8192 * 8192
    got = _dev_fill("normal", n, 7, 0.0, 1.0 / np.sqrt(8192.0), 0, True, dev)
    want = oracle.f32_to_f16(oracle.normal(n, 7, 0.0, 1.0 / np.sqrt(8192.0)))
    assert np.array_equal(got.view(np.uint16), want)


def test_fill_slices_compose(dev):
    # A rank's rows of a matrix generated at its offset equal those rows of
    # the whole matrix.
    import torch
    from cudair import kernels
    whole = torch.empty(64, 1000, device=dev)
    kernels.fill_normal(whole, 11)
    part = torch.empty(16, 1000, device=dev)
    kernels.fill_normal(part, 11, offset=32 * 1000)
    assert torch.equal(whole[32:48], part)


def test_fill_rejects_bad_arguments(dev, cudair):
    import torch
    from cudair import kernels
    from cudair._lib import CudairError
    with pytest.raises(CudairError, match="float32 or float16"):
        kernels.fill_uniform(torch.empty(4, dtype=torch.float64, device=dev), 1)
    L = cudair.lib()
    assert L.cudair_fill(None, 2, 0, 4, 1, 0, 0.0, 1.0, None) == 1
    assert L.cudair_fill(None, 0, 7, 4, 1, 0, 0.0, 1.0, None) == 1
    assert L.cudair_fill(None, 0, 0, -1, 1, 0, 0.0, 1.0, None) == 1
    assert L.cudair_fill(None, 0, 0, 0, 1, 0, 0.0, 1.0, None) == 0
