"""cudair_gemm: the examples/tensor GEMM family (tensor.go:15-98) on the
tcgen05 kernels.  The reference's TestTensor known answers (n = 64, the
asymmetric `elem` operands of tensor_test.go:49-66, compared with ==) for
MmaF16, MmaF16Bias, MmaF16Trans, MmaF16Half and MmaBF16, on each tuned
kernel; the same forms on ragged shapes (exact, integer operands) and on
seeded real data (against an fp32 torch product within the GEMM
tolerance)."""
import numpy as np
import pytest

from test_matmul16_gpu import kat

pytestmark = pytest.mark.gpu


def _elem(n, m_, wi, wj, wij, mod):
    i = np.arange(n).reshape(n, 1)
    j = np.arange(m_).reshape(1, m_)
    return (wi * i + wj * j + wij * i * j) % mod


@pytest.fixture(params=[1, 2, 4], ids=["single", "pair", "pairwide"])
def square_variant(request, dev, cudair):
    from cudair import kernels
    kernels.set_gemm_variant(request.param)
    yield request.param
    kernels.set_gemm_variant(0)


@pytest.fixture(scope="module")
def tensor_kat():
    n = 64
    af = (_elem(n, n, 7, 13, 3, 5) - 2).astype(np.float32)
    bf = (_elem(n, n, 11, 5, 7, 5) - 2).astype(np.float32)
    bias = (_elem(n, n, 3, 7, 5, 11) - 5).astype(np.float32)
    want = (af.astype(np.int64) @ bf.astype(np.int64)).astype(np.float32)
    return n, af, bf, bias, want


def _t(x, dev, dtype):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev).to(dtype)


def test_tensor_family_kats(dev, cudair, square_variant, tensor_kat):
    import torch
    from cudair import kernels
    n, af, bf, bias, want = tensor_kat
    a, b = _t(af, dev, torch.float16), _t(bf, dev, torch.float16)
    # MmaF16: C = A.B into a C full of junk.
    c = torch.full((n, n), 1e9, device=dev)
    kernels.gemm_ex(a, b, c, overwrite=True)
    assert np.array_equal(c.cpu().numpy(), want)
    # MmaF16Bias: C = A.B + bias.
    c = torch.full((n, n), -3.0, device=dev)
    kernels.gemm_ex(a, b, c, bias=_t(bias, dev, torch.float32), overwrite=True)
    assert np.array_equal(c.cpu().numpy(), want + bias)
    # MmaF16Trans: B from its transpose.
    c = torch.zeros(n, n, device=dev)
    kernels.gemm_ex(a, _t(bf.T, dev, torch.float16), c, b_trans=True, overwrite=True)
    assert np.array_equal(c.cpu().numpy(), want)
    # MmaF16Half: a half C (|want| <= 256: exact in half).
    ch = torch.full((n, n), 7.0, dtype=torch.float16, device=dev)
    kernels.gemm_ex(a, b, ch, overwrite=True)
    assert np.array_equal(ch.float().cpu().numpy(), want)
    # MmaBF16: bfloat16 operands.
    c = torch.zeros(n, n, device=dev)
    kernels.gemm_ex(_t(af, dev, torch.bfloat16), _t(bf, dev, torch.bfloat16), c, overwrite=True)
    assert np.array_equal(c.cpu().numpy(), want)


@pytest.mark.parametrize("M,N,K", [(300, 1000, 200), (129, 264, 72), (1000, 520, 1032), (7, 136, 64),
                                   (512, 768, 4096)])
@pytest.mark.parametrize("form", ["trans", "bf16-trans", "f16-out", "bf16-accumulate", "bias-trans"])
def test_forms_ragged_exact(dev, cudair, square_variant, M, N, K, form):
    import torch
    from cudair import kernels
    af, bf, c0, want_acc = kat(M, N, K)
    prod = want_acc - c0
    dt = torch.bfloat16 if form.startswith("bf16") else torch.float16
    a = _t(af, dev, dt)
    b = _t(bf, dev, dt)
    bt = _t(bf.T, dev, dt)
    if form in ("trans", "bf16-trans"):
        c = torch.full((M, N), 5e8, device=dev)
        kernels.gemm_ex(a, bt, c, b_trans=True, overwrite=True)
        assert np.array_equal(c.cpu().numpy(), prod)
    elif form == "f16-out":
        # |prod| <= 6 K stays exact in half only for small K
        if np.abs(prod).max() > 2048:
            pytest.skip("product not exact in half")
        ch = torch.zeros(M, N, dtype=torch.float16, device=dev)
        kernels.gemm_ex(a, bt, ch, b_trans=True, overwrite=True)
        assert np.array_equal(ch.float().cpu().numpy(), prod)
    elif form == "bf16-accumulate":
        c = _t(c0, dev, torch.float32)
        kernels.gemm_ex(a, b, c)
        assert np.array_equal(c.cpu().numpy(), want_acc)
    else:  # bias-trans
        c = torch.zeros(M, N, device=dev)
        kernels.gemm_ex(a, bt, c, bias=_t(c0, dev, torch.float32), b_trans=True, overwrite=True)
        assert np.array_equal(c.cpu().numpy(), want_acc)


@pytest.mark.parametrize("form", ["bf16", "trans", "f16-out"])
def test_forms_seeded_tolerance(dev, cudair, oracle, form):
    # fp32 results: the GEMM tolerance (relative Frobenius error <= 1e-3,
    # max |error| <= 5e-3 sqrt(K) max|a| max|b|) against torch's fp32
    # product of the same operands.  fp16 results: that tolerance plus one
    # rounding to half (relative 2^-11 of each element).
    import torch
    from cudair import kernels
    M, N, K = 2048, 3072, 2048
    g = torch.Generator(device=dev)
    g.manual_seed(91)
    dt = torch.bfloat16 if form == "bf16" else torch.float16
    a = (torch.randn(M, K, generator=g, device=dev) / K ** 0.5).to(dt)
    b = (torch.randn(K, N, generator=g, device=dev) / K ** 0.5).to(dt)
    ref = a.float() @ b.float()
    tol_rel, tol_max = oracle.gemm_tolerance(K, a.float().abs().max().item(), b.float().abs().max().item())
    if form == "f16-out":
        c = torch.empty(M, N, dtype=torch.float16, device=dev)
        kernels.gemm_ex(a, b, c, overwrite=True)
        err = (c.float() - ref).abs()
        assert bool((err <= ref.abs() * 2.0 ** -11 + tol_max).all())
        return
    c = torch.empty(M, N, device=dev)
    if form == "trans":
        kernels.gemm_ex(a, b.t().contiguous(), c, b_trans=True, overwrite=True)
    else:
        kernels.gemm_ex(a, b, c, overwrite=True)
    rel = ((c - ref).norm() / ref.norm()).item()
    mx = (c - ref).abs().max().item()
    assert rel <= tol_rel and mx <= tol_max, (rel, mx)


def test_fewrows_variant_refuses_other_forms(dev, cudair):
    import torch
    from cudair import kernels
    from cudair._lib import CudairError
    a = torch.zeros(16, 64, dtype=torch.float16, device=dev)
    b = torch.zeros(64, 128, dtype=torch.float16, device=dev)
    c = torch.zeros(16, 128, device=dev)
    kernels.set_gemm_variant(3)
    try:
        with pytest.raises(CudairError, match="few-row kernel"):
            kernels.gemm_ex(a, b, c, overwrite=True)
    finally:
        kernels.set_gemm_variant(0)
    kernels.gemm_ex(a, b, c, overwrite=True)  # the automatic choice takes it
    torch.cuda.synchronize()
    assert float(c.abs().max()) == 0.0


def test_overwrite_with_k_zero_clears_c(dev, cudair):
    import torch
    from cudair import kernels
    a = torch.zeros(40, 0, dtype=torch.float16, device=dev)
    b = torch.zeros(0, 64, dtype=torch.float16, device=dev)
    c = torch.full((40, 64), 3.0, device=dev)
    kernels.gemm_ex(a, b, c, overwrite=True)
    bias = torch.full((40, 64), -1.5, device=dev)
    c2 = torch.zeros(40, 64, device=dev)
    kernels.gemm_ex(a, b, c2, bias=bias, overwrite=True)
    torch.cuda.synchronize()
    assert float(c.abs().max()) == 0.0 and bool((c2 == -1.5).all())
