"""The host-buffer entries of the VecAdd and MatMul16 flows, through the C ABI:
cudair_vecadd_host (main_test.go:31-48: upload a and b, launch, copy out back)
bit-exact against the oracle's add, and cudair_matmul16_host
(advanced_test.go:466-483) exact on the reference's integer case and within
the GEMM tolerance on seeded data, at the sizes of both of its paths."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,chunk,pinned", [(1 << 20, 0, True), (1000003, 0, True), (1000003, 4096, False),
                                            (5, 0, True), ((1 << 24) + 7, 0, True), ((1 << 22) + 1, 65536, True)])
def test_vecadd_host_bit_exact(dev, oracle, n, chunk, pinned):
    import torch
    from cudair import kernels
    a, b = oracle.uniform(n, 4), oracle.uniform(n, 5)
    a_h, b_h = torch.from_numpy(a), torch.from_numpy(b)
    out_h = torch.full((n,), float("nan"))
    if pinned:
        a_h, b_h, out_h = a_h.pin_memory(), b_h.pin_memory(), out_h.pin_memory()
    a_d, b_d, out_d = (torch.empty(n, device=dev) for _ in range(3))
    for _ in range(2):  # the second call reuses the library's streams and events
        kernels.vecadd_host(a_h, b_h, out_h, a_d, b_d, out_d, chunk=chunk)
        torch.cuda.current_stream().synchronize()
        assert np.array_equal(out_h.numpy(), oracle.vecadd(a, b))


def test_vecadd_host_reference_kat(dev, oracle, golden_dir):
    import hashlib
    import json
    import os

    import torch
    from cudair import kernels
    kat = json.load(open(os.path.join(golden_dir, "vecadd_kat.json")))
    a, b = oracle.vecadd_kat(kat["n"])
    out_h = torch.empty(kat["n"]).pin_memory()
    a_d, b_d, out_d = (torch.empty(kat["n"], device=dev) for _ in range(3))
    kernels.vecadd_host(torch.from_numpy(a).pin_memory(), torch.from_numpy(b).pin_memory(), out_h,
                        a_d, b_d, out_d)
    torch.cuda.current_stream().synchronize()
    assert hashlib.sha256(out_h.numpy().tobytes()).hexdigest() == kat["sha256"]


@pytest.mark.parametrize("n", [64, 256, 1024])
def test_matmul16_host(dev, oracle, n):
    import torch
    from cudair import kernels
    af, bf, c = oracle.matmul16_kat(n)
    a_d, b_d = (torch.empty(n, n, dtype=torch.float16, device=dev) for _ in range(2))
    c_d = torch.empty(n, n, device=dev)
    c_h = torch.from_numpy(c.copy()).pin_memory()
    kernels.matmul16_host(torch.from_numpy(af).half().pin_memory(), torch.from_numpy(bf).half().pin_memory(),
                          c_h, a_d, b_d, c_d)
    torch.cuda.current_stream().synchronize()
    assert np.array_equal(c_h.numpy(), oracle.gemm_ijk(af, bf, c) if n <= 256 else oracle.gemm_ikj(af, bf, c))

    a16 = oracle.f32_to_f16(oracle.uniform(n * n, 1)).reshape(n, n)
    b16 = oracle.f32_to_f16(oracle.uniform(n * n, 2)).reshape(n, n)
    c = oracle.uniform(n * n, 3).reshape(n, n)
    c_h = torch.from_numpy(c.copy()).pin_memory()
    kernels.matmul16_host(torch.from_numpy(a16.view(np.int16)).view(torch.float16).pin_memory(),
                          torch.from_numpy(b16.view(np.int16)).view(torch.float16).pin_memory(),
                          c_h, a_d, b_d, c_d)
    torch.cuda.current_stream().synchronize()
    want = oracle.gemm_ikj(oracle.f16_to_f32(a16), oracle.f16_to_f32(b16), c)
    rel, mx, bad = oracle.error_norms(c_h.numpy(), want)
    tol_rel, tol_max = oracle.gemm_tolerance(n, 1.0, 1.0)
    assert bad == 0 and rel <= tol_rel and mx <= tol_max, (rel, mx)
    from cudair import kernels as k
    assert k.wait_status(clear=True) == 0


def test_host_entries_allocate_no_device_memory(dev):
    # After a first call on the device (which creates the library's streams
    # and events), further calls of the three host-buffer entries leave the
    # device's free memory and torch's reserved bytes unchanged.
    import torch
    from cudair import kernels
    n = 1 << 20
    a_h, b_h, o_h = (torch.ones(n).pin_memory() for _ in range(3))
    a_d, b_d, o_d = (torch.empty(n, device=dev) for _ in range(3))
    m = 1024
    ga_h = torch.ones(m, m, dtype=torch.float16).pin_memory()
    gb_h = torch.ones(m, m, dtype=torch.float16).pin_memory()
    gc_h = torch.zeros(m, m).pin_memory()
    ga_d, gb_d = (torch.empty(m, m, dtype=torch.float16, device=dev) for _ in range(2))
    gc_d = torch.empty(m, m, device=dev)
    s = 256
    sa_h = torch.ones(s, s, dtype=torch.float16).pin_memory()
    sb_h = torch.ones(s, s, dtype=torch.float16).pin_memory()
    sc_h = torch.zeros(s, s).pin_memory()
    sa_d, sb_d = (torch.empty(s, s, dtype=torch.float16, device=dev) for _ in range(2))
    sc_d = torch.empty(s, s, device=dev)

    def calls():
        kernels.vecadd_host(a_h, b_h, o_h, a_d, b_d, o_d)
        kernels.gemm_host(ga_h, gb_h, gc_h, ga_d, gb_d, gc_d)
        kernels.matmul16_host(sa_h, sb_h, sc_h, sa_d, sb_d, sc_d)
        torch.cuda.synchronize()

    calls()
    free0, _ = torch.cuda.mem_get_info()
    held0 = torch.cuda.memory_reserved()
    calls()
    calls()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_reserved() == held0
    assert torch.equal(o_h, torch.full((n,), 2.0))
