"""ReduceF32 (examples/blackwell/blackwell.go:8-17) on the B200: per-warp
min/max with redux.sync.{min,max}.f32, checked as TestBlackwell does
(advanced_test.go:564-580) and on the edge cases of Go's math.Min/Max."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run_module(dev, x):
    import torch
    from cudair import host
    n = x.size
    m = host.LoadModule(host.KernelsImage())
    try:
        din = torch.from_numpy(x).to(dev)
        dout = torch.zeros(n // 16, dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        m.Function("ReduceF32").LaunchEx(host.LaunchConfig1D(n, 256), host.LaunchAttrs(),
                                         host.ArgBuffer(din), host.ArgBuffer(dout))
        return dout.cpu().numpy()
    finally:
        m.Close()


def _same(got, want):
    return np.array_equal(got.view(np.uint32), want.view(np.uint32)) or all(
        (g == w and np.signbit(g) == np.signbit(w)) or (np.isnan(g) and np.isnan(w))
        for g, w in zip(got, want))


def test_reduce_kat_reference_launch(dev, cudair, oracle, golden_dir):
    t = np.load(os.path.join(golden_dir, "reduce_kat.npz"))
    out = _run_module(dev, t["x"])
    assert np.array_equal(out[: 2 * (1024 // 32)], t["want"])
    assert np.all(out[2 * (1024 // 32):] == 0)


def test_reduce_launcher_matches_oracle(dev, cudair, oracle):
    import torch
    from cudair import kernels
    for n in (32, 96, 1024, 1 << 20):
        x = oracle.uniform(n, 21 + n)
        dout = torch.zeros(2 * (n // 32), dtype=torch.float32, device=dev)
        kernels.reduce_f32(torch.from_numpy(x).to(dev), dout)
        assert np.array_equal(dout.cpu().numpy(), oracle.reduce_f32(x))


def test_reduce_go_min_max_edge_cases(dev, cudair, oracle):
    # NaN propagates, -0 orders below +0, infinities win (math.Min/Max).
    import torch
    from cudair import kernels
    x = np.zeros(32 * 6, dtype=np.float32)
    x[0:32] = np.linspace(-1, 1, 32)
    x[5] = np.nan
    x[32:64] = 0.0
    x[40] = -0.0
    x[64:96] = np.arange(32)
    x[70] = np.inf
    x[96:128] = np.arange(32)
    x[100] = -np.inf
    x[128:160] = -0.0
    x[150] = 0.0
    x[160:192] = np.float32(1e-45) * np.arange(32)
    dout = torch.zeros(12, dtype=torch.float32, device=dev)
    kernels.reduce_f32(torch.from_numpy(x).to(dev), dout)
    got = dout.cpu().numpy()
    assert _same(got, oracle.reduce_f32(x)), (got, oracle.reduce_f32(x))
