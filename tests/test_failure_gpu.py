"""Failure detection without a GPU fault: a bounded mbarrier wait that nobody
satisfies gives up after a short limit, records its site in the status word
and returns; the host reads the status and the context stays usable."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SITE_SELFTEST = 1 << 5


def test_bounded_wait_times_out_and_context_survives(dev, cudair, oracle):
    import torch
    from cudair import kernels
    assert kernels.wait_status(clear=True) == 0
    kernels.wait_timeout_selftest(2_000_000)  # 2 ms
    with pytest.raises(cudair.CudairError) as e:
        kernels.wait_status(clear=True)
    assert e.value.code == 4
    assert e.value.status & SITE_SELFTEST
    assert kernels.wait_status(clear=True) == 0
    # The context is still usable: a kernel runs and is exact.
    a, b = oracle.uniform(4099, 31), oracle.uniform(4099, 32)
    da, db = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    out = torch.empty_like(da)
    kernels.vecadd(da, db, out)
    assert np.array_equal(out.cpu().numpy(), oracle.vecadd(a, b))


def test_status_stays_clear_after_normal_gemm(dev, cudair):
    import torch
    from cudair import kernels
    a = torch.ones(256, 256, dtype=torch.float16, device=dev)
    c = torch.zeros(256, 256, dtype=torch.float32, device=dev)
    kernels.matmul16(a, a, c)
    assert kernels.wait_status(clear=True) == 0
    assert torch.all(c == 256).item()
