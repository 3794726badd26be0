"""Shared test set-up.

  -m "not gpu"  the oracle against the golden fixtures, the C-ABI library's
                exports and host-side validation, the multi-GPU host logic on
                gloo ranks: all on CPU.
  -m gpu        parity of the sm_100a kernels (through the C ABI) against the
                oracle and the golden fixtures, on a B200.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(REPO, "cuda-ir.go_b200"), os.path.join(REPO, "oracle"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def cudair():
    import cudair as c
    c.lib()
    return c


@pytest.fixture(scope="session")
def dev():
    """The B200 the GPU tests run on; fails (not skips) without one, since a
    -m gpu run is only meaningful on a GPU."""
    import torch
    assert torch.cuda.is_available(), "the gpu tests need a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert major == 10, f"the gpu tests need an sm_100 device, found {major}.{minor}"
    torch.cuda.set_device(0)
    torch.cuda.init()
    return torch.device("cuda:0")
