"""cudair_launch_ex with the launch attributes of host.LaunchAttrs
(host/launchex.go:105-173): a runtime cluster shape, the cooperative launch
and programmatic stream serialisation, on the module's own kernels, plus an
asynchronous launch on a torch stream."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def vecadd_fn(dev, cudair):
    from cudair import host
    m = host.LoadModule(host.KernelsImage())
    yield m.Function("VecAdd")
    m.Close()


def _buffers(dev, oracle, n, seed):
    import torch
    a, b = oracle.uniform(n, seed), oracle.uniform(n, seed + 1)
    return a, b, torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev), \
        torch.zeros(n, dtype=torch.float32, device=dev)


@pytest.mark.parametrize("attrs", [
    dict(ClusterDim=(1, 1, 1)), dict(ClusterDim=(2, 1, 1)), dict(ClusterDim=(4, 1, 1)),
    dict(Cooperative=True), dict(ProgrammaticStreamSerialization=True),
])
def test_launch_attributes(dev, cudair, oracle, vecadd_fn, attrs):
    import torch
    from cudair import host
    n = 8 * 256 * 4
    a, b, da, db, dout = _buffers(dev, oracle, n, 41)
    torch.cuda.synchronize()
    vecadd_fn.LaunchEx(host.LaunchConfig(GridX=8, BlockX=256), host.LaunchAttrs(**attrs),
                       host.ArgBuffer(da), host.ArgBuffer(db), host.ArgBuffer(dout),
                       host.ArgValue(ctypes.c_int32(n)))
    assert np.array_equal(dout.cpu().numpy(), oracle.vecadd(a, b))


def test_launch_on_stream_is_asynchronous(dev, cudair, oracle, vecadd_fn):
    import torch
    from cudair import host
    n = 1 << 20
    a, b, da, db, dout = _buffers(dev, oracle, n, 51)
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    vecadd_fn.LaunchExOn(s, host.LaunchConfig1D(n, 256), host.LaunchAttrs(),
                         host.ArgBuffer(da), host.ArgBuffer(db), host.ArgBuffer(dout),
                         host.ArgValue(ctypes.c_int32(n)))
    s.synchronize()
    assert np.array_equal(dout.cpu().numpy(), oracle.vecadd(a, b))


def test_unknown_function_is_an_error(dev, cudair):
    from cudair import host
    m = host.LoadModule(host.KernelsImage())
    try:
        with pytest.raises(cudair.CudairError) as e:
            m.Function("NoSuchKernel")
        assert "NoSuchKernel" in str(e.value) and "CUDA_ERROR_NOT_FOUND" in str(e.value)
    finally:
        m.Close()


def test_encode_tiled_valid_descriptor_on_device(dev, cudair):
    # TestTensorMap/Encode's valid case: accepted by the driver.
    import torch
    from cudair import host
    d = torch.zeros(64 * 64, dtype=torch.float32, device=dev)
    m = host.EncodeTiled(d, host.TiledTensor(DataType=host.TensorMapFloat32, GlobalDim=[64, 64],
                                             GlobalStrides=[64 * 4], BoxDim=[32, 32]))
    assert len(m.Bytes()) == 128 and any(m.Bytes())
