"""cudair: the B200 (sm_100a) build of cuda-ir.go's MatMul16 / VecAdd path.

  cudair.host     the reference's host/ package over the C ABI (tensor maps,
                  module loading, cuLaunchKernelEx launches)
  cudair.kernels  launchers of the tuned sm_100a kernels (torch tensors in)

The compute lives in libcudair_b200.so and cudair_kernels.cubin, built
in-tree by cuda-ir.go_b200/build.py; nothing here computes on the CPU.
"""
from ._lib import CudairError, lib, last_error, LIB_PATH, CUBIN_PATH  # noqa: F401
from . import host, kernels  # noqa: F401
