"""The C ABI from a C program (tests/c_client/matmul16_client.c): dlopen of
libcudair_b200.so, the MatMul16 test flow through the host entry and the
tuned kernel, VecAdd and the error path, with no Python between the caller
and the library.  Compiled here with gcc against the CUDA runtime."""
import os
import shutil
import subprocess

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def test_c_client(tmp_path, dev, cudair):
    from cudair import _lib
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    exe = tmp_path / "matmul16_client"
    subprocess.run([cc, "-O2", "-std=c11", os.path.join(HERE, "c_client", "matmul16_client.c"),
                    "-I", os.path.join(cuda, "include"), "-L", os.path.join(cuda, "lib64"),
                    "-Wl,-rpath," + os.path.join(cuda, "lib64"), "-o", str(exe), "-ldl", "-lcudart"],
                   check=True)
    r = subprocess.run([str(exe), _lib.LIB_PATH], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith("ok"), r.stdout
