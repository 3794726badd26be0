"""include/cudair_b200.h is the drop-in boundary for C callers: it must
compile on its own as C99, C11 and C++17 with warnings as errors, and
declare every entry point the library exports (checked against the .so in
test_abi.py)."""
import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_SRC = """#include "cudair_b200.h"
#include <stddef.h>
/* Take the address of a few entry points so their declarations are used. */
int (*const p_matmul16)(const void *, const void *, float *, int32_t, void *) = cudair_matmul16;
int (*const p_vecadd)(const float *, const float *, float *, int32_t, void *) = cudair_vecadd;
int (*const p_host)(const void *, const void *, float *, int64_t, int64_t, int64_t, int64_t, int64_t,
                    int64_t, void *, void *, float *, int64_t, void *) = cudair_gemm_f16f32_host;
int probe(void) { return CUDAIR_OK + CUDAIR_ERR_INVALID + (int)sizeof(cudair_module); }
"""


@pytest.mark.parametrize("lang,std", [("c", "c99"), ("c", "c11"), ("c++", "c++17")])
def test_header_compiles_standalone(tmp_path, lang, std):
    cc = shutil.which("g++" if lang == "c++" else "gcc")
    if cc is None:
        pytest.skip("no compiler")
    src = tmp_path / ("probe.cpp" if lang == "c++" else "probe.c")
    src.write_text(_SRC)
    r = subprocess.run([cc, "-std=" + std, "-Wall", "-Wextra", "-Werror", "-pedantic", "-c", str(src),
                        "-I", os.path.join(REPO, "include"), "-o", str(tmp_path / "probe.o")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
