"""Pins the CPU oracle (oracle/oracle.c) against the golden fixtures, which
tests/golden/make_golden.py computes with numpy independently of the oracle,
from the known-answer inputs of the reference's own tests."""
import hashlib
import json
import os

import numpy as np
import pytest


def test_f16_rounding_matches_ieee_table(oracle, golden_dir):
    # float32ToHalf (advanced_test.go:597-623) against numpy's IEEE RNE.
    t = np.load(os.path.join(golden_dir, "f16_table.npz"))
    got = oracle.f32_to_f16(t["inputs"])
    bad = np.nonzero(got != t["halves"])[0]
    assert bad.size == 0, f"{bad.size} mismatches, first input {t['inputs'][bad[0]]!r}"


def test_f16_rounding_nan_maps_to_inf(oracle):
    # The reference's converter has no NaN branch: exponent 255 >= 31 -> inf.
    nan = np.array([np.nan, -np.nan], dtype=np.float32)
    nan[1] = -abs(nan[1])
    got = oracle.f32_to_f16(nan)
    assert got[0] == 0x7C00 and got[1] == 0xFC00


def test_f16_rounding_exhaustive_normals(oracle):
    # Every float32 exponent and the 2^13 mantissa patterns around each
    # rounding boundary, against numpy.
    e = np.arange(0, 255, dtype=np.uint32)
    m = np.concatenate([np.arange(0, 0x2000, dtype=np.uint32) << 10,
                        np.arange(0x0FF0, 0x1010, dtype=np.uint32)])
    bits = ((e[:, None] << 23) | m[None, :]).ravel()
    bits = np.concatenate([bits, bits | 0x80000000]).astype(np.uint32)
    x = bits.view(np.float32)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.f32_to_f16(x), want)


def test_f16_widening_is_exact(oracle):
    h = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    got = oracle.f16_to_f32(h)
    want = h.view(np.float16).astype(np.float32)
    fin = np.isfinite(want)
    assert np.array_equal(got[fin].view(np.uint32), want[fin].view(np.uint32))
    assert np.all(np.isnan(got[~fin & np.isnan(want)]))


def test_matmul16_kat64_exact(oracle, golden_dir):
    # TestHopper/MatMul16 (advanced_test.go:457-483): exact == against the CPU loop.
    af, bf, c = oracle.matmul16_kat(64)
    want = np.load(os.path.join(golden_dir, "matmul16_kat64.npz"))["want"]
    got = oracle.matmul16(af, bf, c)
    assert np.array_equal(got, want)


def test_matmul16_kat_fp16_inputs_are_exact(oracle):
    af, bf, _ = oracle.matmul16_kat(64)
    assert np.array_equal(oracle.f16_to_f32(oracle.f32_to_f16(af)), af)
    assert np.array_equal(oracle.f16_to_f32(oracle.f32_to_f16(bf)), bf)


def test_matmul16_n256_within_tolerance(oracle, golden_dir):
    n = 256
    a = oracle.f16_to_f32(oracle.f32_to_f16(oracle.uniform(n * n, 1))).reshape(n, n)
    b = oracle.f16_to_f32(oracle.f32_to_f16(oracle.uniform(n * n, 2))).reshape(n, n)
    c = oracle.uniform(n * n, 3).reshape(n, n)
    got = oracle.matmul16(a, b, c)
    want = np.load(os.path.join(golden_dir, "matmul16_n256.npz"))["want"]
    rel, mx, bad = oracle.error_norms(got, want)
    tol_rel, tol_max = oracle.gemm_tolerance(n, np.abs(a).max(), np.abs(b).max())
    assert bad == 0 and rel <= tol_rel and mx <= tol_max
    # The i-j-k float32 loop is far inside the bound (fp32 rounding only).
    assert rel < 1e-5


def test_gemm_ijk_row_range_and_threads_agree(oracle):
    M, N, K = 37, 24, 19
    a = oracle.uniform(M * K, 11).reshape(M, K)
    b = oracle.uniform(K * N, 12).reshape(K, N)
    c = oracle.uniform(M * N, 13).reshape(M, N)
    full = oracle.gemm_ijk(a, b, c)
    part = oracle.gemm_ijk(a, b, c, rows=(5, 20), threads=4)
    assert np.array_equal(full[5:20], part)
    ikj = oracle.gemm_ikj(a, b, c, threads=3)
    rel, _, _ = oracle.error_norms(ikj, full)
    assert rel < 1e-6


def test_vecadd_kat_exact(oracle, golden_dir):
    # TestVecAdd (main_test.go:26-60).
    g = json.load(open(os.path.join(golden_dir, "vecadd_kat.json")))
    a, b = oracle.vecadd_kat(g["n"])
    out = oracle.vecadd(a, b, threads=4)
    assert hashlib.sha256(out.tobytes()).hexdigest() == g["sha256"]
    for k, v in g["samples"].items():
        assert out[int(k)] == np.float32(v)


def test_vecadd_matches_numpy_on_random_bits(oracle):
    rng = np.random.default_rng(7)
    a = rng.integers(0, 2 ** 32, 100003, dtype=np.uint64).astype(np.uint32).view(np.float32)
    b = rng.integers(0, 2 ** 32, 100003, dtype=np.uint64).astype(np.uint32).view(np.float32)
    with np.errstate(all="ignore"):
        want = a + b
    got = oracle.vecadd(a, b)
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all()


def test_reduce_kat(oracle, golden_dir):
    # TestBlackwell (advanced_test.go:564-580).
    t = np.load(os.path.join(golden_dir, "reduce_kat.npz"))
    assert np.array_equal(oracle.reduce_kat(1024), t["x"])
    assert np.array_equal(oracle.reduce_f32(t["x"]), t["want"])


def test_reduce_go_semantics(oracle):
    # math.Min/Max: NaN propagates, -0 < +0, infinities win.
    x = np.zeros(32 * 4, dtype=np.float32)
    x[0:32] = np.linspace(-1, 1, 32)
    x[5] = np.nan
    x[32:64] = 0.0
    x[40] = -0.0
    x[64:96] = np.arange(32)
    x[70] = np.inf
    x[96:128] = np.arange(32)
    x[100] = -np.inf
    out = oracle.reduce_f32(x)
    assert np.isnan(out[0]) and np.isnan(out[1])
    assert out[2] == 0 and np.signbit(out[2]) and not np.signbit(out[3])
    assert out[4] == 0 and out[5] == np.inf
    assert out[6] == -np.inf and out[7] == 31


@pytest.mark.parametrize("seed", [1, 2, 3, 4, 5, 6, 7, 8])
def test_generator_pinned(oracle, golden_dir, seed):
    g = json.load(open(os.path.join(golden_dir, "generator.json")))[str(seed)]
    assert [oracle.stream_word(seed, i) for i in range(8)] == g["words"]
    assert np.array_equal(oracle.uniform(8, seed), np.array(g["uniform"], dtype=np.float32))
    # Box-Muller goes through libm log/cos in double: allow one float32 ulp.
    got = oracle.normal(8, seed)
    want = np.array(g["normal"], dtype=np.float32)
    assert np.all(np.abs(got - want) <= np.spacing(np.abs(want)))


def test_generator_offsets_compose(oracle):
    full = oracle.uniform(1000, 9)
    assert np.array_equal(full[300:700], oracle.uniform(400, 9, offset=300))


def test_golden_fixtures_are_reproducible(tmp_path, golden_dir):
    # tests/golden/make_golden.py (numpy only) regenerates every committed
    # fixture bit for bit.
    import json
    import os
    import shutil
    import subprocess
    import sys
    shutil.copy(os.path.join(golden_dir, "make_golden.py"), tmp_path)
    subprocess.run([sys.executable, str(tmp_path / "make_golden.py")], check=True, capture_output=True,
                   timeout=300)
    fixtures = [f for f in os.listdir(golden_dir) if f.endswith((".npz", ".json"))]
    assert fixtures
    for f in fixtures:
        a, b = os.path.join(golden_dir, f), str(tmp_path / f)
        if f.endswith(".npz"):
            A, B = np.load(a), np.load(b)
            assert set(A.files) == set(B.files), f
            for k in A.files:
                assert np.array_equal(A[k], B[k]), (f, k)
        else:
            assert json.load(open(a)) == json.load(open(b)), f
