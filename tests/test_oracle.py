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
    # Box-Muller's logarithm and cosine are fixed sequences of correctly
    # rounded operations, so the numpy restatement matches bit for bit.
    assert np.array_equal(oracle.normal(8, seed), np.array(g["normal"], dtype=np.float32))


@pytest.mark.parametrize("key", ["6/1", "7/1/sqrt(8192)", "8/1", "9/1", "11/1/sqrt(8192)",
                                 "12/1/sqrt(8192)"])
def test_normal_stream_pinned_by_hash(oracle, golden_dir, key):
    import hashlib
    want = json.load(open(os.path.join(golden_dir, "generator.json")))["normal_sha256"][key]
    seed, _, scale = key.partition("/")
    std = 1.0 if scale == "1" else 1.0 / np.sqrt(8192.0)
    got = oracle.normal(1 << 16, int(seed), 0.0, std)
    assert hashlib.sha256(got.tobytes()).hexdigest() == want


def test_normal_stream_statistics(oracle):
    # The restated ln/cos keep Box-Muller's distribution: mean 0, variance 1,
    # and within 1e-6 of libm's transform on the same words.
    z = oracle.normal(1 << 20, 21)
    assert abs(float(z.mean())) < 5e-3 and abs(float(z.std()) - 1.0) < 5e-3
    words = np.array([oracle.stream_word(21, i) for i in range(4096)], dtype=np.uint64)
    u1 = (((words >> np.uint64(40)) & np.uint64(0xFFFFFF)).astype(np.float64) + 1.0) / 16777216.0
    u2 = ((words >> np.uint64(8)) & np.uint64(0xFFFFFF)).astype(np.float64) / 16777216.0
    libm = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    assert np.max(np.abs(z[:4096] - libm)) < 1e-6


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
