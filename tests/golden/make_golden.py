"""Generates the golden fixtures in tests/golden/ with numpy only, independently
of the C oracle, from the closed-form inputs of cuda-ir.go's own tests:

  matmul16_kat64.npz   TestHopper/MatMul16 (advanced_test.go:457-483): n=64,
                       af=(i+2j)%7-3, bf=(3i+j)%5-2, c=j-i; the answer is exact
                       integer arithmetic (int64 here), so it is the one value
                       any correct float32 evaluation must produce.
  vecadd_kat.json      TestVecAdd (main_test.go:26-60): n=2^20, a=0.5i,
                       b=1000-i; sha256 of numpy's float32 a+b plus samples.
  reduce_kat.npz       TestBlackwell (advanced_test.go:564-580): float32(sin(i)),
                       n=1024, per-warp min/max.
  f16_table.npz        fp32 -> fp16 RNE for special values, every binade edge
                       and 2^14 random bit patterns, from numpy's IEEE
                       conversion (NaN inputs excluded: the reference maps them
                       to infinity, which test_oracle.py checks separately).
  generator.json       the first words / values of the seeded streams the
                       tests and the bench use, from a numpy restatement of the
                       counter-based splitmix64 generator, and sha256 pins of
                       2^16-value runs of the normal streams.
  matmul16_n256.npz    the seeded n=256 MatMul16 case (A,B = fp16(U(-1,1)),
                       C = U(-1,1), seeds 1,2,3): expected C in float64,
                       rounded to float32.

Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        x = x + GOLDEN
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return x ^ (x >> np.uint64(31))


def stream_words(seed: int, n: int, offset: int = 0) -> np.ndarray:
    with np.errstate(over="ignore"):
        base = np.uint64(seed) * GOLDEN
        idx = np.arange(offset, offset + n, dtype=np.uint64)
        return splitmix64(base + idx)


def uniform(seed: int, n: int, lo=-1.0, hi=1.0) -> np.ndarray:
    w = stream_words(seed, n)
    u = (w >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    return (np.float32(lo) + (np.float32(hi) - np.float32(lo)) * u).astype(np.float32)


# Box-Muller with its logarithm and cosine as fixed sequences of correctly
# rounded float64 operations (numpy never fuses a multiply and an add), the
# same steps in the same order as the oracle's C code: ln(m 2^-24) through
# ln f = 2 atanh((f-1)/(f+1)) with f in [sqrt(1/2), sqrt(2)), and cos(2 pi
# v 2^-24) by quadrant, complement above pi/4 and the nested Taylor series.
LN_COEF = [float.fromhex(h) for h in (
    "0x1.0000000000000p+0", "0x1.5555555555555p-2", "0x1.999999999999ap-3", "0x1.2492492492492p-3",
    "0x1.c71c71c71c71cp-4", "0x1.745d1745d1746p-4", "0x1.3b13b13b13b14p-4", "0x1.1111111111111p-4",
    "0x1.e1e1e1e1e1e1ep-5", "0x1.af286bca1af28p-5", "0x1.8618618618618p-5", "0x1.642c8590b2164p-5",
    "0x1.47ae147ae147bp-5")]
SIN_COEF = [0.0] + [float.fromhex(h) for h in (
    "0x1.5555555555555p-3", "0x1.999999999999ap-5", "0x1.8618618618618p-6", "0x1.c71c71c71c71cp-7",
    "0x1.29e4129e4129ep-7", "0x1.a41a41a41a41ap-8", "0x1.3813813813814p-8", "0x1.e1e1e1e1e1e1ep-9",
    "0x1.7f405fd017f40p-9", "0x1.3813813813814p-9")]
COS_COEF = [0.0] + [float.fromhex(h) for h in (
    "0x1.0000000000000p-1", "0x1.5555555555555p-4", "0x1.1111111111111p-5", "0x1.2492492492492p-6",
    "0x1.6c16c16c16c17p-7", "0x1.f07c1f07c1f08p-8", "0x1.6816816816817p-8", "0x1.1111111111111p-8",
    "0x1.ac5701ac5701bp-9", "0x1.58ed2308158edp-9")]
LN2 = float.fromhex("0x1.62e42fefa39efp-1")
SQRT2 = float.fromhex("0x1.6a09e667f3bcdp+0")
PI_OVER_2P23 = float.fromhex("0x1.921fb54442d18p-22")


def ln_u24(m: np.ndarray) -> np.ndarray:
    mant, ex = np.frexp(m.astype(np.float64))  # m = mant 2^ex, mant in [0.5, 1)
    f = mant * 2.0
    e = (ex - 1).astype(np.float64)
    big = f > SQRT2
    f = np.where(big, f * 0.5, f)
    e = np.where(big, e + 1.0, e)
    s = (f - 1.0) / (f + 1.0)
    w = s * s
    p = np.full_like(s, LN_COEF[12])
    for k in range(11, -1, -1):
        p = LN_COEF[k] + w * p
    return (2.0 * s) * p + (e - 24.0) * LN2


def cos_2pi_u24(v: np.ndarray) -> np.ndarray:
    q = v >> np.uint64(22)
    r = v & np.uint64(0x3FFFFF)
    want_sin = (q & np.uint64(1)) == 1
    neg = (q == 1) | (q == 2)
    comp = r > (1 << 21)
    y = np.where(comp, np.uint64(1 << 22) - r, r)
    want_sin = want_sin ^ comp
    x = y.astype(np.float64) * PI_OVER_2P23
    x2 = x * x
    ps = np.ones_like(x)
    pc = np.ones_like(x)
    for k in range(10, 0, -1):
        ps = 1.0 - (x2 * SIN_COEF[k]) * ps
        pc = 1.0 - (x2 * COS_COEF[k]) * pc
    res = np.where(want_sin, x * ps, pc)
    return np.where(neg, -res, res)


def normal(seed: int, n: int, mean=0.0, std=1.0) -> np.ndarray:
    w = stream_words(seed, n)
    m = ((w >> np.uint64(40)) & np.uint64(0xFFFFFF)) + np.uint64(1)
    v = (w >> np.uint64(8)) & np.uint64(0xFFFFFF)
    z = np.sqrt(-2.0 * ln_u24(m)) * cos_2pi_u24(v)
    return (mean + std * z).astype(np.float32)


def kat_matrices(n: int):
    i = np.arange(n).reshape(n, 1)
    j = np.arange(n).reshape(1, n)
    return (i + 2 * j) % 7 - 3, (3 * i + j) % 5 - 2, j - i


def main():
    # -- MatMul16 KATs (exact integer answer)
    for n in (64,):
        af, bf, c = kat_matrices(n)
        want = (af.astype(np.int64) @ bf.astype(np.int64) + c).astype(np.float32)
        np.savez_compressed(os.path.join(HERE, f"matmul16_kat{n}.npz"), want=want)

    # -- VecAdd KAT
    n = 1 << 20
    i = np.arange(n, dtype=np.float32)
    a = (i * np.float32(0.5)).astype(np.float32)
    b = (np.float32(1000) - i).astype(np.float32)
    out = (a + b).astype(np.float32)
    sample_idx = [0, 1, 2, 3, 9, 1000, 2001, 65535, n // 2, n - 1]
    json.dump({"n": n, "sha256": hashlib.sha256(out.tobytes()).hexdigest(),
               "samples": {str(k): float(out[k]) for k in sample_idx}},
              open(os.path.join(HERE, "vecadd_kat.json"), "w"), indent=1)

    # -- ReduceF32 KAT
    x = np.sin(np.arange(1024, dtype=np.float64)).astype(np.float32)
    w = x.reshape(-1, 32)
    mm = np.stack([w.min(axis=1), w.max(axis=1)], axis=1).reshape(-1).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "reduce_kat.npz"), x=x, want=mm)

    # -- fp32 -> fp16 table
    rng = np.random.default_rng(12345)
    specials = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65519.99, 65520.0, 65536.0, 1e9, -1e9,
                         np.inf, -np.inf, 2.0 ** -14, 2.0 ** -24, 2.0 ** -25, 2.0 ** -26,
                         1.5 * 2.0 ** -25, 2.0 ** -25 * (1 + 2.0 ** -20), 6.1e-5, 5.96e-8,
                         0.1, 1.0 / 3.0, 2049.0, 2051.0, 4097.0], dtype=np.float32)
    edges = []
    for e in range(-30, 17):
        for m in (1.0, 1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11, 1.0 + 2.0 ** -10, 2.0 - 2.0 ** -23):
            edges.append(m * 2.0 ** e)
    edges = np.array(edges, dtype=np.float32)
    bits = rng.integers(0, 2 ** 32, size=1 << 14, dtype=np.uint64).astype(np.uint32)
    rnd = bits.view(np.float32)
    inputs = np.concatenate([specials, edges, -edges, rnd]).astype(np.float32)
    inputs = inputs[~np.isnan(inputs)]
    with np.errstate(over="ignore"):
        halves = inputs.astype(np.float16).view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "f16_table.npz"), inputs=inputs, halves=halves)

    # -- generator pins
    gen = {}
    for seed in (1, 2, 3, 4, 5, 6, 7, 8):
        gen[str(seed)] = {
            "words": [int(v) for v in stream_words(seed, 8)],
            "uniform": [float(v) for v in uniform(seed, 8)],
            "normal": [float(v) for v in normal(seed, 8)],
        }
    # Longer runs of the normal stream, pinned by hash: the bench's operand
    # scale 1/sqrt(8192) and the unit scale, 2^16 values each.
    gen["normal_sha256"] = {
        f"{seed}/{name}": hashlib.sha256(normal(seed, 1 << 16, 0.0, std).tobytes()).hexdigest()
        for seed in (6, 7, 8, 9, 11, 12)
        for name, std in (("1", 1.0), ("1/sqrt(8192)", 1.0 / np.sqrt(8192.0)))}
    json.dump(gen, open(os.path.join(HERE, "generator.json"), "w"), indent=1)

    # -- seeded n = 256 MatMul16 case
    n = 256
    a16 = uniform(1, n * n).reshape(n, n).astype(np.float16)
    b16 = uniform(2, n * n).reshape(n, n).astype(np.float16)
    c = uniform(3, n * n).reshape(n, n)
    want = (a16.astype(np.float64) @ b16.astype(np.float64) + c.astype(np.float64)).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "matmul16_n256.npz"), want=want)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
