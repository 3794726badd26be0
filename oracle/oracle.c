/*
 * CPU oracle for the MatMul16 / VecAdd / ReduceF32 path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, in plain C, the CPU models
 * that cuda-ir.go's own Go tests use to check its kernels.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it, and only as
 * the checker or the timed CPU baseline: no product code path calls it.
 *
 * Compiled with -O2 -ffp-contract=off so that every float expression below
 * rounds exactly like the Go loops it restates (Go never fuses a*b+c).
 *
 * Parity pin: the Go toolchain is absent, so the reference cannot be built or
 * run here.  The restatement is pinned by (1) the reference tests' closed-form
 * known-answer inputs (the n=64 integer-valued matmul, the 2^20 VecAdd
 * ramp, the sin(i) warp reduction), whose answers are reproduced by an
 * independent numpy computation in tests/golden/make_golden.py, and (2)
 * numpy's IEEE float16 conversion for the fp32->fp16 rounding.
 * See tests/test_oracle.py.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stddef.h>
#include <pthread.h>
#include <unistd.h>

#define EXPORT __attribute__((visibility("default")))

/* ---- a minimal parallel-for over index ranges ------------------------- */

typedef void (*range_fn)(void *ctx, int64_t lo, int64_t hi);

struct par_job {
    range_fn fn;
    void *ctx;
    int64_t n, chunk;
    int64_t next; /* claimed with __atomic_fetch_add */
};

static void *par_worker(void *p)
{
    struct par_job *j = (struct par_job *)p;
    for (;;) {
        int64_t lo = __atomic_fetch_add(&j->next, j->chunk, __ATOMIC_RELAXED);
        if (lo >= j->n)
            break;
        int64_t hi = lo + j->chunk < j->n ? lo + j->chunk : j->n;
        j->fn(j->ctx, lo, hi);
    }
    return NULL;
}

/* Runs fn over [0, n) in chunks on `threads` threads (the caller is one). */
static void par_for(int64_t n, int threads, int64_t chunk, range_fn fn, void *ctx)
{
    if (n <= 0)
        return;
    if (chunk < 1)
        chunk = 1;
    if (threads > 64)
        threads = 64;
    if (threads <= 1 || n <= chunk) {
        fn(ctx, 0, n);
        return;
    }
    struct par_job job = {fn, ctx, n, chunk, 0};
    pthread_t tid[64];
    int started = 0;
    for (int t = 1; t < threads; t++)
        if (pthread_create(&tid[started], NULL, par_worker, &job) == 0)
            started++;
    par_worker(&job);
    for (int t = 0; t < started; t++)
        pthread_join(tid[t], NULL);
}

EXPORT int oracle_num_threads(void)
{
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

static int auto_threads(int64_t n)
{
    return n > (1 << 20) ? oracle_num_threads() : 1;
}

/* ---- fp16 conversion -------------------------------------------------- */

/*
 * fp32 -> IEEE binary16, round to nearest even.
 * Follows float32ToHalf in advanced_test.go:597-623 step for step: the
 * exponent is rebiased (-127+15); exponents >= 31 give infinity (so a NaN
 * input also gives infinity: the reference has no NaN branch); exponents
 * <= 0 produce a subnormal by shifting the mantissa with its hidden bit,
 * and values below 2^-25 (exp < -10) flush to signed zero; the dropped bits
 * decide the rounding (above half rounds up, exactly half rounds to even).
 * A carry out of the mantissa propagates into the exponent, which is what
 * makes 65520 round up to infinity.
 */
EXPORT uint16_t oracle_f32_to_f16(float f)
{
    uint32_t b;
    memcpy(&b, &f, 4);
    uint16_t sign = (uint16_t)(b >> 16) & 0x8000u;
    int32_t exp = (int32_t)((b >> 23) & 0xffu) - 127 + 15;
    uint32_t mant = b & 0x7fffffu;
    if (exp >= 31)
        return sign | 0x7c00u;
    if (exp <= 0) {
        if (exp < -10)
            return sign;
        mant |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - exp);
        uint16_t h = (uint16_t)(mant >> shift);
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (h & 1u)))
            h++;
        return sign | h;
    }
    uint16_t h = sign | (uint16_t)((uint32_t)exp << 10) | (uint16_t)(mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u)))
        h++;
    return h;
}

/* binary16 -> fp32, exact (every half is a float). */
EXPORT float oracle_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else { /* subnormal: value = mant * 2^-24, exact in float */
            float v = (float)mant * (1.0f / 16777216.0f);
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

struct cvt_ctx {
    const void *in;
    void *out;
};

static void f2h_range(void *p, int64_t lo, int64_t hi)
{
    struct cvt_ctx *c = (struct cvt_ctx *)p;
    const float *in = (const float *)c->in;
    uint16_t *out = (uint16_t *)c->out;
    for (int64_t i = lo; i < hi; i++)
        out[i] = oracle_f32_to_f16(in[i]);
}

static void h2f_range(void *p, int64_t lo, int64_t hi)
{
    struct cvt_ctx *c = (struct cvt_ctx *)p;
    const uint16_t *in = (const uint16_t *)c->in;
    float *out = (float *)c->out;
    for (int64_t i = lo; i < hi; i++)
        out[i] = oracle_f16_to_f32(in[i]);
}

EXPORT void oracle_f32_to_f16_array(const float *in, uint16_t *out, int64_t n)
{
    struct cvt_ctx c = {in, out};
    par_for(n, auto_threads(n), 1 << 16, f2h_range, &c);
}

EXPORT void oracle_f16_to_f32_array(const uint16_t *in, float *out, int64_t n)
{
    struct cvt_ctx c = {in, out};
    par_for(n, auto_threads(n), 1 << 16, h2f_range, &c);
}

/* ---- MatMul16 CPU model ---------------------------------------------- */

struct gemm_ctx {
    int64_t M, N, K;
    const float *af;
    int64_t lda;
    const float *bf;
    int64_t ldb;
    const float *c;
    int64_t ldc;
    float *out;
    int64_t ldo;
    int64_t row0;
};

/* Rows [row0+lo, row0+hi) of the i-j-k loop nest. */
static void ijk_rows(void *p, int64_t lo, int64_t hi)
{
    struct gemm_ctx *g = (struct gemm_ctx *)p;
    for (int64_t r = lo; r < hi; r++) {
        int64_t i = g->row0 + r;
        for (int64_t j = 0; j < g->N; j++) {
            float s = g->c[i * g->ldc + j];
            for (int64_t k = 0; k < g->K; k++)
                s += g->af[i * g->lda + k] * g->bf[k * g->ldb + j];
            g->out[r * g->ldo + j] = s;
        }
    }
}

/*
 * want[i][j] = c[i][j] + sum_k af[i][k] * bf[k][j], in float32, k ascending
 * from 0 with the accumulator initialised to c[i][j]: the i-j-k loop of
 * advanced_test.go:466-475.  af/bf are the fp16-rounded operands widened to
 * float32 (the test builds af/bf first and converts them to half).
 *
 * Generalised to M x N x K with leading dimensions and a row range
 * [row0, row1) (out holds rows row0.. at stride ldo) so a bounded sample of
 * rows can be timed; rows are independent, so the sample's cost scales
 * exactly with the row count.  threads <= 1 runs the reference's single loop
 * nest; threads > 1 hands whole rows to threads without changing any
 * per-element arithmetic.
 */
EXPORT void oracle_gemm_ijk(int64_t M, int64_t N, int64_t K,
                            const float *af, int64_t lda,
                            const float *bf, int64_t ldb,
                            const float *c, int64_t ldc,
                            float *out, int64_t ldo,
                            int64_t row0, int64_t row1, int threads)
{
    if (row1 > M)
        row1 = M;
    struct gemm_ctx g = {M, N, K, af, lda, bf, ldb, c, ldc, out, ldo, row0};
    par_for(row1 - row0, threads, 1, ijk_rows, &g);
}

/* Square form with the reference's signature shape (n x n, ld = n). */
EXPORT void oracle_matmul16(const float *af, const float *bf, const float *c,
                            float *out, int32_t n)
{
    oracle_gemm_ijk(n, n, n, af, n, bf, n, c, n, out, n, 0, n, 1);
}

static void ikj_rows(void *p, int64_t lo, int64_t hi)
{
    struct gemm_ctx *g = (struct gemm_ctx *)p;
    for (int64_t r = lo; r < hi; r++) {
        int64_t i = g->row0 + r;
        float *o = g->out + r * g->ldo;
        for (int64_t j = 0; j < g->N; j++)
            o[j] = g->c[i * g->ldc + j];
        for (int64_t k = 0; k < g->K; k++) {
            float a = g->af[i * g->lda + k];
            const float *br = g->bf + k * g->ldb;
            for (int64_t j = 0; j < g->N; j++)
                o[j] += a * br[j];
        }
    }
}

/*
 * fp32 GEMM over a row range in a cache-friendly i-k-j order: the tolerance
 * reference at sizes the i-j-k loop cannot finish in seconds.  Its summation
 * order differs from the i-j-k model, which the tolerance-based GEMM checks
 * allow; the exact small-integer checks use oracle_gemm_ijk.
 */
EXPORT void oracle_gemm_ikj(int64_t M, int64_t N, int64_t K,
                            const float *af, int64_t lda,
                            const float *bf, int64_t ldb,
                            const float *c, int64_t ldc,
                            float *out, int64_t ldo,
                            int64_t row0, int64_t row1, int threads)
{
    if (row1 > M)
        row1 = M;
    struct gemm_ctx g = {M, N, K, af, lda, bf, ldb, c, ldc, out, ldo, row0};
    par_for(row1 - row0, threads, 1, ikj_rows, &g);
}

/* ---- VecAdd CPU model -------------------------------------------------- */

struct add_ctx {
    const float *a, *b;
    float *out;
};

static void add_range(void *p, int64_t lo, int64_t hi)
{
    struct add_ctx *c = (struct add_ctx *)p;
    for (int64_t i = lo; i < hi; i++)
        c->out[i] = c->a[i] + c->b[i];
}

/* out[i] = a[i] + b[i] in float32: the check of main_test.go:51. */
EXPORT void oracle_vecadd(const float *a, const float *b, float *out,
                          int64_t n, int threads)
{
    struct add_ctx c = {a, b, out};
    par_for(n, threads, 1 << 16, add_range, &c);
}

/* ---- Saxpy / Square CPU models (examples/vecadd/run/main.go:62-76) ------- */

/* y[i] = alpha * x[i] + y[i], product and sum rounded separately. */
EXPORT void oracle_saxpy(float alpha, const float *x, float *y, int64_t n)
{
    for (int64_t i = 0; i < n; i++) {
        float p = alpha * x[i];
        y[i] = p + y[i];
    }
}

/* x[i] = x[i] * x[i]. */
EXPORT void oracle_square(float *x, int64_t n)
{
    for (int64_t i = 0; i < n; i++)
        x[i] = x[i] * x[i];
}

/* ---- ReduceF32 CPU model ----------------------------------------------- */

/* Go's math.Min / math.Max on float64 (-Inf/+Inf win, then NaN, -0 < +0). */
static double go_min(double x, double y)
{
    if (isinf(x) && x < 0) return x;
    if (isinf(y) && y < 0) return y;
    if (isnan(x) || isnan(y)) return NAN;
    if (x == 0 && x == y) return signbit(x) ? x : y;
    return x < y ? x : y;
}

static double go_max(double x, double y)
{
    if (isinf(x) && x > 0) return x;
    if (isinf(y) && y > 0) return y;
    if (isnan(x) || isnan(y)) return NAN;
    if (x == 0 && x == y) return signbit(x) ? y : x;
    return x > y ? x : y;
}

/*
 * out[2w] = min, out[2w+1] = max of in[32w .. 32w+31], folded left to right
 * through float64 math.Min/Max and back to float32, as
 * advanced_test.go:572-579 does.
 */
EXPORT void oracle_reduce_f32(const float *in, float *out, int32_t n)
{
    for (int32_t w = 0; w < n / 32; w++) {
        float mn = in[w * 32], mx = in[w * 32];
        for (int32_t l = 0; l < 32; l++) {
            float v = in[w * 32 + l];
            mn = (float)go_min((double)mn, (double)v);
            mx = (float)go_max((double)mx, (double)v);
        }
        out[2 * w] = mn;
        out[2 * w + 1] = mx;
    }
}

/* ---- seeded synthetic inputs ------------------------------------------ */

/*
 * Counter-based generator: element i of stream `seed` is
 * splitmix64(seed * 0x9E3779B97F4A7C15 + i), so any slice can be produced
 * independently (and in parallel) and a second implementation (numpy, in
 * tests/golden/make_golden.py) reproduces it bit for bit.
 */
static inline uint64_t splitmix64(uint64_t x)
{
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static inline uint64_t stream_word(uint64_t seed, uint64_t i)
{
    return splitmix64(seed * 0x9E3779B97F4A7C15ull + i);
}

EXPORT uint64_t oracle_stream_word(uint64_t seed, uint64_t i)
{
    return stream_word(seed, i);
}

struct fill_ctx {
    float *out;
    uint64_t seed;
    int64_t offset;
    double a, b;
};

/* U(lo, hi) from 24 random bits: lo + (hi - lo) * ((w >> 40) * 2^-24). */
static void uniform_range(void *p, int64_t lo, int64_t hi)
{
    struct fill_ctx *c = (struct fill_ctx *)p;
    float flo = (float)c->a, fhi = (float)c->b;
    for (int64_t i = lo; i < hi; i++) {
        uint64_t w = stream_word(c->seed, (uint64_t)(c->offset + i));
        float u = (float)(w >> 40) * (1.0f / 16777216.0f);
        c->out[i] = flo + (fhi - flo) * u;
    }
}

EXPORT void oracle_fill_uniform(float *out, int64_t n, uint64_t seed,
                                int64_t offset, float lo, float hi)
{
    struct fill_ctx c = {out, seed, offset, lo, hi};
    par_for(n, auto_threads(n), 1 << 16, uniform_range, &c);
}

/*
 * The logarithm and cosine of the Box-Muller transform below, written with
 * correctly rounded double +, -, *, / and sqrt only, in a fixed order, so
 * that any IEEE-754 evaluation of the same steps (numpy in
 * tests/golden/make_golden.py, the library's device fill kernel) gets the
 * same bits; libm's log and cos differ between implementations in the last
 * bit.  The coefficients are exact hex literals of the rounded reciprocals.
 *
 * ln(m 2^-24), integer 1 <= m <= 2^24: m = f 2^e with f in [sqrt(1/2),
 * sqrt(2)); ln f = 2 atanh(s), s = (f-1)/(f+1), by the series
 * atanh(s) = s (1 + s^2/3 + s^4/5 + ...) to the s^24 term (|s| <= 0.1716,
 * so the first dropped term is below 2^-60 of the sum).
 */
static const double kLnCoef[13] = {
    0x1.0000000000000p+0, 0x1.5555555555555p-2, 0x1.999999999999ap-3, 0x1.2492492492492p-3,
    0x1.c71c71c71c71cp-4, 0x1.745d1745d1746p-4, 0x1.3b13b13b13b14p-4, 0x1.1111111111111p-4,
    0x1.e1e1e1e1e1e1ep-5, 0x1.af286bca1af28p-5, 0x1.8618618618618p-5, 0x1.642c8590b2164p-5,
    0x1.47ae147ae147bp-5}; /* 1/(2k+1) */
/* Taylor series of sin and cos in nested form: 1/((2k)(2k+1)), 1/((2k-1)(2k)). */
static const double kSinCoef[11] = {
    0.0, 0x1.5555555555555p-3, 0x1.999999999999ap-5, 0x1.8618618618618p-6, 0x1.c71c71c71c71cp-7,
    0x1.29e4129e4129ep-7, 0x1.a41a41a41a41ap-8, 0x1.3813813813814p-8, 0x1.e1e1e1e1e1e1ep-9,
    0x1.7f405fd017f40p-9, 0x1.3813813813814p-9};
static const double kCosCoef[11] = {
    0.0, 0x1.0000000000000p-1, 0x1.5555555555555p-4, 0x1.1111111111111p-5, 0x1.2492492492492p-6,
    0x1.6c16c16c16c17p-7, 0x1.f07c1f07c1f08p-8, 0x1.6816816816817p-8, 0x1.1111111111111p-8,
    0x1.ac5701ac5701bp-9, 0x1.58ed2308158edp-9};
static const double kLn2 = 0x1.62e42fefa39efp-1;
static const double kSqrt2 = 0x1.6a09e667f3bcdp+0;
static const double kPiOver2p23 = 0x1.921fb54442d18p-22; /* pi / 2^23 */

static double ln_u24(uint32_t m)
{
    int e = 31 - __builtin_clz(m);           /* floor(log2 m) */
    double f = (double)m / (double)(1u << e); /* exact, in [1, 2) */
    if (f > kSqrt2) {
        f = f * 0.5; /* exact */
        e += 1;
    }
    double s = (f - 1.0) / (f + 1.0); /* f - 1 and f + 1 are exact */
    double w = s * s;
    double p = kLnCoef[12];
    for (int k = 11; k >= 0; k--)
        p = kLnCoef[k] + w * p;
    double t = (2.0 * s) * p;
    return t + (double)(e - 24) * kLn2;
}

/* cos(2 pi v 2^-24), integer 0 <= v < 2^24: the quadrant q and the angle
 * x = r pi 2^-23 inside it (r < 2^22) come from the integer exactly; for
 * x > pi/4 the complement pi/2 - x = (2^22 - r) pi 2^-23 is used, so the
 * series (to the x^20 term) only sees |x| <= pi/4. */
static double cos_2pi_u24(uint32_t v)
{
    uint32_t q = v >> 22, r = v & 0x3fffffu;
    int want_sin = (int)(q & 1u);      /* q = 1, 3: -sin x, sin x */
    int neg = (q == 1u || q == 2u);
    uint32_t y = r;
    if (r > (1u << 21)) {
        y = (1u << 22) - r;
        want_sin ^= 1;
    }
    double x = (double)y * kPiOver2p23;
    double x2 = x * x;
    double p = 1.0;
    double res;
    if (want_sin) {
        for (int k = 10; k >= 1; k--)
            p = 1.0 - (x2 * kSinCoef[k]) * p;
        res = x * p;
    } else {
        for (int k = 10; k >= 1; k--)
            p = 1.0 - (x2 * kCosCoef[k]) * p;
        res = p;
    }
    return neg ? -res : res;
}

/*
 * N(mean, std) by Box-Muller on two 24-bit uniforms taken from one 64-bit
 * word: u1 = (bits 40..63 + 1) * 2^-24 in (0,1], u2 = bits 8..31 * 2^-24 in
 * [0,1); z = sqrt(-2 ln u1) cos(2 pi u2) in double (ln and cos as above),
 * then mean + std z rounded to float.
 */
static double normal_z(uint64_t w)
{
    uint32_t m = (uint32_t)((w >> 40) & 0xffffffu) + 1u;
    uint32_t v = (uint32_t)((w >> 8) & 0xffffffu);
    double r = sqrt(-2.0 * ln_u24(m));
    return r * cos_2pi_u24(v);
}

static void normal_range(void *p, int64_t lo, int64_t hi)
{
    struct fill_ctx *c = (struct fill_ctx *)p;
    for (int64_t i = lo; i < hi; i++) {
        uint64_t w = stream_word(c->seed, (uint64_t)(c->offset + i));
        double z = normal_z(w);
        c->out[i] = (float)(c->a + c->b * z);
    }
}

EXPORT void oracle_fill_normal(float *out, int64_t n, uint64_t seed,
                               int64_t offset, double mean, double stddev)
{
    struct fill_ctx c = {out, seed, offset, mean, stddev};
    par_for(n, auto_threads(n), 1 << 16, normal_range, &c);
}

/* ---- tolerance checker -------------------------------------------------- */

/*
 * Error norms of got against want over n elements, accumulated in double:
 *   res[0] = ||got - want||_F / ||want||_F   (relative Frobenius)
 *   res[1] = max |got - want|
 *   res[2] = number of non-finite entries in got
 */
EXPORT void oracle_error_norms(const float *got, const float *want, int64_t n,
                               double *res)
{
    double num = 0, den = 0, mx = 0, bad = 0;
    for (int64_t i = 0; i < n; i++) {
        double g = got[i], w = want[i];
        if (!isfinite(g)) {
            bad += 1;
            continue;
        }
        double d = g - w;
        num += d * d;
        den += w * w;
        double ad = fabs(d);
        if (ad > mx)
            mx = ad;
    }
    res[0] = den > 0 ? sqrt(num / den) : sqrt(num);
    res[1] = mx;
    res[2] = bad;
}
