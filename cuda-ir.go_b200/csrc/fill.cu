// fill.cu - seeded synthetic operands generated in HBM: the counter-based
// splitmix64 streams that the benchmark and the tests draw their inputs
// from, as uniform or Box-Muller normal values in fp32 or fp16.
//
// Element i of stream `seed` is computed from the 64-bit word
// splitmix64(seed * 0x9E3779B97F4A7C15 + offset + i) alone, so any slice of
// a matrix (a rank's block of rows of A, say) is generated where it lives,
// with no host round trip.  Every step is a correctly rounded IEEE operation
// in a fixed order (__fadd_rn / __dmul_rn / __ddiv_rn / __dsqrt_rn: nothing
// fused), and the logarithm and cosine of the Box-Muller transform are
// evaluated by short series in the same way, so the values are bit for bit
// those of any other evaluation of the same steps, in particular the CPU
// restatement the parity tests check against:
//   uniform  lo + (hi - lo) * (w >> 40) * 2^-24, in fp32;
//   normal   z = sqrt(-2 ln u1) cos(2 pi u2) in double with
//            u1 = (bits 40..63 + 1) 2^-24, u2 = bits 8..31 2^-24, then
//            mean + std z rounded to fp32;
//   fp16     the fp32 value rounded to nearest even.
// ln(m 2^-24): m = f 2^e, f in [sqrt(1/2), sqrt(2)), ln f = 2 atanh(s) with
// s = (f - 1)/(f + 1) and atanh(s) = s (1 + s^2/3 + s^4/5 + ...) to the
// s^24 term.  cos(2 pi v 2^-24): quadrant and angle from the integer v,
// the complement above pi/4, then the nested Taylor series of sin or cos to
// the x^20 term.  The coefficients are the rounded reciprocals, written as
// exact hexadecimal literals.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "cudair_internal.h"

namespace cudair {
namespace fill {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__device__ __forceinline__ double ln_u24(uint32_t m) {
    constexpr double kCoef[13] = {
        0x1.0000000000000p+0, 0x1.5555555555555p-2, 0x1.999999999999ap-3, 0x1.2492492492492p-3,
        0x1.c71c71c71c71cp-4, 0x1.745d1745d1746p-4, 0x1.3b13b13b13b14p-4, 0x1.1111111111111p-4,
        0x1.e1e1e1e1e1e1ep-5, 0x1.af286bca1af28p-5, 0x1.8618618618618p-5, 0x1.642c8590b2164p-5,
        0x1.47ae147ae147bp-5};  // 1/(2k+1)
    constexpr double kLn2 = 0x1.62e42fefa39efp-1;
    constexpr double kSqrt2 = 0x1.6a09e667f3bcdp+0;
    int e = 31 - __clz(m);  // floor(log2 m)
    double f = __ddiv_rn(static_cast<double>(m), static_cast<double>(1u << e));  // exact, [1, 2)
    if (f > kSqrt2) {
        f = __dmul_rn(f, 0.5);
        e += 1;
    }
    const double s = __ddiv_rn(__dsub_rn(f, 1.0), __dadd_rn(f, 1.0));
    const double w = __dmul_rn(s, s);
    double p = kCoef[12];
#pragma unroll
    for (int k = 11; k >= 0; --k) p = __dadd_rn(kCoef[k], __dmul_rn(w, p));
    const double t = __dmul_rn(__dmul_rn(2.0, s), p);
    return __dadd_rn(t, __dmul_rn(static_cast<double>(e - 24), kLn2));
}

__device__ __forceinline__ double cos_2pi_u24(uint32_t v) {
    constexpr double kSin[11] = {
        0.0, 0x1.5555555555555p-3, 0x1.999999999999ap-5, 0x1.8618618618618p-6, 0x1.c71c71c71c71cp-7,
        0x1.29e4129e4129ep-7, 0x1.a41a41a41a41ap-8, 0x1.3813813813814p-8, 0x1.e1e1e1e1e1e1ep-9,
        0x1.7f405fd017f40p-9, 0x1.3813813813814p-9};  // 1/((2k)(2k+1))
    constexpr double kCos[11] = {
        0.0, 0x1.0000000000000p-1, 0x1.5555555555555p-4, 0x1.1111111111111p-5, 0x1.2492492492492p-6,
        0x1.6c16c16c16c17p-7, 0x1.f07c1f07c1f08p-8, 0x1.6816816816817p-8, 0x1.1111111111111p-8,
        0x1.ac5701ac5701bp-9, 0x1.58ed2308158edp-9};  // 1/((2k-1)(2k))
    constexpr double kPiOver2p23 = 0x1.921fb54442d18p-22;
    const uint32_t q = v >> 22, r = v & 0x3fffffu;
    bool want_sin = (q & 1u) != 0;
    const bool neg = (q == 1u || q == 2u);
    uint32_t y = r;
    if (r > (1u << 21)) {
        y = (1u << 22) - r;
        want_sin = !want_sin;
    }
    const double x = __dmul_rn(static_cast<double>(y), kPiOver2p23);
    const double x2 = __dmul_rn(x, x);
    double p = 1.0, res;
    if (want_sin) {
#pragma unroll
        for (int k = 10; k >= 1; --k) p = __dsub_rn(1.0, __dmul_rn(__dmul_rn(x2, kSin[k]), p));
        res = __dmul_rn(x, p);
    } else {
#pragma unroll
        for (int k = 10; k >= 1; --k) p = __dsub_rn(1.0, __dmul_rn(__dmul_rn(x2, kCos[k]), p));
        res = p;
    }
    return neg ? -res : res;
}

// One value of the stream as fp32.
template <int DIST>
__device__ __forceinline__ float value(uint64_t w, double p0, double p1) {
    if (DIST == CUDAIR_FILL_UNIFORM) {
        const float lo = static_cast<float>(p0), hi = static_cast<float>(p1);
        const float u = __fmul_rn(static_cast<float>(w >> 40), 1.0f / 16777216.0f);
        return __fadd_rn(lo, __fmul_rn(__fsub_rn(hi, lo), u));
    }
    const uint32_t m = static_cast<uint32_t>((w >> 40) & 0xffffffu) + 1u;
    const uint32_t v = static_cast<uint32_t>((w >> 8) & 0xffffffu);
    const double r = __dsqrt_rn(__dmul_rn(-2.0, ln_u24(m)));
    const double z = __dmul_rn(r, cos_2pi_u24(v));
    return __double2float_rn(__dadd_rn(p0, __dmul_rn(p1, z)));
}

// Grid-stride over the n outputs; elements of a warp are consecutive, so
// the stores are coalesced.
template <int DIST, bool F16>
__global__ void __launch_bounds__(256) fill_kernel(void *__restrict__ out, long long n, uint64_t seed,
                                                   long long offset, double p0, double p1) {
    const uint64_t base = seed * 0x9E3779B97F4A7C15ull + static_cast<uint64_t>(offset);
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float x = value<DIST>(splitmix64(base + static_cast<uint64_t>(i)), p0, p1);
        if (F16)
            static_cast<__half *>(out)[i] = __float2half_rn(x);
        else
            static_cast<float *>(out)[i] = x;
    }
}

}  // namespace fill
}  // namespace cudair

using namespace cudair;

CUDAIR_API int cudair_fill(void *out, uint32_t out_type, uint32_t dist, int64_t n, uint64_t seed,
                           int64_t offset, double p0, double p1, void *stream) {
    clear_error();
    if (out_type != CUDAIR_FILL_F32 && out_type != CUDAIR_FILL_F16)
        return set_error(CUDAIR_ERR_INVALID, "cudair: fill: output type %u, want 0 (fp32) or 1 (fp16)", out_type);
    if (dist != CUDAIR_FILL_UNIFORM && dist != CUDAIR_FILL_NORMAL)
        return set_error(CUDAIR_ERR_INVALID, "cudair: fill: distribution %u, want 0 (uniform) or 1 (normal)",
                         dist);
    if (n < 0 || offset < 0)
        return set_error(CUDAIR_ERR_INVALID, "cudair: fill: n = %lld, offset = %lld", (long long)n,
                         (long long)offset);
    if (n == 0) return CUDAIR_OK;
    if (!out) return set_error(CUDAIR_ERR_INVALID, "cudair: fill: nil pointer");
    if (reinterpret_cast<uintptr_t>(out) & (out_type == CUDAIR_FILL_F16 ? 1u : 3u))
        return set_error(CUDAIR_ERR_INVALID, "cudair: fill: output not aligned to its element size");
    int sms = 0;
    int rc = sm_count_current_device(&sms);  // refuses a device other than sm_100
    if (rc != CUDAIR_OK) return rc;
    const long long blocks_needed = (n + 255) / 256;
    const unsigned grid = static_cast<unsigned>(blocks_needed < 8LL * sms ? blocks_needed : 8LL * sms);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const long long nn = static_cast<long long>(n), off = static_cast<long long>(offset);
    if (dist == CUDAIR_FILL_UNIFORM) {
        if (out_type == CUDAIR_FILL_F16)
            fill::fill_kernel<CUDAIR_FILL_UNIFORM, true><<<grid, 256, 0, s>>>(out, nn, seed, off, p0, p1);
        else
            fill::fill_kernel<CUDAIR_FILL_UNIFORM, false><<<grid, 256, 0, s>>>(out, nn, seed, off, p0, p1);
    } else {
        if (out_type == CUDAIR_FILL_F16)
            fill::fill_kernel<CUDAIR_FILL_NORMAL, true><<<grid, 256, 0, s>>>(out, nn, seed, off, p0, p1);
        else
            fill::fill_kernel<CUDAIR_FILL_NORMAL, false><<<grid, 256, 0, s>>>(out, nn, seed, off, p0, p1);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "fill_kernel launch");
    return CUDAIR_OK;
}
