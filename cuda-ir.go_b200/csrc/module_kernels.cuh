// module_kernels.cuh - the kernels that keep the reference's entry-point
// names and parameter ABI (one 8-byte pointer per cuda.Buf[T], int32 n), so a
// caller that loads the module and launches them by name with the reference's
// own launch configurations gets the same results.
//
// Compiled twice: into cudair_kernels.cubin (the loadable module that stands
// in for the PTX the reference's compiler emits) and into libcudair_b200.so
// (behind the C-ABI launchers).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

// ---- Streaming helper (VecAdd, Saxpy, Square) ----------------------------------

namespace cudair_detail {

// out[i] = f(in0[i] (, in1[i])) over n4 16-byte vectors, in chunks of
// blockDim.x * V vectors: block b takes chunks b, b + gridDim.x, ..., and
// thread t of a block the vectors t, t + blockDim.x, ... of its chunk, so
// every warp access is coalesced and all of a thread's loads are issued
// before its stores.  Under the library's launch (one chunk per block, many
// blocks) the hardware hands chunks to SMs as they finish, so SMs that get
// more bandwidth stream more; a persistent grid-stride split fixes every
// SM's share in advance and ends with the slowest one (VecAdd at 2^28:
// 0.50 against 0.455 ms).  Under any other launch the loop still covers all
// vectors.  Streaming (evict-first) cache policy: every byte is touched once.
template <int V, int NIN, class F>
__device__ __forceinline__ void stream_chunks(const float4 *in0, const float4 *in1, float4 *out,
                                              int64_t n4, F f) {
    // n4 < 2^29 (n is an int32), so every vector index inside a chunk fits
    // 32 bits; only the chunk cursor, whose stride can be huge under an
    // arbitrary launch, is kept in 64.
    const uint32_t T = blockDim.x, chunk = T * V;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * chunk;
    for (uint64_t c0 = static_cast<uint64_t>(blockIdx.x) * chunk; c0 < static_cast<uint64_t>(n4); c0 += stride) {
        const uint32_t i = static_cast<uint32_t>(c0) + threadIdx.x;
        float4 x[V], y[V];
        if (c0 + chunk <= static_cast<uint64_t>(n4)) {
#pragma unroll
            for (int k = 0; k < V; ++k) {
                x[k] = __ldcs(in0 + (i + k * T));
                if constexpr (NIN == 2) y[k] = __ldcs(in1 + (i + k * T));
            }
#pragma unroll
            for (int k = 0; k < V; ++k) {
                if constexpr (NIN == 2) __stcs(out + (i + k * T), f(x[k], y[k]));
                else __stcs(out + (i + k * T), f(x[k]));
            }
        } else {
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const uint32_t j = i + k * T;
                if (j < static_cast<uint64_t>(n4)) {
                    x[k] = __ldcs(in0 + j);
                    if constexpr (NIN == 2) {
                        y[k] = __ldcs(in1 + j);
                        __stcs(out + j, f(x[k], y[k]));
                    } else {
                        __stcs(out + j, f(x[k]));
                    }
                }
            }
        }
    }
}

// Vectors per thread and chunk: two 16-byte loads in flight per thread (at
// 2048 threads per SM, 64 KB per SM), the fastest of 1/2/4/8 at 128-512
// threads per block.
constexpr int kVecAddV = 1;  // two inputs
constexpr int kSquareV = 2;  // one input

struct AddOp {
    __device__ __forceinline__ float4 operator()(const float4 &a, const float4 &b) const {
        return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
    }
};
struct SaxpyOp {
    float alpha;
    __device__ __forceinline__ float4 operator()(const float4 &x, const float4 &y) const {
        return make_float4(__fadd_rn(__fmul_rn(alpha, x.x), y.x), __fadd_rn(__fmul_rn(alpha, x.y), y.y),
                           __fadd_rn(__fmul_rn(alpha, x.z), y.z), __fadd_rn(__fmul_rn(alpha, x.w), y.w));
    }
};
struct SquareOp {
    __device__ __forceinline__ float4 operator()(const float4 &x) const {
        return make_float4(__fmul_rn(x.x, x.x), __fmul_rn(x.y, x.y), __fmul_rn(x.z, x.z), __fmul_rn(x.w, x.w));
    }
};

}  // namespace cudair_detail

// ---- VecAdd -----------------------------------------------------------------

// out[i] = a[i] + b[i] for i < n.  examples/vecadd/vecadd.go:6-11.
//
// The reference gives each thread one scalar element (launched
// LaunchConfig1D(n, 256), main_test.go:37).  Here the 16-byte-aligned middle
// of the arrays streams in chunks of 16-byte vectors (stream_chunks above),
// with a few scalar elements before and after it, so the same entry is
// correct under that launch and saturates HBM under the library's launch of
// one 512-vector chunk per block.  When the three pointers do not share their
// offset within 16 bytes every element is done by a scalar loop.  The add is
// IEEE round-to-nearest, bit-exact with the CPU's float32 add.
extern "C" __global__ void __launch_bounds__(1024, 2)
    VecAdd(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ out,
           int n) {
    if (n <= 0) return;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const uintptr_t mis = reinterpret_cast<uintptr_t>(out) & 15u;
    if ((reinterpret_cast<uintptr_t>(a) & 15u) == mis &&
        (reinterpret_cast<uintptr_t>(b) & 15u) == mis && (mis & 3u) == 0) {
        int64_t head = static_cast<int64_t>((16u - mis) & 15u) >> 2;  // scalars before 16B
        if (head > n) head = n;
        for (int64_t j = tid; j < head; j += nthr) out[j] = __fadd_rn(a[j], b[j]);
        const int64_t n4 = (n - head) >> 2;
        cudair_detail::stream_chunks<cudair_detail::kVecAddV, 2>(
            reinterpret_cast<const float4 *>(a + head), reinterpret_cast<const float4 *>(b + head),
            reinterpret_cast<float4 *>(out + head), n4, cudair_detail::AddOp{});
        for (int64_t t = head + 4 * n4 + tid; t < n; t += nthr) out[t] = __fadd_rn(a[t], b[t]);
    } else {
        for (int64_t i = tid; i < n; i += nthr) out[i] = __fadd_rn(a[i], b[i]);
    }
}

// ---- Saxpy, Square (the rest of the vecadd package) ------------------------------

// y[i] = alpha * x[i] + y[i] for i < n (examples/vecadd/vecadd.go:13-18),
// streamed like VecAdd (scalar head and tail, 16-byte chunks between, a
// scalar loop when x and y do not share their offset within 16 bytes).  The
// product and the sum are rounded separately (no fused multiply-add), as the
// reference's CPU check computes them (vecadd/run/main.go:62-69).
extern "C" __global__ void __launch_bounds__(1024, 2)
    Saxpy(float alpha, const float *__restrict__ x, float *__restrict__ y, int n) {
    if (n <= 0) return;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const uintptr_t mis = reinterpret_cast<uintptr_t>(y) & 15u;
    if ((reinterpret_cast<uintptr_t>(x) & 15u) == mis && (mis & 3u) == 0) {
        int64_t head = static_cast<int64_t>((16u - mis) & 15u) >> 2;
        if (head > n) head = n;
        for (int64_t j = tid; j < head; j += nthr) y[j] = __fadd_rn(__fmul_rn(alpha, x[j]), y[j]);
        const int64_t n4 = (n - head) >> 2;
        cudair_detail::stream_chunks<cudair_detail::kVecAddV, 2>(
            reinterpret_cast<const float4 *>(x + head), reinterpret_cast<const float4 *>(y + head),
            reinterpret_cast<float4 *>(y + head), n4, cudair_detail::SaxpyOp{alpha});
        for (int64_t t = head + 4 * n4 + tid; t < n; t += nthr) y[t] = __fadd_rn(__fmul_rn(alpha, x[t]), y[t]);
    } else {
        for (int64_t i = tid; i < n; i += nthr) y[i] = __fadd_rn(__fmul_rn(alpha, x[i]), y[i]);
    }
}

// x[i] = x[i] * x[i] in place (vecadd.go:20-28; the reference gives each
// thread one element), streamed like VecAdd.
extern "C" __global__ void __launch_bounds__(1024, 2) Square(float *__restrict__ x, int n) {
    if (n <= 0) return;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const uintptr_t mis = reinterpret_cast<uintptr_t>(x) & 15u;
    if ((mis & 3u) == 0) {
        int64_t head = static_cast<int64_t>((16u - mis) & 15u) >> 2;
        if (head > n) head = n;
        for (int64_t j = tid; j < head; j += nthr) x[j] = __fmul_rn(x[j], x[j]);
        const int64_t n4 = (n - head) >> 2;
        float4 *x4 = reinterpret_cast<float4 *>(x + head);
        cudair_detail::stream_chunks<cudair_detail::kSquareV, 1>(x4, nullptr, x4, n4, cudair_detail::SquareOp{});
        for (int64_t t = head + 4 * n4 + tid; t < n; t += nthr) x[t] = __fmul_rn(x[t], x[t]);
    } else {
        for (int64_t i = tid; i < n; i += nthr) x[i] = __fmul_rn(x[i], x[i]);
    }
}

// ---- MatMul16 ---------------------------------------------------------------

namespace cudair_detail {

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void *p) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a));
}

// D = A(16x16, row) . B(16x8, col) + D, fp16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 16-byte global -> shared copy that bypasses L1 (cp.async.cg); completes
// with the thread's next cp.async.wait_group.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace cudair_detail

// C = A.B + C for n x n row-major matrices (fp16 A, B; fp32 C in place),
// examples/hopper/hopper.go:201-226, under the reference's launch contract:
// grid (n/16, n/16), one 32-thread block per 16x16 tile of C
// (advanced_test.go:477).  n must be a multiple of 16, as there.
//
// This entry serves callers that launch the module kernel themselves with
// that geometry; the throughput path is the tcgen05 kernel behind
// cudair_matmul16(), which needs tensor-map parameters this signature cannot
// carry (cudair_matmul16 also launches this kernel for n <= 512, where its
// latency is the lower one).  The warp keeps its C tile in mma.sync
// accumulators initialised from C and streams 16-wide k-slices of A and B
// through a ring of MM_STAGES slices in padded shared memory (48-byte rows:
// conflict-free ldmatrix), filled by cp.async, so up to MM_STAGES slices are
// in flight at once: at n <= 256 the whole K panel is requested together and
// the loads cost one round trip instead of one per slice.  Each slice feeds
// two m16n8k16 MMAs; C is written back once.  Threads beyond the first warp
// return.
constexpr int MM_STAGES = 16;  // 2 x 16 x 768 B = 24 KB of static shared memory

extern "C" __global__ void __launch_bounds__(32)
    MatMul16(const __half *__restrict__ a, const __half *__restrict__ b, float *__restrict__ c,
             int n) {
    using namespace cudair_detail;
    if (threadIdx.x >= 32 || threadIdx.y != 0 || threadIdx.z != 0) return;
    const int row0 = blockIdx.y * 16, col0 = blockIdx.x * 16;
    if (n <= 0 || (n & 15) != 0 || row0 >= n || col0 >= n) return;

    __shared__ __align__(16) __half sa[MM_STAGES][16][24];  // 48-byte rows
    __shared__ __align__(16) __half sb[MM_STAGES][16][24];

    const int lane = threadIdx.x, g = lane >> 2, t = lane & 3;
    const size_t N = static_cast<size_t>(n);
    const int nk = n / 16;

    // Lane l copies 8 halves (16 bytes) of row l/2 of each A and B slice.
    const int sr = lane >> 1, sc = (lane & 1) * 8;
    const __half *ap = a + (row0 + sr) * N + sc;
    const __half *bp = b + sr * N + col0 + sc;
    auto fetch = [&](int ks) {
        const int slot = ks % MM_STAGES;
        cp_async16(&sa[slot][sr][sc], ap + static_cast<size_t>(ks) * 16);
        cp_async16(&sb[slot][sr][sc], bp + static_cast<size_t>(ks) * 16 * N);
    };
    // Slices 0 .. MM_STAGES-2 go out first, one commit group each (empty
    // groups past the end keep the group count uniform).
#pragma unroll 1
    for (int s = 0; s < MM_STAGES - 1; ++s) {
        if (s < nk) fetch(s);
        cp_async_commit();
    }

    float acc[2][4];
#pragma unroll
    for (int nf = 0; nf < 2; ++nf) {
        const float2 lo = *reinterpret_cast<const float2 *>(c + (row0 + g) * N + col0 + nf * 8 + 2 * t);
        const float2 hi =
            *reinterpret_cast<const float2 *>(c + (row0 + g + 8) * N + col0 + nf * 8 + 2 * t);
        acc[nf][0] = lo.x;
        acc[nf][1] = lo.y;
        acc[nf][2] = hi.x;
        acc[nf][3] = hi.y;
    }

#pragma unroll 1
    for (int ks = 0; ks < nk; ++ks) {
        // Slice ks + MM_STAGES - 1 reuses the slot of slice ks - 1, which the
        // previous iteration finished reading before its closing __syncwarp.
        if (ks + MM_STAGES - 1 < nk) fetch(ks + MM_STAGES - 1);
        cp_async_commit();
        // All but the newest MM_STAGES - 1 groups are complete: slice ks has
        // landed (this lane's copies); the __syncwarp makes every lane's
        // copies visible to the warp.
        cp_async_wait<MM_STAGES - 1>();
        __syncwarp();
        const int slot = ks % MM_STAGES;
        uint32_t fa[4], fb[4];
        ldsm_x4(fa, &sa[slot][lane & 15][(lane >> 4) * 8]);
        ldsm_x4_trans(fb, &sb[slot][lane & 15][(lane >> 4) * 8]);
        mma_16816(acc[0], fa, fb[0], fb[1]);
        mma_16816(acc[1], fa, fb[2], fb[3]);
        __syncwarp();
    }
    cp_async_wait<0>();

#pragma unroll
    for (int nf = 0; nf < 2; ++nf) {
        *reinterpret_cast<float2 *>(c + (row0 + g) * N + col0 + nf * 8 + 2 * t) =
            make_float2(acc[nf][0], acc[nf][1]);
        *reinterpret_cast<float2 *>(c + (row0 + g + 8) * N + col0 + nf * 8 + 2 * t) =
            make_float2(acc[nf][2], acc[nf][3]);
    }
}

// ---- ReduceF32 ----------------------------------------------------------------

// out[2w] = min, out[2w+1] = max of the 32 values of warp w,
// examples/blackwell/blackwell.go:8-17, with Blackwell's float warp
// reductions (redux.sync.{min,max}.f32, sm_100a).  The .NaN form propagates a
// NaN, like Go's math.Min/Max in the reference's check.  Like the reference,
// every launched thread reads one element: the launch covers exactly n.
extern "C" __global__ void ReduceF32(const float *__restrict__ in, float *__restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const float v = in[i];
    float mn, mx;
    asm volatile("redux.sync.min.NaN.f32 %0, %1, 0xffffffff;" : "=f"(mn) : "f"(v));
    asm volatile("redux.sync.max.NaN.f32 %0, %1, 0xffffffff;" : "=f"(mx) : "f"(v));
    if ((threadIdx.x & 31) == 0) {
        out[2 * (i / 32)] = mn;
        out[2 * (i / 32) + 1] = mx;
    }
}
