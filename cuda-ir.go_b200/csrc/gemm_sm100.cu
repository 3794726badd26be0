// gemm_sm100.cu - C = A.B + C with fp16 A (M x K, row-major), fp16 B
// (K x N, row-major), fp32 C (M x N) updated in place, fp32 accumulation:
// the operation of MatMul16 (examples/hopper/hopper.go:194-226) for any
// M, N, K, as a persistent, warp-specialised tcgen05 kernel for sm_100a.
//
// Design (one CTA per SM, 192 threads):
//   warp 0     TMA producer: one thread streams 128x64 A tiles and 64x256 B
//              tiles (four 64x64 boxes) into a 4-stage shared-memory ring with
//              128-byte swizzle, each stage completing on a `full` mbarrier.
//   warp 1     MMA issuer: allocates 512 TMEM columns (two 128x256 fp32
//              accumulators), and one thread issues tcgen05.mma.kind::f16
//              (M=128, N=256, K=16) from shared-memory descriptors: A K-major,
//              B MN-major (B is read as stored; no transpose pass).  Each stage
//              is released with tcgen05.commit on its `empty` mbarrier; a
//              finished accumulator is announced on `acc_full`.
//   warps 2-5  epilogue: each warp owns the 32 TMEM lanes (rows) of its
//              quarter, reads 32 columns at a time with tcgen05.ld, adds C
//              from global memory and stores the sum; the accumulator is handed
//              back on `acc_empty`, so the epilogue of tile i overlaps the
//              mainloop of tile i+1.
// Tiles are visited in groups of 16 row-blocks so the CTAs resident at one
// time share A row-panels and B column-panels in L2.
//
// Every mbarrier wait is bounded (sm100.cuh, mbar_wait): a wait that gives up
// records its site in g_wait_status, raises the CTA's abort flag, and all
// roles unwind; the producer first waits (bounded) for its copies in flight,
// the MMA thread for its MMAs, and TMEM is always freed before exit.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "cudair_internal.h"
#include "sm100.cuh"

namespace cudair {

__device__ unsigned int g_wait_status;

namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int GROUP_M = 16;
constexpr int THREADS = 192;
constexpr uint32_t A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr uint32_t B_BOX_BYTES = 64 * BK * 2;    // 8 KB: 64 n x 64 k
constexpr uint32_t B_STAGE_BYTES = BN * BK * 2;  // 32 KB
constexpr uint32_t STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators
constexpr uint32_t BAR_BYTES = 256;
constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

// Row-block / column-block of persistent tile index t (grouped raster).
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int &m_blk, int &n_blk) {
    const int per_group = GROUP_M * num_n;
    const int group = t / per_group;
    const int first_m = group * GROUP_M;
    const int gsize = min(num_m - first_m, GROUP_M);
    const int r = t - group * per_group;
    m_blk = first_m + r % gsize;
    n_blk = r / gsize;
}

// Bounded wait that ignores the abort flag: used while unwinding.
__device__ __forceinline__ void drain_wait(uint64_t *bar, uint32_t parity, unsigned int *status) {
    int never = 0;
    mbar_wait(bar, parity, &never, status, kSiteDrain);
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_f16f32_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB, float *__restrict__ C, int M,
                       int N, int K, long long ldc, int vec4) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);  // 1024-aligned tiles

    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_STAGE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sB + STAGES * B_STAGE_BYTES);
    uint64_t *full = bars;
    uint64_t *empty = bars + STAGES;
    uint64_t *acc_full = bars + 2 * STAGES;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const uint32_t warp = warp_id(), lane = lane_id();
    const int num_m = (M + BM - 1) / BM;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + BK - 1) / BK;
    unsigned int *status = &g_wait_status;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_map(&tmA);
        tma_prefetch_map(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_normal();
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                int m_blk, n_blk;
                tile_coords(t, num_m, num_n, m_blk, n_blk);
                const int m0 = m_blk * BM, n0 = n_blk * BN;
                // B boxes that start at or beyond column N are not loaded: the
                // accumulator columns they would feed are never stored.
                const int nb = min(BN / 64, (N - n0 + 63) / 64);
                const uint32_t tx = A_STAGE_BYTES + static_cast<uint32_t>(nb) * B_BOX_BYTES;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status,
                                   kSiteProducerEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], tx);
                    const int k0 = kb * BK;
                    tma_load_2d(sA + stage * A_STAGE_BYTES, &tmA, &full[stage], k0, m0, policy);
                    for (int j = 0; j < nb; ++j)
                        tma_load_2d(sB + stage * B_STAGE_BYTES + j * B_BOX_BYTES, &tmB,
                                    &full[stage], n0 + 64 * j, k0, policy);
                    ++issued;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // Let the copies still in flight land before the CTA exits.
                const uint32_t outstanding = issued < STAGES ? issued : STAGES;
                for (uint32_t i = 1; i <= outstanding; ++i) {
                    const uint32_t idx = issued - i;
                    drain_wait(&full[idx % STAGES], (idx / STAGES) & 1u, status);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(BM, BN, false, true);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true, issued_any = false;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, status,
                               kSiteMmaAccEmpty)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, status, kSiteMmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t a_base = smem_u32(sA + stage * A_STAGE_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * B_STAGE_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        // A: K-major rows of 128 B; +32 B per 16-wide k step.
                        const uint64_t a_desc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                        // B: MN-major; 16 k-rows of 128 B per k step, n-blocks 8 KB apart.
                        const uint64_t b_desc =
                            smem_desc_sw128(b_base + kk * 2048, B_BOX_BYTES, 1024);
                        umma_f16_ss(d_tmem, a_desc, b_desc, idesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    issued_any = true;
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit(&acc_full[acc]);
                acc ^= 1u;
                if (acc == 0) acc_phase ^= 1u;
            }
            if (!ok && issued_any) {
                umma_commit(drain);  // completes once every MMA issued above has
                drain_wait(drain, 0, status);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const uint32_t q = warp & 3u;  // the TMEM lane quarter this warp may read
        uint32_t acc = 0, acc_phase = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            int m_blk, n_blk;
            tile_coords(t, num_m, num_n, m_blk, n_blk);
            const int m0 = m_blk * BM, n0 = n_blk * BN;
            if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, status, kSiteEpilogueAccFull))
                break;
            tc_fence_after_sync();
            const int row = m0 + static_cast<int>(q * 32 + lane);
            const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * BN;
            float *crow = C + static_cast<long long>(row) * ldc;
#pragma unroll 1
            for (int ch = 0; ch < BN / 32; ++ch) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_row + ch * 32, r);
                tmem_ld_wait();
                const int col = n0 + ch * 32;
                if (row < M && col < N) {
                    if (vec4) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            if (col + 4 * j < N) {
                                float4 *p = reinterpret_cast<float4 *>(crow + col + 4 * j);
                                float4 v = *p;
                                v.x += __uint_as_float(r[4 * j + 0]);
                                v.y += __uint_as_float(r[4 * j + 1]);
                                v.z += __uint_as_float(r[4 * j + 2]);
                                v.w += __uint_as_float(r[4 * j + 3]);
                                *p = v;
                            }
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col + j < N) crow[col + j] += __uint_as_float(r[j]);
                    }
                }
            }
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
            acc ^= 1u;
            if (acc == 0) acc_phase ^= 1u;
        }
        __syncwarp();
    }

    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// One CTA that waits on a barrier nobody arrives on, with a short limit: the
// bounded wait must give up, record kSiteSelfTest and return.
__global__ void wait_timeout_selftest_kernel(uint64_t limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0)
        mbar_wait(&bar, 0, &abort_flag, &g_wait_status, kSiteSelfTest, limit_ns);
}

}  // namespace gemm

namespace {

struct DeviceInfo {
    int sm_count = 0;
    int major = 0, minor = 0;
    bool attr_set = false;
};

std::mutex g_dev_mu;
DeviceInfo g_dev[64];

int device_info(DeviceInfo **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return set_error(CUDAIR_ERR_INVALID, "cudair: device index %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DeviceInfo &d = g_dev[dev];
    if (d.sm_count == 0) {
        if ((e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return cuda_error(e, "cudaDeviceGetAttribute");
        cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
    }
    if (d.major != 10)
        return set_error(CUDAIR_ERR_UNSUPPORTED,
                         "cudair: device %d has compute capability %d.%d; this build targets sm_100a",
                         dev, d.major, d.minor);
    if (!d.attr_set) {
        e = cudaFuncSetAttribute(gemm::gemm_f16f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(gemm::SMEM_BYTES));
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute");
        d.attr_set = true;
    }
    *out = &d;
    return CUDAIR_OK;
}

}  // namespace

int sm_count_current_device(int *count) {
    DeviceInfo *d = nullptr;
    int rc = device_info(&d);
    if (rc != CUDAIR_OK) return rc;
    *count = d->sm_count;
    return CUDAIR_OK;
}

int gemm_f16f32_launch(const void *a, const void *b, float *c, int64_t M, int64_t N, int64_t K,
                       int64_t lda, int64_t ldb, int64_t ldc, cudaStream_t stream) {
    if (M < 0 || N < 0 || K < 0)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: negative size M=%lld N=%lld K=%lld",
                         (long long)M, (long long)N, (long long)K);
    if (M == 0 || N == 0 || K == 0) return CUDAIR_OK;  // C = C
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: sizes must fit int32");
    if (!a || !b || !c) return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: nil pointer");
    if (lda < K || ldb < N || ldc < N)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm: leading dimensions lda=%lld ldb=%lld ldc=%lld too small",
                         (long long)lda, (long long)ldb, (long long)ldc);
    if (lda % 8 || ldb % 8)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm: lda=%lld and ldb=%lld must be multiples of 8 (16-byte rows)",
                         (long long)lda, (long long)ldb);
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15u)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: A and B must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(c) & 3u)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: C must be 4-byte aligned");

    DeviceInfo *dev = nullptr;
    int rc = device_info(&dev);
    if (rc != CUDAIR_OK) return rc;

    alignas(64) CUtensorMap tmA, tmB;
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
        const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
        const uint32_t box[2] = {64, gemm::BM};
        rc = encode_tiled_internal(&tmA, CUDAIR_TENSOR_MAP_FLOAT16, 2,
                                   reinterpret_cast<uint64_t>(a), dims, strides, box, nullptr,
                                   CUDAIR_INTERLEAVE_NONE, CUDAIR_SWIZZLE_128B,
                                   CUDAIR_L2_PROMOTION_256B, CUDAIR_OOB_FILL_NONE);
        if (rc != CUDAIR_OK) return rc;
    }
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K)};
        const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
        const uint32_t box[2] = {64, gemm::BK};
        rc = encode_tiled_internal(&tmB, CUDAIR_TENSOR_MAP_FLOAT16, 2,
                                   reinterpret_cast<uint64_t>(b), dims, strides, box, nullptr,
                                   CUDAIR_INTERLEAVE_NONE, CUDAIR_SWIZZLE_128B,
                                   CUDAIR_L2_PROMOTION_256B, CUDAIR_OOB_FILL_NONE);
        if (rc != CUDAIR_OK) return rc;
    }

    const int64_t tiles = ((M + gemm::BM - 1) / gemm::BM) * ((N + gemm::BN - 1) / gemm::BN);
    const int grid = static_cast<int>(tiles < dev->sm_count ? tiles : dev->sm_count);
    const int vec4 = ((reinterpret_cast<uintptr_t>(c) & 15u) == 0 && ldc % 4 == 0 && N % 4 == 0) ? 1 : 0;
    gemm::gemm_f16f32_kernel<<<grid, gemm::THREADS, gemm::SMEM_BYTES, stream>>>(
        tmA, tmB, c, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
        static_cast<long long>(ldc), vec4);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "gemm_f16f32_kernel launch");
    return CUDAIR_OK;
}

}  // namespace cudair

using namespace cudair;

CUDAIR_API int cudair_matmul16(const void *a, const void *b, float *c, int32_t n, void *stream) {
    clear_error();
    if (n < 0 || (n & 15) != 0)
        return set_error(CUDAIR_ERR_INVALID, "cudair: MatMul16: n = %d, want a non-negative multiple of 16", n);
    if (n == 0) return CUDAIR_OK;
    if ((reinterpret_cast<uintptr_t>(c) & 15u) != 0)
        return set_error(CUDAIR_ERR_INVALID, "cudair: MatMul16: C must be 16-byte aligned");
    return gemm_f16f32_launch(a, b, c, n, n, n, n, n, n, static_cast<cudaStream_t>(stream));
}

CUDAIR_API int cudair_gemm_f16f32(const void *a, const void *b, float *c, int64_t M, int64_t N,
                                  int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void *stream) {
    clear_error();
    return gemm_f16f32_launch(a, b, c, M, N, K, lda, ldb, ldc, static_cast<cudaStream_t>(stream));
}

CUDAIR_API int cudair_wait_status(uint32_t *status, int clear) {
    clear_error();
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_error(e, "cudaDeviceSynchronize");
    unsigned int v = 0;
    e = cudaMemcpyFromSymbol(&v, g_wait_status, sizeof(v));
    if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyFromSymbol(g_wait_status)");
    if (status) *status = v;
    if (clear && v) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_wait_status, &zero, sizeof(zero));
        if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyToSymbol(g_wait_status)");
    }
    if (v) return set_error(CUDAIR_ERR_TIMEOUT, "cudair: a bounded device wait gave up (status 0x%x)", v);
    return CUDAIR_OK;
}

CUDAIR_API int cudair_wait_timeout_selftest(uint64_t limit_ns, void *stream) {
    clear_error();
    gemm::wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "wait_timeout_selftest launch");
    return CUDAIR_OK;
}
