// gemm_small_sm100.cu - C = A.B + C for small problems (K <= 512), the size of
// the reference's MatMul16 test (n = 64 .. 512), on Blackwell's own
// primitives: one tile of C per CTA, the whole K panel of A and B requested
// by TMA at once, tcgen05.mma into TMEM, and C updated straight from
// registers.
//
// The persistent kernels of gemm_sm100.cu pay for a pipeline (rings, tile
// scheduling, accumulator hand-over, a TMA reduce-add epilogue) that a
// problem of a few tiles cannot amortise.  Here a CTA does one thing once:
//   * thread 0 initialises one mbarrier per 64-wide k-block and issues every
//     k-block's A box (128 x 64) and B box (64 n x 64 k) at once, so the set-up
//     is a single round trip to memory (up to 192 KB of shared memory at
//     K = 512);
//   * warp 1 allocates 64 TMEM columns and issues the MMAs of each k-block as
//     soon as its barrier completes (tcgen05.mma.cta_group::1, M = 128,
//     N = 64, K = 16; A K-major and B MN-major, exactly as stored);
//   * warps 2-5 load their rows of C into registers while the MMAs run, then
//     read the accumulator (tcgen05.ld) and store C + A.B, one rounding per
//     element.
// The result is C + (A.B) with A.B accumulated in fp32, like the other
// tcgen05 kernels.  Every wait is bounded; a wait that gives up records its
// site in the status word, the copies in flight are waited for and TMEM is
// freed before the CTA exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "cudair_internal.h"
#include "sm100.cuh"

namespace cudair {
namespace small {

constexpr int BM = 128;  // rows of C per CTA (the MMA's M)
constexpr int BN = 64;   // columns of C per CTA (the MMA's N)
constexpr int BK = 64;   // k per box: one 128-byte swizzle row of fp16
constexpr int THREADS = 192;
constexpr uint32_t A_BOX = BM * BK * 2;  // 16 KB
constexpr uint32_t B_BOX = BN * BK * 2;  // 8 KB
constexpr uint32_t TMEM_COLS = 64;
constexpr uint32_t BAR_BYTES = 256;

__host__ __device__ constexpr size_t smem_for(int nkb) {
    return 1024 + static_cast<size_t>(nkb) * (A_BOX + B_BOX) + BAR_BYTES;
}
static_assert(smem_for(kSmallMaxKBlocks) <= 227 * 1024, "shared memory budget");
static_assert(8 * (kSmallMaxKBlocks + 2) + 8 <= BAR_BYTES, "barrier area");

__device__ __forceinline__ void drain(uint64_t *bar, unsigned int *status) {
    int never = 0;
    mbar_wait(bar, 0, &never, status, kSiteDrain);
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_small_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      float *__restrict__ C, int M, int N, int K, long long ldc, unsigned int *status) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);  // 1024-aligned boxes

    const int nkb = (K + BK - 1) / BK;  // 1 .. kSmallMaxKBlocks (checked by the launcher)
    uint8_t *sA = smem;
    uint8_t *sB = smem + nkb * A_BOX;
    uint64_t *full = reinterpret_cast<uint64_t *>(sB + nkb * B_BOX);
    uint64_t *done = full + kSmallMaxKBlocks;
    uint64_t *drained = done + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drained + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const uint32_t warp = warp_id(), lane = lane_id();
    const int m0 = static_cast<int>(blockIdx.y) * BM, n0 = static_cast<int>(blockIdx.x) * BN;

    if (threadIdx.x == 0) {
        for (int kb = 0; kb < nkb; ++kb) mbar_init(&full[kb], 1);
        mbar_init(done, 1);
        mbar_init(drained, 1);
        *abort_flag = 0;
        fence_mbar_init();
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
        // ---------------- TMA: the whole K panel at once ----------------
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_normal();
            for (int kb = 0; kb < nkb; ++kb) {
                mbar_arrive_expect_tx(&full[kb], A_BOX + B_BOX);
                tma_load_2d(sA + kb * A_BOX, &tmA, &full[kb], kb * BK, m0, policy);
                tma_load_2d(sB + kb * B_BOX, &tmB, &full[kb], n0, kb * BK, policy);
            }
            // No copy may still be writing this CTA's shared memory when it
            // exits: wait for every box (these waits end at once in a normal
            // run, since the MMAs needed the same boxes).
            for (int kb = 0; kb < nkb; ++kb) drain(&full[kb], status);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_f16_f32(BM, BN, false, true);
            bool ok = true, issued_any = false;
            for (int kb = 0; kb < nkb; ++kb) {
                if (!mbar_wait(&full[kb], 0, abort_flag, status, kSiteMmaFull)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t a_base = smem_u32(sA + kb * A_BOX);
                const uint32_t b_base = smem_u32(sB + kb * B_BOX);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    // A: K-major 128-byte rows, +32 B per 16-wide k step.
                    const uint64_t a_desc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                    // B as stored: MN-major, 16 k rows of 128 B per k step.
                    const uint64_t b_desc = smem_desc_sw128(b_base + kk * 2048, B_BOX, 1024);
                    umma_f16_ss(tmem_base, a_desc, b_desc, idesc, (kb | kk) != 0 ? 1u : 0u);
                }
                issued_any = true;
            }
            if (ok) {
                umma_commit(done);
            } else if (issued_any) {
                umma_commit(drained);  // the MMAs issued so far finish before TMEM is freed
                drain(drained, status);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const uint32_t q = warp & 3u;  // the TMEM lane quarter this warp may read
        const int row = m0 + static_cast<int>(q * 32u + lane);
        float *crow = C + static_cast<long long>(row) * ldc + n0;
        const bool vec = n0 + BN <= N && (ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(C) & 15u) == 0;
        // This thread's 64 elements of C, loaded while the MMAs run.
        float cv[BN];
        if (row < M) {
            if (vec) {
#pragma unroll
                for (int j = 0; j < BN / 4; ++j) {
                    const float4 v = __ldcs(reinterpret_cast<const float4 *>(crow) + j);
                    cv[4 * j] = v.x;
                    cv[4 * j + 1] = v.y;
                    cv[4 * j + 2] = v.z;
                    cv[4 * j + 3] = v.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < BN; ++j) cv[j] = (n0 + j < N) ? crow[j] : 0.f;
            }
        }
        // tcgen05.ld is warp-wide: the warp goes on only if every lane saw the
        // accumulator finished.
        const bool ok = __all_sync(0xffffffffu, mbar_wait(done, 0, abort_flag, status, kSiteEpilogueAccFull));
        if (ok) {
            tc_fence_after_sync();
            const uint32_t t_row = tmem_base + ((q * 32u) << 16);
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(t_row, r0);
            tmem_ld_32x32b_x32(t_row + 32, r1);
            tmem_ld_wait();
            if (row < M) {
                if (vec) {
#pragma unroll
                    for (int j = 0; j < BN / 4; ++j) {
                        const uint32_t *r = (j < 8) ? r0 + 4 * j : r1 + 4 * (j - 8);
                        float4 v;
                        v.x = cv[4 * j] + __uint_as_float(r[0]);
                        v.y = cv[4 * j + 1] + __uint_as_float(r[1]);
                        v.z = cv[4 * j + 2] + __uint_as_float(r[2]);
                        v.w = cv[4 * j + 3] + __uint_as_float(r[3]);
                        __stcs(reinterpret_cast<float4 *>(crow) + j, v);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < BN; ++j)
                        if (n0 + j < N) crow[j] = cv[j] + __uint_as_float(j < 32 ? r0[j] : r1[j - 32]);
                }
            }
        }
    }

    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

}  // namespace small

namespace {
std::mutex g_small_mu;
bool g_small_attr[64];
}  // namespace

int gemm_small_launch(const CUtensorMap &tmA, const CUtensorMap &tmB, float *c, int64_t M, int64_t N,
                      int64_t K, int64_t ldc, unsigned int *status, cudaStream_t stream) {
    const int nkb = static_cast<int>((K + small::BK - 1) / small::BK);
    if (K < 1 || nkb > kSmallMaxKBlocks)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: the small-problem kernel takes 1 <= K <= %d, got %lld",
                         kSmallMaxKBlocks * small::BK, (long long)K);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
    {
        std::lock_guard<std::mutex> lk(g_small_mu);
        if (dev >= 0 && dev < 64 && !g_small_attr[dev]) {
            e = cudaFuncSetAttribute(small::gemm_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(small::smem_for(kSmallMaxKBlocks)));
            if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(small)");
            g_small_attr[dev] = true;
        }
    }
    const dim3 grid(static_cast<unsigned>((N + small::BN - 1) / small::BN),
                    static_cast<unsigned>((M + small::BM - 1) / small::BM), 1);
    small::gemm_small_kernel<<<grid, small::THREADS, small::smem_for(nkb), stream>>>(
        tmA, tmB, c, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), static_cast<long long>(ldc),
        status);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "gemm_small_kernel launch");
    return CUDAIR_OK;
}

}  // namespace cudair
