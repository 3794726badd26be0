// gemm_skinny_sm100.cu - the same C = A.B + C for few rows (M <= 128: the
// decode-shaped GEMM, e.g. M = 16, N = 14336, K = 4096), where the
// square-tile kernels leave most SMs idle and the time is the one pass over
// B (K x N fp16) through HBM.
//
// Design:
//   * swap of operands: D^T (N x M) = B^T . A^T, so the 128-row side of
//     tcgen05.mma (M = 128) runs over N and the small M becomes the MMA's N
//     (mpad = M rounded up to 16).  B is read MN-major exactly as stored, A
//     K-major; the accumulator is 128 TMEM lanes (n) x mpad columns (m).
//   * stream-K: the (n-tile x 64-wide k-block) space is cut into one
//     contiguous range per CTA, one CTA per SM, so every SM streams the same
//     share of B however N and K divide.  A range covers whole n-tiles
//     (written straight into C) and at most two partial ones.
//   * deterministic fix-up: a partial n-tile's contributors store their
//     fp32 partials in a workspace, count themselves on the tile's counter,
//     and the last to arrive adds C and the partials in CTA order (so the sum
//     order, and the result, do not depend on timing), stores C and resets
//     the counter to zero for the next launch.  The last contributor checks
//     the counter first and, when it is last, adds its own part straight from
//     TMEM without storing it.
//   * a TMA ring of 16 KB B tiles (two 64 x 64 boxes) plus mpad x 64 A tiles,
//     as many stages as fit (12 at M <= 16, 7 at M = 128), keeps up to
//     192 KB of B in flight per SM.
//
// Roles as in gemm_sm100.cu (192 threads): warp 0 TMA producer, warp 1 TMEM
// owner and MMA issuer, warps 2-5 epilogue and fix-up.  All waits are
// bounded.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "cudair_internal.h"
#include "sm100.cuh"

namespace cudair {

namespace skinny {

constexpr int BN_T = 128;  // n per tile (the MMA's M)
constexpr int BK = 64;
constexpr int MAX_STAGES = 12;
constexpr int THREADS = 192;
constexpr int MAX_M = 128;
constexpr uint32_t B_BOX_BYTES = 64 * BK * 2;        // 64 n x 64 k
constexpr uint32_t B_STAGE_BYTES = 2 * B_BOX_BYTES;  // 16 KB
constexpr uint32_t BAR_BYTES = 256;
constexpr size_t SMEM_BYTES = 227 * 1024;  // the launch's dynamic shared memory limit

// The ring holds as many stages of (B tile + this M's A tile) as fit: with
// M <= 16 that is 12 stages (192 KB of B in flight per SM), with M = 64 nine,
// with M = 128 seven.
__host__ __device__ constexpr int stages_for(int mpad) {
    return static_cast<int>((SMEM_BYTES - 1024 - BAR_BYTES) / (B_STAGE_BYTES + mpad * BK * 2)) < MAX_STAGES
               ? static_cast<int>((SMEM_BYTES - 1024 - BAR_BYTES) / (B_STAGE_BYTES + mpad * BK * 2))
               : MAX_STAGES;
}
__host__ __device__ constexpr size_t smem_for(int mpad) {
    return 1024 + static_cast<size_t>(stages_for(mpad)) * (B_STAGE_BYTES + mpad * BK * 2) + BAR_BYTES;
}
static_assert(smem_for(16) <= SMEM_BYTES && smem_for(MAX_M) <= SMEM_BYTES, "shared memory budget");
static_assert(2 * MAX_STAGES * 8 + 5 * 8 + 12 <= BAR_BYTES, "barrier area");

// Workspace layout: tile counters first, then two partial slots per CTA.
constexpr size_t COUNTER_BYTES = 256 * 1024;  // 65536 n-tiles
constexpr int MAX_TILES = COUNTER_BYTES / 4;
__device__ __forceinline__ long long range_start(int c, long long T, int G) {
    return (static_cast<long long>(c) * T) / G;
}
// The CTA whose range contains k-block unit x.
__device__ __forceinline__ int cta_of(long long x, long long T, int G) {
    return static_cast<int>(((x + 1) * G - 1) / T);
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA,
                       float *__restrict__ C, int M, int N, int K, long long ldc, int mpad,
                       unsigned int *__restrict__ counters, float *__restrict__ partials,
                       unsigned int *status, int b_early) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

    const uint32_t a_stage_bytes = static_cast<uint32_t>(mpad) * BK * 2;  // multiple of 1024
    const int STAGES = stages_for(mpad);
    uint8_t *sB = smem;
    uint8_t *sA = smem + STAGES * B_STAGE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sA + STAGES * a_stage_bytes);
    uint64_t *full = bars;
    uint64_t *empty = bars + STAGES;
    uint64_t *acc_full = bars + 2 * STAGES;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int *last_flag = abort_flag + 1;

    const uint32_t warp = warp_id(), lane = lane_id();
    const int n_tiles = (N + BN_T - 1) / BN_T;
    const int num_kb = (K + BK - 1) / BK;
    const long long T = static_cast<long long>(n_tiles) * num_kb;
    const int G = static_cast<int>(gridDim.x);
    const int c = static_cast<int>(blockIdx.x);
    const long long r0 = range_start(c, T, G), r1 = range_start(c + 1, T, G);
    const uint32_t tmem_cols = mpad <= 16 ? 32u : (mpad <= 32 ? 64u : (mpad <= 64 ? 128u : 256u));

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_map(&tmA);
        tma_prefetch_map(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    // Every CTA is resident: the next kernel in the stream may be launched
    // (it takes an SM when one of these CTAs exits).
    if (threadIdx.x == 0) grid_launch_dependents();

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const uint64_t policy_b = l2_policy_evict_normal();
            const uint64_t policy_a = l2_policy_evict_last();  // A is re-read by every CTA
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            long long x = r0;
            if (b_early) {
                // B does not depend on the preceding kernel (the caller's
                // promise): the first ring of B boxes is requested before the
                // dependency wait, A and the rest after it.
                const long long pre_end = min(r1, r0 + static_cast<long long>(STAGES));
                for (long long y = r0; y < pre_end; ++y) {
                    const int t = static_cast<int>(y / num_kb), kb = static_cast<int>(y % num_kb);
                    const int n0 = t * BN_T, k0 = kb * BK, s_ = static_cast<int>(y - r0);
                    const int nb = (n0 + 64 < N) ? 2 : 1;
                    mbar_arrive_expect_tx(&full[s_], nb * B_BOX_BYTES + a_stage_bytes);
                    for (int j = 0; j < nb; ++j)
                        tma_load_2d(sB + s_ * B_STAGE_BYTES + j * B_BOX_BYTES, &tmB, &full[s_],
                                    n0 + 64 * j, k0, policy_b);
                }
                grid_dependency_wait();
                for (long long y = r0; y < pre_end; ++y) {
                    const int s_ = static_cast<int>(y - r0);
                    tma_load_2d(sA + s_ * a_stage_bytes, &tmA, &full[s_],
                                static_cast<int>(y % num_kb) * BK, 0, policy_a);
                }
                issued = static_cast<uint32_t>(pre_end - r0);
                stage = issued % static_cast<uint32_t>(STAGES);
                phase = (issued == static_cast<uint32_t>(STAGES)) ? 1u : 0u;
                x = pre_end;
            } else {
                grid_dependency_wait();
            }
            for (; x < r1 && ok; ++x) {
                const int t = static_cast<int>(x / num_kb), kb = static_cast<int>(x % num_kb);
                const int n0 = t * BN_T, k0 = kb * BK;
                const int nb = (n0 + 64 < N) ? 2 : 1;  // skip a box wholly beyond N
                if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status, kSiteProducerEmpty)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[stage], nb * B_BOX_BYTES + a_stage_bytes);
                for (int j = 0; j < nb; ++j)
                    tma_load_2d(sB + stage * B_STAGE_BYTES + j * B_BOX_BYTES, &tmB, &full[stage],
                                n0 + 64 * j, k0, policy_b);
                tma_load_2d(sA + stage * a_stage_bytes, &tmA, &full[stage], k0, 0, policy_a);
                ++issued;
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) {
                const uint32_t outstanding = issued < STAGES ? issued : STAGES;
                for (uint32_t i = 1; i <= outstanding; ++i) {
                    const uint32_t idx = issued - i;
                    int never = 0;
                    mbar_wait(&full[idx % STAGES], (idx / STAGES) & 1u, &never, status, kSiteDrain);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            // The bounded waits below time this launch's own pipeline, not
            // the preceding kernel (A arrives only after that wait anyway).
            grid_dependency_wait();
            const uint32_t idesc = idesc_f16_f32(BN_T, static_cast<uint32_t>(mpad), true, false);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true, issued_any = false;
            long long x = r0;
            while (x < r1 && ok) {
                const int t = static_cast<int>(x / num_kb);
                const long long seg_end = min(r1, static_cast<long long>(t + 1) * num_kb);
                if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, status, kSiteMmaAccEmpty)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t d_tmem = tmem_base + acc * static_cast<uint32_t>(mpad);
                bool first = true;
                for (; x < seg_end; ++x) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, status, kSiteMmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t b_base = smem_u32(sB + stage * B_STAGE_BYTES);
                    const uint32_t a_base = smem_u32(sA + stage * a_stage_bytes);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        // B^T: MN-major, n-blocks 8 KB apart, k groups 1 KB apart.
                        const uint64_t b_desc = smem_desc_sw128(b_base + kk * 2048, B_BOX_BYTES, 1024);
                        // A^T: K-major rows of 128 B (one per m).
                        const uint64_t a_desc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                        umma_f16_ss(d_tmem, b_desc, a_desc, idesc, (first && kk == 0) ? 0u : 1u);
                    }
                    first = false;
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
                umma_commit(drain);
                int never = 0;
                mbar_wait(drain, 0, &never, status, kSiteDrain);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue and fix-up (warps 2..5) ----------------
        grid_dependency_wait();  // C and the workspace may be the preceding kernel's
        const uint32_t q = warp & 3u;
        const int nl = static_cast<int>(q * 32 + lane);  // n within the tile
        const bool leader = (warp == 2 && lane == 0);
        uint32_t acc = 0, acc_phase = 0;
        long long x = r0;
        while (x < r1) {
            const int t = static_cast<int>(x / num_kb);
            const long long tile_lo = static_cast<long long>(t) * num_kb, tile_hi = tile_lo + num_kb;
            const long long seg_end = min(r1, tile_hi);
            const bool whole = (x == tile_lo && seg_end == tile_hi);
            const int slot = (x == r0) ? 0 : 1;  // a partial segment is the range's first or last
            x = seg_end;
            const int n = t * BN_T + nl;
            // The four warps decide together whether to go on (a barrier that
            // ORs every thread's answer: the abort flag may be raised by
            // another role while they read it).
            const bool ok = mbar_wait(&acc_full[acc], acc_phase, abort_flag, status, kSiteEpilogueAccFull);
            if (named_bar_or(1, 128, !ok || *abort_flag != 0)) break;
            tc_fence_after_sync();
            // This thread's column of the accumulator, read from TMEM sixteen
            // rows at a time wherever it is needed; the accumulator is handed
            // back only after the tile is done.
            const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * static_cast<uint32_t>(mpad);
            const int chunks = mpad / 16;
            if (whole) {
                for (int j = 0; j < chunks; ++j) {
                    uint32_t r[16];
                    tmem_ld_32x32b_x16(t_row + 16 * j, r);
                    tmem_ld_wait();
                    if (n < N) {
                        float v[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            v[i] = (16 * j + i < M) ? C[static_cast<long long>(16 * j + i) * ldc + n] : 0.f;
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (16 * j + i < M)
                                C[static_cast<long long>(16 * j + i) * ldc + n] = v[i] + __uint_as_float(r[i]);
                    }
                }
            } else {
                // Partial tile.  Contributors c_lo .. c_hi; the one that
                // finishes last adds C and every contributor's part in CTA
                // order (so the result does not depend on timing) and resets
                // the tile counter.  Each other contributor writes its part to
                // the workspace, makes it visible and counts itself in.  A
                // contributor that finds all the others counted in already is
                // last without writing its part.
                const int c_lo = cta_of(tile_lo, T, G), c_hi = cta_of(tile_hi - 1, T, G);
                const unsigned int others = static_cast<unsigned int>(c_hi - c_lo);
                if (leader) *last_flag = (ld_acquire_gpu_u32(&counters[t]) == others) ? 1 : 0;
                named_bar_sync(1, 128);
                bool last = *last_flag != 0;
                if (!last) {
                    float *part = partials + (static_cast<size_t>(c) * 2 + slot) * BN_T * mpad;
                    for (int j = 0; j < chunks; ++j) {
                        uint32_t r[16];
                        tmem_ld_32x32b_x16(t_row + 16 * j, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i) part[(16 * j + i) * BN_T + nl] = __uint_as_float(r[i]);
                    }
                    __threadfence();
                    named_bar_sync(1, 128);
                    if (leader) {
                        const unsigned int prev = atomicAdd(&counters[t], 1u);
                        *last_flag = (prev == others) ? 1 : 0;
                    }
                    named_bar_sync(1, 128);
                    last = *last_flag != 0;
                }
                if (last) {
                    __threadfence();
                    // Sixteen rows at a time: this CTA's part from TMEM, C and
                    // up to four other contributors' parts loaded together
                    // (one memory latency per four contributors), then added
                    // in contributor order.
                    for (int j = 0; j < chunks; ++j) {
                        if (16 * j >= M) break;
                        uint32_t r[16];
                        tmem_ld_32x32b_x16(t_row + 16 * j, r);
                        tmem_ld_wait();
                        if (n < N) {
                            float v[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                v[i] = (16 * j + i < M) ? C[static_cast<long long>(16 * j + i) * ldc + n] : 0.f;
                            for (int cb = c_lo; cb <= c_hi; cb += 4) {
                                float pv[4][16];
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    const int cc = cb + k;
                                    if (cc > c_hi || cc == c) continue;
                                    const long long s_cc = range_start(cc, T, G);
                                    const int sl = (s_cc / num_kb == t) ? 0 : 1;
                                    const float *pc = partials + (static_cast<size_t>(cc) * 2 + sl) * BN_T * mpad;
#pragma unroll
                                    for (int i = 0; i < 16; ++i)
                                        pv[k][i] = (16 * j + i < M) ? __ldcg(pc + (16 * j + i) * BN_T + nl) : 0.f;
                                }
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    const int cc = cb + k;
                                    if (cc > c_hi) break;
#pragma unroll
                                    for (int i = 0; i < 16; ++i)
                                        v[i] += (cc == c) ? __uint_as_float(r[i]) : pv[k][i];
                                }
                            }
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                if (16 * j + i < M) C[static_cast<long long>(16 * j + i) * ldc + n] = v[i];
                        }
                    }
                    if (leader) counters[t] = 0u;
                }
                named_bar_sync(1, 128);  // last_flag is reused by the next partial tile
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
        tmem_dealloc(tmem_base, tmem_cols);
    }
}

}  // namespace skinny

namespace {

struct Workspace {
    void *ptr = nullptr;
    size_t bytes = 0;
    bool attr_set = false;
};
std::mutex g_ws_mu;
Workspace g_ws[64];

// Tile counters, then two partial slots (128 x M fp32) per CTA for up to 160
// CTAs at M = 128: 21.25 MB.
constexpr size_t kWorkspaceBytes =
    skinny::COUNTER_BYTES + 160u * 2u * skinny::BN_T * skinny::MAX_M * sizeof(float);

// The library's per-device workspace of the skinny kernel (tile counters +
// partial slots), allocated and zeroed on the first call on a device.
int workspace(Workspace **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return set_error(CUDAIR_ERR_INVALID, "cudair: device index %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_ws_mu);
    Workspace &w = g_ws[dev];
    if (!w.ptr) {
        e = cudaMalloc(&w.ptr, kWorkspaceBytes);
        if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(skinny workspace)");
        e = cudaMemset(w.ptr, 0, kWorkspaceBytes);
        if (e != cudaSuccess) return cuda_error(e, "cudaMemset(skinny workspace)");
        // The zeroing runs on the legacy default stream; a launch on a
        // non-blocking stream is not ordered after it, so wait for it here
        // (once per device).
        e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_error(e, "cudaDeviceSynchronize(skinny workspace)");
        w.bytes = kWorkspaceBytes;
    }
    if (!w.attr_set) {
        e = cudaFuncSetAttribute(skinny::gemm_skinny_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(skinny::SMEM_BYTES));
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(skinny)");
        w.attr_set = true;
    }
    *out = &w;
    return CUDAIR_OK;
}

}  // namespace

// Launches the few-row kernel.  pdl > 0 adds programmatic stream
// serialization: the kernel may be launched while the preceding kernel in the
// stream finishes, and waits on it (griddepcontrol.wait) before it reads A, C
// or the workspace; pdl == 2 also lets it request B before that wait.
cudaError_t launch_skinny(int grid, size_t smem, cudaStream_t stream, int pdl, const CUtensorMap &tmB,
                          const CUtensorMap &tmA, float *c, int M, int N, int K, long long ldc, int mpad,
                          unsigned int *counters, float *partials, unsigned int *status) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(skinny::THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl > 0) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, skinny::gemm_skinny_kernel, tmB, tmA, c, M, N, K, ldc, mpad, counters,
                              partials, status, pdl == 2 ? 1 : 0);
}

// Called after a bounded wait gave up: a launch that unwound early may have
// left tile counters raised, so they are zeroed before the next launch.
int skinny_reset_workspace() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CUDAIR_OK;
    std::lock_guard<std::mutex> lk(g_ws_mu);
    if (g_ws[dev].ptr) {
        cudaError_t e = cudaMemset(g_ws[dev].ptr, 0, g_ws[dev].bytes);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_error(e, "cudaMemset(skinny workspace)");
    }
    return CUDAIR_OK;
}

int gemm_skinny_launch(const void *a, const void *b, float *c, int M, int N, int K, int64_t lda,
                       int64_t ldb, int64_t ldc, int sm_count, unsigned int *status,
                       cudaStream_t stream) {
    if (M < 1 || M > skinny::MAX_M)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: the few-row kernel takes 1 <= M <= %d, got %d",
                         skinny::MAX_M, M);
    const int n_tiles = (N + skinny::BN_T - 1) / skinny::BN_T;
    if (n_tiles > skinny::MAX_TILES)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: N = %d too large for the few-row kernel", N);
    Workspace *ws = nullptr;
    int rc = workspace(&ws);
    if (rc != CUDAIR_OK) return rc;
    const int mpad = (M + 15) / 16 * 16;

    alignas(64) CUtensorMap tmB, tmA;
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K)};
        const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
        const uint32_t box[2] = {64, skinny::BK};
        rc = encode_tiled_internal(&tmB, CUDAIR_TENSOR_MAP_FLOAT16, 2, reinterpret_cast<uint64_t>(b),
                                   dims, strides, box, nullptr, CUDAIR_INTERLEAVE_NONE,
                                   CUDAIR_SWIZZLE_128B, CUDAIR_L2_PROMOTION_256B, CUDAIR_OOB_FILL_NONE);
        if (rc != CUDAIR_OK) return rc;
    }
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
        const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
        const uint32_t box[2] = {skinny::BK, static_cast<uint32_t>(mpad)};
        rc = encode_tiled_internal(&tmA, CUDAIR_TENSOR_MAP_FLOAT16, 2, reinterpret_cast<uint64_t>(a),
                                   dims, strides, box, nullptr, CUDAIR_INTERLEAVE_NONE,
                                   CUDAIR_SWIZZLE_128B, CUDAIR_L2_PROMOTION_256B, CUDAIR_OOB_FILL_NONE);
        if (rc != CUDAIR_OK) return rc;
    }
    const long long T = static_cast<long long>(n_tiles) * ((K + skinny::BK - 1) / skinny::BK);
    // One CTA per SM, as many as there are units and as the partial slots hold.
    const long long slots_fit = static_cast<long long>(ws->bytes - skinny::COUNTER_BYTES) /
                                (2LL * skinny::BN_T * mpad * static_cast<long long>(sizeof(float)));
    long long g = T < sm_count ? T : sm_count;
    if (g > slots_fit) g = slots_fit;
    const int grid = static_cast<int>(g);
    unsigned int *counters = static_cast<unsigned int *>(ws->ptr);
    float *partials = reinterpret_cast<float *>(static_cast<uint8_t *>(ws->ptr) + skinny::COUNTER_BYTES);
    cudaError_t e = launch_skinny(grid, skinny::smem_for(mpad), stream, gemm_pdl_mode(), tmB, tmA, c, M, N,
                                  K, static_cast<long long>(ldc), mpad, counters, partials, status);
    if (e != cudaSuccess) return cuda_error(e, "gemm_skinny_kernel launch");
    return CUDAIR_OK;
}

}  // namespace cudair

// =============================================================================
// The same few-row GEMM for callers that cannot allocate device memory.
//
// Some hosts must not allocate device memory themselves: their device memory
// is owned end to end by another allocator (a framework's caching allocator,
// or a pool reserved at start-up), or allocation is forbidden once they are
// serving, because cudaMalloc may synchronise the device and stall every
// other stream.  cudair_gemm_f16f32 allocates the few-row kernel's 21 MB
// workspace on its first call on a device; this entry point instead keeps
// that scratch space in a fixed array that is part of the library's device
// image.  The CUDA runtime reserves the array in a device's memory when it
// loads that image into the device's context.  Under lazy module loading
// (the runtime's default since CUDA 12.2) that happens on first use, which
// for this array is this entry's first call on the device (it looks up the
// array's address), unless another call of the library on that device loaded
// the image before.  So a caller that must not allocate after start-up makes
// one call per device at start-up (or runs with CUDA_MODULE_LOADING=EAGER,
// which loads the image when the context is created); later calls reserve
// nothing.
// =============================================================================

namespace cudair {
namespace {
// Tile counters for up to 4096 n-tiles (N <= 524288), then 4 MiB of partial
// sums: 4 MiB + 16 KiB in all.
constexpr int kNoAllocMaxTiles = 4096;
constexpr int kNoAllocMaxM = 64;
constexpr size_t kNoAllocCounterBytes = kNoAllocMaxTiles * sizeof(unsigned int);
constexpr size_t kNoAllocPartialBytes = 4u << 20;
}  // namespace
}  // namespace cudair

// The scratch array.  It is part of the library's device image, so every GPU
// that loads the library holds it until the process exits.
static __device__ __align__(256) unsigned char
    g_noalloc_scratch[cudair::kNoAllocCounterBytes + cudair::kNoAllocPartialBytes];

namespace cudair {
namespace {

// Host code cannot use g_noalloc_scratch as a pointer: on the host the name
// only stands in for the device variable.  The device address is looked up
// once per device, with that device current, and cached.  It is the address
// in the device's primary context; the entry point runs only there
// (sm_count_current_device refuses any other context first).
std::mutex g_noalloc_mu;
unsigned char *g_noalloc_ptr[64];
bool g_noalloc_attr[64];

int noalloc_scratch(unsigned char **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64)
        return set_error(CUDAIR_ERR_INVALID, "cudair: device index %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
        g_noalloc_ptr[dev] = static_cast<unsigned char *>(p);
    }
    if (!g_noalloc_attr[dev]) {
        e = cudaFuncSetAttribute(skinny::gemm_skinny_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(skinny::SMEM_BYTES));
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(skinny)");
        g_noalloc_attr[dev] = true;
    }
    *out = g_noalloc_ptr[dev];
    return CUDAIR_OK;
}

}  // namespace
}  // namespace cudair

// C (M x N) += A (M x K) . B (K x N) for 1 <= M <= 64 and N <= 524288, with
// the same operands, layout rules and results as cudair_gemm_f16f32 (up to
// fp32 rounding order), without allocating.  The first call on a device looks
// up the scratch array's address (under lazy module loading, this is when the
// runtime loads the image and reserves the array) and sets the kernel's
// shared-memory limit; make that first call at start-up, before any stream
// capture.  Each call clears the tile
// counters it uses (cudaMemsetAsync on `stream`) and then launches; all calls
// share the one array, so calls that overlap on the GPU (e.g. on different
// streams at once) race and must be avoided.  With M > 16 the kernel runs on
// fewer CTAs so that the partial sums fit the array.
CUDAIR_API int cudair_gemm_f16f32_noalloc(const void *a, const void *b, float *c, int64_t M,
                                          int64_t N, int64_t K, int64_t lda, int64_t ldb,
                                          int64_t ldc, void *stream) {
    using namespace cudair;
    clear_error();
    if (M < 0 || N < 0 || K < 0)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm_noalloc: negative size M=%lld N=%lld K=%lld",
                         (long long)M, (long long)N, (long long)K);
    if (M == 0 || N == 0 || K == 0) return CUDAIR_OK;  // C = C
    if (M > kNoAllocMaxM)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm_noalloc: M = %lld exceeds the maximum of %d rows", (long long)M,
                         kNoAllocMaxM);
    if (N > static_cast<int64_t>(kNoAllocMaxTiles) * skinny::BN_T)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm_noalloc: N = %lld exceeds the maximum of %d columns", (long long)N,
                         kNoAllocMaxTiles * skinny::BN_T);
    if (K > INT32_MAX)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm_noalloc: K must fit int32");
    if (!a || !b || !c) return set_error(CUDAIR_ERR_INVALID, "cudair: gemm_noalloc: nil pointer");
    if (lda < K || ldb < N || ldc < N)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm_noalloc: leading dimensions lda=%lld ldb=%lld ldc=%lld too small",
                         (long long)lda, (long long)ldb, (long long)ldc);
    if (lda % 8 || ldb % 8)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm_noalloc: lda=%lld and ldb=%lld must be multiples of 8",
                         (long long)lda, (long long)ldb);
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15u)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm_noalloc: A and B must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(c) & 3u)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm_noalloc: C must be 4-byte aligned");

    int sms = 0;
    int rc = sm_count_current_device(&sms);
    if (rc != CUDAIR_OK) return rc;
    unsigned int *status = nullptr;
    if ((rc = wait_status_current_device(&status)) != CUDAIR_OK) return rc;
    unsigned char *scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch)) != CUDAIR_OK) return rc;

    const int Mi = static_cast<int>(M), Ni = static_cast<int>(N), Ki = static_cast<int>(K);
    const int mpad = (Mi + 15) / 16 * 16;
    alignas(64) CUtensorMap tmB, tmA;
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K)};
        const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
        const uint32_t box[2] = {64, skinny::BK};
        rc = encode_tiled_internal(&tmB, CUDAIR_TENSOR_MAP_FLOAT16, 2, reinterpret_cast<uint64_t>(b),
                                   dims, strides, box, nullptr, CUDAIR_INTERLEAVE_NONE,
                                   CUDAIR_SWIZZLE_128B, CUDAIR_L2_PROMOTION_256B, CUDAIR_OOB_FILL_NONE);
        if (rc != CUDAIR_OK) return rc;
    }
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
        const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
        const uint32_t box[2] = {skinny::BK, static_cast<uint32_t>(mpad)};
        rc = encode_tiled_internal(&tmA, CUDAIR_TENSOR_MAP_FLOAT16, 2, reinterpret_cast<uint64_t>(a),
                                   dims, strides, box, nullptr, CUDAIR_INTERLEAVE_NONE,
                                   CUDAIR_SWIZZLE_128B, CUDAIR_L2_PROMOTION_256B, CUDAIR_OOB_FILL_NONE);
        if (rc != CUDAIR_OK) return rc;
    }
    const int n_tiles = (Ni + skinny::BN_T - 1) / skinny::BN_T;
    const long long T = static_cast<long long>(n_tiles) * ((Ki + skinny::BK - 1) / skinny::BK);
    const long long slot_pair = 2LL * skinny::BN_T * mpad * static_cast<long long>(sizeof(float));
    long long grid = T < sms ? T : sms;
    const long long fit = static_cast<long long>(kNoAllocPartialBytes) / slot_pair;
    if (grid > fit) grid = fit;

    unsigned int *counters = reinterpret_cast<unsigned int *>(scratch);
    float *partials = reinterpret_cast<float *>(scratch + kNoAllocCounterBytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(counters, 0, static_cast<size_t>(n_tiles) * sizeof(unsigned int), s);
    if (e != cudaSuccess) return cuda_error(e, "cudaMemsetAsync(no-alloc tile counters)");
    skinny::gemm_skinny_kernel<<<static_cast<unsigned>(grid), skinny::THREADS, skinny::smem_for(mpad), s>>>(
        tmB, tmA, c, Mi, Ni, Ki, static_cast<long long>(ldc), mpad, counters, partials, status, 0);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "gemm_skinny_kernel launch (no-alloc)");
    return CUDAIR_OK;
}
