// gemm_sm100.cu - C = A.B + C with fp16 A (M x K, row-major), fp16 B
// (K x N, row-major), fp32 C (M x N) updated in place, fp32 accumulation:
// the operation of MatMul16 (examples/hopper/hopper.go:194-226) for any
// M, N, K, as persistent, warp-specialised tcgen05 kernels for sm_100a.
//
// Three variants share the roles, the tile order and the epilogue:
//
//   pair (M > 128): clusters of two CTAs on two SMs compute 256 x 256 tiles
//     with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16).  Each CTA
//     loads its own 128 rows of A and its own 128 columns of B (no
//     multicast), so a CTA moves 32 KB per 64-wide k-block instead of 48 KB;
//     six 32 KB stages fit beside the epilogue's staging boxes.  The even CTA
//     issues the MMAs.
//   pair, wide (M > 128, large K): the same with 256 x 512 tiles (two N = 256
//     MMAs per k-step into one accumulator that fills TMEM; each CTA loads
//     48 KB per k-block for twice the FLOPs, a four-stage ring).  The
//     launcher picks between the two pair tiles with a makespan estimate.
//   single (M <= 128): one CTA per SM computes 128 x 256 tiles with
//     tcgen05.mma.cta_group::1 from a four-stage ring of 48 KB stages.
//
// Roles (192 threads per CTA):
//   warp 0     TMA producer (one thread): A boxes of 128 x 64 and B boxes of
//              64 (n) x 64 (k), 128-byte swizzle, completing on a `full`
//              mbarrier with expect-tx (for a pair, the even CTA's barrier
//              counts both CTAs' bytes).
//   warp 1     TMEM owner (512 columns: two 256-column fp32 accumulators) and
//              MMA issuer (one thread).  A is read K-major, B MN-major exactly
//              as stored; tcgen05.commit releases each stage on `empty` and
//              announces a finished accumulator on `acc_full` (multicast to
//              both CTAs of a pair).
//   warps 2-5  epilogue: warp w owns TMEM lanes 32 (w mod 4) .. +31 (one row
//              per thread), reads 32 columns at a time with tcgen05.ld,
//              stages them as a 32 x 32 box in shared memory and hands the
//              box to a TMA reduce-add, so L2 adds it into C (C is never
//              loaded into the SM); the accumulator is handed back on
//              `acc_empty` (for a pair, the even CTA's, counting the eight
//              epilogue warps of both CTAs) as soon as it is read, so tile
//              i's epilogue overlaps tile i+1's mainloop.
// Tiles are visited in groups of row-blocks so that the CTAs resident at one
// time share A row-panels and B column-panels in L2.
//
// Every mbarrier wait is bounded (sm100.cuh, mbar_wait): a wait that gives up
// records its site in g_wait_status and raises the abort flag (of both CTAs
// of a pair); all roles unwind, in-flight copies and MMAs are waited for
// (with limits), and TMEM is always freed before exit.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include <cuda_fp16.h>

#include "cudair_internal.h"
#include "sm100.cuh"

namespace cudair {

__device__ unsigned int g_wait_status;

namespace gemm {

constexpr int BN = 256;  // N per tile (and per MMA)
constexpr int BK = 64;   // K per stage: one 128-byte swizzle row of fp16
constexpr int THREADS = 192;
constexpr uint32_t A_BOX_BYTES = 128 * BK * 2;  // 16 KB: 128 rows x 64 k
constexpr uint32_t B_BOX_BYTES = 64 * BK * 2;   // 8 KB: 64 n x 64 k
constexpr uint32_t TMEM_COLS = 2 * BN;           // two accumulators
constexpr uint32_t BAR_BYTES = 256;
// Epilogue staging: two 32 x 32 fp32 boxes per epilogue warp.
constexpr uint32_t EPI_BOX_BYTES = 32 * 32 * 4;
constexpr uint32_t EPI_BYTES = 4 * 2 * EPI_BOX_BYTES;  // 32 KB

// single-CTA variant
constexpr int S_BM = 128;
constexpr int S_STAGES = 4;
constexpr int S_GROUP_M = 16;
constexpr uint32_t S_STAGE_B = BN / 64 * B_BOX_BYTES;  // 32 KB
constexpr size_t S_SMEM = 1024 + S_STAGES * (A_BOX_BYTES + S_STAGE_B) + EPI_BYTES + BAR_BYTES;

// CTA-pair variants: NB 256-column MMA blocks per tile (NB = 1: 256 x 256
// tiles, two accumulators; NB = 2: 256 x 512 tiles, one accumulator filling
// TMEM, a quarter fewer operand bytes per FLOP).
constexpr int P_BM = 256;  // rows per pair tile, 128 per CTA
#ifndef CUDAIR_P_GROUP_M
#define CUDAIR_P_GROUP_M 8
#endif
constexpr int P_GROUP_M = CUDAIR_P_GROUP_M;
template <int NB>
struct PairCfg {
    static constexpr int TILE_N = 256 * NB;
    static constexpr uint32_t STAGE_B = NB * 2 * B_BOX_BYTES;  // this CTA's 128 x NB columns
    static constexpr uint32_t STAGE = A_BOX_BYTES + STAGE_B;
    static constexpr int STAGES_FIT = static_cast<int>((227 * 1024 - 1024 - EPI_BYTES - BAR_BYTES) / STAGE);
    static constexpr int STAGES = STAGES_FIT < 7 ? STAGES_FIT : 7;
    static constexpr int ACCS = 2 / NB;  // accumulator buffers in 512 TMEM columns
    static constexpr size_t SMEM = 1024 + STAGES * STAGE + EPI_BYTES + BAR_BYTES;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

static_assert(S_SMEM <= 227 * 1024, "shared memory budget");

// Row-block / column-block of persistent tile index t: groups of group_m
// row-blocks, visited column by column, with the column order reversed in
// every other group (so a group starts on the B column-panels the previous
// one ended on, still in L2: ~0.6 % faster than one direction at 8192^3).
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int group_m, int &m_blk,
                                            int &n_blk) {
    const int per_group = group_m * num_n;
    const int group = t / per_group;
    const int first_m = group * group_m;
    const int gsize = min(num_m - first_m, group_m);
    const int r = t - group * per_group;
    m_blk = first_m + r % gsize;
    n_blk = r / gsize;
    if (group & 1) n_blk = num_n - 1 - n_blk;
}

// Bounded wait that ignores the abort flag: used while unwinding.
__device__ __forceinline__ void drain_wait(uint64_t *bar, uint32_t parity, unsigned int *status) {
    int never = 0;
    mbar_wait(bar, parity, &never, status, kSiteDrain);
}

// C is read once and written once per launch, inside L2 by the reduce-add
// (or by the scalar path's loads and stores): marked first to leave L2, so the
// stream of C does not push out the A and B panels that other tiles re-read.
__device__ __forceinline__ uint64_t c_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// How the epilogue writes the accumulator into C.
enum Epilogue : int {
    kEpiScalarAdd = 0,  // C += acc, fp32, element by element (C not 16-byte aligned)
    kEpiReduceF32 = 1,  // C += acc, fp32, TMA reduce-add in L2
    kEpiStoreF32 = 2,   // C = acc, fp32, TMA store
    kEpiStoreF16 = 3,   // C = acc rounded to fp16, TMA store
};

// Writes this warp's 32 accumulator rows (TMEM lanes from t_row, 256 columns)
// into C through TMA.  Each chunk goes TMEM -> registers -> a 4 KB staging box
// in shared memory (the 128-byte swizzled layout of tmC, so the
// row-per-thread stores are free of bank conflicts) -> one bulk tensor copy:
//   kEpiReduceF32: 32 x 32 fp32 boxes through cp.reduce.async.bulk.tensor, so
//     L2 adds the box into C: C never enters the SM, and each element of C
//     gets exactly one add, C + (A.B), rounded once;
//   kEpiStoreF32: the same boxes stored (C = A.B);
//   kEpiStoreF16: 32 x 64 boxes rounded to fp16 (round to nearest) and stored.
// Rows and columns outside C are clipped by the tensor map.  The warp's two
// boxes alternate (`buf` carries over between calls); lane 0 issues and
// tracks the bulk groups, and a box is rewritten only after the copy that
// last read it has finished reading.
__device__ __forceinline__ void epilogue_rows_tma(uint32_t t_row, const CUtensorMap *tmC,
                                                  uint32_t boxes, int row0, int n0, int N,
                                                  uint64_t pol, uint32_t &buf, int epi) {
    const uint32_t lane = lane_id();
    const int width = (epi == kEpiStoreF16) ? 64 : 32;  // columns per box
#pragma unroll 1
    for (int col0 = 0; col0 < BN; col0 += width) {
        const int col = n0 + col0;
        if (col >= N) break;  // the rest of the block lies beyond C
        uint32_t r[32], r2[32];
        tmem_ld_32x32b_x32(t_row + col0, r);
        if (epi == kEpiStoreF16) tmem_ld_32x32b_x32(t_row + col0 + 32, r2);
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        tmem_ld_wait();
        const uint32_t box = boxes + buf * EPI_BOX_BYTES;
        const uint32_t row_addr = box + lane * 128u;
        if (epi == kEpiStoreF16) {
            uint32_t h[32];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const __half2 lo = __floats2half2_rn(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
                const __half2 hi = __floats2half2_rn(__uint_as_float(r2[2 * k]), __uint_as_float(r2[2 * k + 1]));
                h[k] = *reinterpret_cast<const uint32_t *>(&lo);
                h[16 + k] = *reinterpret_cast<const uint32_t *>(&hi);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
                st_shared_v4(row_addr + ((static_cast<uint32_t>(j) ^ (lane & 7u)) << 4), h[4 * j],
                             h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                st_shared_v4(row_addr + ((static_cast<uint32_t>(j) ^ (lane & 7u)) << 4), r[4 * j],
                             r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            if (epi == kEpiReduceF32)
                tma_reduce_add_2d(tmC, box, col, row0, pol);
            else
                tma_store_2d(tmC, box, col, row0, pol);
            bulk_commit_group();
        }
        buf ^= 1u;
    }
}

// Same, for C whose rows are not 16-byte aligned: scalar accesses.
__device__ __forceinline__ void epilogue_rows_scalar(uint32_t t_row, float *crow, int row, int n0,
                                                     int M, int N) {
#pragma unroll 1
    for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + ch * 32, r);
        tmem_ld_wait();
        const int col = n0 + ch * 32;
        if (row < M) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col + j < N) crow[col + j] += __uint_as_float(r[j]);
        }
    }
}

// =============================================================================
// Single-CTA variant: 128 x 256 tiles.  BT: B is stored transposed (N x K,
// K-major) instead of K x N.  idesc: the MMA's instruction descriptor (fp16
// or bf16 operands); epi: an Epilogue mode.
// =============================================================================
template <bool BT>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_f16f32_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmC, float *__restrict__ C, int M,
                       int N, int K, long long ldc, uint32_t idesc, int epi) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);  // 1024-aligned tiles

    uint8_t *sA = smem;
    uint8_t *sB = smem + S_STAGES * A_BOX_BYTES;
    uint8_t *sEpi = sB + S_STAGES * S_STAGE_B;  // 1024-aligned staging boxes
    uint64_t *bars = reinterpret_cast<uint64_t *>(sEpi + EPI_BYTES);
    uint64_t *full = bars;
    uint64_t *empty = bars + S_STAGES;
    uint64_t *acc_full = bars + 2 * S_STAGES;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const uint32_t warp = warp_id(), lane = lane_id();
    const int num_m = (M + S_BM - 1) / S_BM;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + BK - 1) / BK;
    unsigned int *status = &g_wait_status;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S_STAGES; ++s) {
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
        if (epi != kEpiScalarAdd) tma_prefetch_map(&tmC);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    // Programmatic dependent launch (cudair_set_gemm_pdl): every CTA is set
    // up, so the next kernel in the stream may be launched; this one waits
    // for the preceding kernel before it reads A, B or C (no-ops without the
    // launch attribute).
    if (threadIdx.x == 0) grid_launch_dependents();

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            grid_dependency_wait();
            const uint64_t policy = l2_policy_evict_normal();
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                int m_blk, n_blk;
                tile_coords(t, num_m, num_n, S_GROUP_M, m_blk, n_blk);
                const int m0 = m_blk * S_BM, n0 = n_blk * BN;
                // B boxes that start at or beyond column N are not loaded: the
                // accumulator columns they would feed are never stored.
                const int nb = min(BN / 64, (N - n0 + 63) / 64);
                const uint32_t tx = A_BOX_BYTES + static_cast<uint32_t>(nb) * B_BOX_BYTES;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status,
                                   kSiteProducerEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], tx);
                    const int k0 = kb * BK;
                    tma_load_2d(sA + stage * A_BOX_BYTES, &tmA, &full[stage], k0, m0, policy);
                    // 64-column B boxes: (n, k) for B as stored, (k, n) for B^T.
                    for (int j = 0; j < nb; ++j)
                        tma_load_2d(sB + stage * S_STAGE_B + j * B_BOX_BYTES, &tmB, &full[stage],
                                    BT ? k0 : n0 + 64 * j, BT ? n0 + 64 * j : k0, policy);
                    ++issued;
                    if (++stage == S_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // Let the copies still in flight land before the CTA exits.
                const uint32_t outstanding = issued < S_STAGES ? issued : S_STAGES;
                for (uint32_t i = 1; i <= outstanding; ++i) {
                    const uint32_t idx = issued - i;
                    drain_wait(&full[idx % S_STAGES], (idx / S_STAGES) & 1u, status);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            // The bounded waits below time this launch's own pipeline, not
            // the preceding kernel (operands arrive only after that wait).
            grid_dependency_wait();
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
                    const uint32_t a_base = smem_u32(sA + stage * A_BOX_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * S_STAGE_B);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        // A: K-major rows of 128 B; +32 B per 16-wide k step.
                        const uint64_t a_desc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                        // B as stored: MN-major, 16 k-rows of 128 B per k step, n-blocks
                        // 8 KB apart.  B^T: K-major like A.
                        const uint64_t b_desc =
                            BT ? smem_desc_sw128(b_base + kk * 32, 16, 1024)
                               : smem_desc_sw128(b_base + kk * 2048, B_BOX_BYTES, 1024);
                        umma_f16_ss(d_tmem, a_desc, b_desc, idesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    issued_any = true;
                    umma_commit(&empty[stage]);
                    if (++stage == S_STAGES) {
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
        grid_dependency_wait();  // C may be the preceding kernel's
        const uint32_t q = warp & 3u;  // the TMEM lane quarter this warp may read
        const uint64_t cpol = c_policy();
        const uint32_t boxes = smem_u32(sEpi) + q * 2 * EPI_BOX_BYTES;
        uint32_t acc = 0, acc_phase = 0, buf = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            int m_blk, n_blk;
            tile_coords(t, num_m, num_n, S_GROUP_M, m_blk, n_blk);
            const int m0 = m_blk * S_BM, n0 = n_blk * BN;
            const int row0 = m0 + static_cast<int>(q * 32);
            if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, status, kSiteEpilogueAccFull))
                break;
            tc_fence_after_sync();
            const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * BN;
            if (epi != kEpiScalarAdd) {
                if (row0 < M) epilogue_rows_tma(t_row, &tmC, boxes, row0, n0, N, cpol, buf, epi);
            } else {
                const int row = row0 + static_cast<int>(lane);
                epilogue_rows_scalar(t_row, C + static_cast<long long>(row) * ldc, row, n0, M, N);
            }
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
            acc ^= 1u;
            if (acc == 0) acc_phase ^= 1u;
        }
        // The reduces still in flight read this CTA's shared memory: they
        // finish before the CTA exits.
        if (lane == 0) bulk_wait_group<0>();
        __syncwarp();
    }

    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// =============================================================================
// CTA-pair variants: clusters of 2, 256 x (256 NB) tiles, cta_group::2.
// =============================================================================
template <int NB, bool BT>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_f16f32_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                            const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmC, float *__restrict__ C, int M,
                            int N, int K, long long ldc, uint32_t idesc, int epi) {
    using Cfg = PairCfg<NB>;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);  // same offset in both CTAs

    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_BOX_BYTES;
    uint8_t *sEpi = sB + STAGES * Cfg::STAGE_B;  // 1024-aligned staging boxes
    uint64_t *bars = reinterpret_cast<uint64_t *>(sEpi + EPI_BYTES);
    uint64_t *full = bars;                     // used in the even CTA only
    uint64_t *empty = bars + STAGES;           // both CTAs
    uint64_t *acc_full = bars + 2 * STAGES;    // both CTAs
    uint64_t *acc_empty = acc_full + 2;        // even CTA only
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const uint32_t warp = warp_id(), lane = lane_id();
    const uint32_t rank = cluster_ctarank();  // 0 = even CTA (issues the MMAs)
    const uint32_t peer = rank ^ 1u;
    const int cluster = static_cast<int>(blockIdx.x >> 1);
    const int num_clusters = static_cast<int>(gridDim.x >> 1);
    const int num_m = (M + P_BM - 1) / P_BM;
    const int num_n = (N + Cfg::TILE_N - 1) / Cfg::TILE_N;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + BK - 1) / BK;
    unsigned int *status = &g_wait_status;
    const uint32_t peer_abort = mapa_shared(smem_u32(const_cast<int *>(abort_flag)), peer);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 8);  // the epilogue warps of both CTAs
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_map(&tmA);
        tma_prefetch_map(&tmB);
        if (epi != kEpiScalarAdd) tma_prefetch_map(&tmC);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before_sync();
    cluster_sync();  // barriers of both CTAs initialised before any remote arrive
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;
    // Programmatic dependent launch: as in the single-CTA kernel.
    if (threadIdx.x == 0) grid_launch_dependents();

    // A wait that gave up here also stops the peer CTA.
    auto give_up = [&]() { st_shared_cluster_u32(peer_abort, 1u); };
    // 64-column B boxes that start inside the tensor, among the 128 columns from n.
    auto boxes = [&](int n) { return max(0, min(2, (N - n + 63) / 64)); };

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            grid_dependency_wait();
            const uint64_t policy = l2_policy_evict_normal();
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            for (int t = cluster; t < num_tiles && ok; t += num_clusters) {
                int m_blk, n_blk;
                tile_coords(t, num_m, num_n, P_GROUP_M, m_blk, n_blk);
                const int m_pair = m_blk * P_BM, n_pair = n_blk * Cfg::TILE_N;
                // Block h of this CTA holds columns n_pair + 256 h + 128 rank + [0, 128):
                // MMA h takes its first 128 columns from the even CTA, the next 128
                // from the odd one.  Boxes and rows entirely outside the tensor are
                // not loaded (their accumulator rows / columns are never stored).
                const int m_mine = m_pair + 128 * static_cast<int>(rank);
                const int a_mine = (m_mine < M) ? 1 : 0;
                const int a_odd = (m_pair + 128 < M) ? 1 : 0;
                uint32_t tx = static_cast<uint32_t>(1 + a_odd) * A_BOX_BYTES;
                for (int h = 0; h < NB; ++h)
                    tx += static_cast<uint32_t>(boxes(n_pair + 256 * h) + boxes(n_pair + 256 * h + 128)) *
                          B_BOX_BYTES;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status,
                                   kSiteProducerEmpty)) {
                        give_up();
                        ok = false;
                        break;
                    }
                    const uint32_t full_even = mapa_shared(smem_u32(&full[stage]), 0);
                    if (rank == 0) mbar_arrive_expect_tx(&full[stage], tx);
                    const int k0 = kb * BK;
                    if (a_mine)
                        tma_load_2d_pair(sA + stage * A_BOX_BYTES, &tmA, full_even, k0, m_mine,
                                         policy);
#pragma unroll
                    for (int h = 0; h < NB; ++h) {
                        const int n_mine = n_pair + 256 * h + 128 * static_cast<int>(rank);
                        const int nb_mine = boxes(n_mine);
                        // 64-column B boxes: (n, k) for B as stored, (k, n) for B^T.
                        for (int j = 0; j < nb_mine; ++j)
                            tma_load_2d_pair(sB + stage * Cfg::STAGE_B + (2 * h + j) * B_BOX_BYTES,
                                             &tmB, full_even, BT ? k0 : n_mine + 64 * j,
                                             BT ? n_mine + 64 * j : k0, policy);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // This CTA's copies complete on the even CTA's barriers, which
                // only that CTA can wait on: give them time to land.
                spin_ns(2000000);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (even CTA) ----------------
        if (lane == 0 && rank == 0) {
            grid_dependency_wait();  // as in the single-CTA kernel
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true, issued_any = false;
            // The MMAs of k-block kb (held in stage st) into the 256-column
            // blocks [h_lo, h_hi) of accumulator acc.
            auto issue = [&](uint32_t st, int kb, int h_lo, int h_hi) {
                const uint32_t a_base = smem_u32(sA + st * A_BOX_BYTES);
                const uint32_t b_base = smem_u32(sB + st * Cfg::STAGE_B);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t a_desc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                    for (int h = h_lo; h < h_hi; ++h) {
                        const uint32_t b_blk = b_base + h * 2 * B_BOX_BYTES;
                        const uint64_t b_desc =
                            BT ? smem_desc_sw128(b_blk + kk * 32, 16, 1024)
                               : smem_desc_sw128(b_blk + kk * 2048, B_BOX_BYTES, 1024);
                        umma_f16_ss_pair(tmem_base + acc * 256 + h * 256, a_desc, b_desc, idesc,
                                         (kb | kk) != 0 ? 1u : 0u);
                    }
                }
                issued_any = true;
            };
            // k-blocks [lo, hi) of one tile, both halves, releasing each stage.
            auto plain = [&](int lo, int hi) -> bool {
                for (int kb = lo; kb < hi; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, status, kSiteMmaFull)) return false;
                    tc_fence_after_sync();
                    issue(stage, kb, 0, NB);
                    umma_commit_pair_multicast(&empty[stage], 0x3);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                return true;
            };
            // 256 x 512 tiles: one accumulator fills TMEM, so its epilogue
            // cannot overlap the next tile's mainloop; its two 256-column
            // halves are handed over separately instead.  In the first and
            // the last ring-full of k-blocks of a tile (a "window", the k-blocks
            // all resident at once), half 0 is multiplied for every k-block
            // before half 1.  So the tile's half 0 is finished, and its
            // epilogue starts, while half 1's last MMAs run; and the next tile
            // starts on half 0 while half 1 is still being drained.
            auto window = [&](int lo, int hi, bool first, bool last) -> bool {
                const uint32_t st0 = stage;
                if (first) {
                    if (!mbar_wait(&acc_empty[0], acc_phase ^ 1u, abort_flag, status, kSiteMmaAccEmpty))
                        return false;
                    tc_fence_after_sync();
                }
                for (int kb = lo; kb < hi; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, status, kSiteMmaFull)) return false;
                    tc_fence_after_sync();
                    issue(stage, kb, 0, 1);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (last) umma_commit_pair_multicast(&acc_full[0], 0x3);
                if (first) {
                    if (!mbar_wait(&acc_empty[1], acc_phase ^ 1u, abort_flag, status, kSiteMmaAccEmpty))
                        return false;
                    tc_fence_after_sync();
                }
                uint32_t st = st0;
                for (int kb = lo; kb < hi; ++kb) {
                    issue(st, kb, 1, 2);
                    umma_commit_pair_multicast(&empty[st], 0x3);
                    if (++st == STAGES) st = 0;
                }
                if (last) umma_commit_pair_multicast(&acc_full[1], 0x3);
                return true;
            };
            for (int t = cluster; t < num_tiles && ok; t += num_clusters) {
                if (NB == 2) {
                    const int head_end = min(STAGES, num_kb);
                    const int tail_lo = max(head_end, num_kb - STAGES);
                    ok = window(0, head_end, true, head_end == num_kb) && plain(head_end, tail_lo) &&
                         (tail_lo == num_kb || window(tail_lo, num_kb, false, true));
                    if (!ok) {
                        give_up();
                        break;
                    }
                    acc_phase ^= 1u;
                } else {
                    if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, status,
                                   kSiteMmaAccEmpty)) {
                        give_up();
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    if (!plain(0, num_kb)) {
                        give_up();
                        ok = false;
                        break;
                    }
                    umma_commit_pair_multicast(&acc_full[acc], 0x3);
                    acc ^= 1u;
                    if (acc == 0) acc_phase ^= 1u;
                }
            }
            if (!ok && issued_any) {
                umma_commit_pair_local(drain);
                drain_wait(drain, 0, status);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 2..5, both CTAs) ----------------
        grid_dependency_wait();  // C may be the preceding kernel's
        const uint32_t q = warp & 3u;
        const uint64_t cpol = c_policy();
        const uint32_t boxes = smem_u32(sEpi) + q * 2 * EPI_BOX_BYTES;
        uint32_t acc = 0, acc_phase = 0, buf = 0;
        for (int t = cluster; t < num_tiles; t += num_clusters) {
            int m_blk, n_blk;
            tile_coords(t, num_m, num_n, P_GROUP_M, m_blk, n_blk);
            const int m0 = m_blk * P_BM + 128 * static_cast<int>(rank), n0 = n_blk * Cfg::TILE_N;
            const int row0 = m0 + static_cast<int>(q * 32);
            // 256 x 256 tiles: accumulator `acc` (of two) in one piece.  256 x
            // 512 tiles: the one accumulator's two halves, each announced on
            // its own acc_full and handed back on its own acc_empty.
            bool aborted = false;
#pragma unroll 1
            for (int h = 0; h < NB; ++h) {
                const uint32_t bar = (NB == 2) ? static_cast<uint32_t>(h) : acc;
                if (!mbar_wait(&acc_full[bar], acc_phase, abort_flag, status, kSiteEpilogueAccFull)) {
                    give_up();
                    aborted = true;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * 256 + 256 * h;
                if (epi != kEpiScalarAdd) {
                    if (row0 < M)
                        epilogue_rows_tma(t_row, &tmC, boxes, row0, n0 + 256 * h, N, cpol, buf, epi);
                } else {
                    const int row = row0 + static_cast<int>(lane);
                    epilogue_rows_scalar(t_row, C + static_cast<long long>(row) * ldc, row, n0 + 256 * h,
                                         M, N);
                }
                tc_fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[bar]), 0));
            }
            if (aborted) break;
            if (Cfg::ACCS == 2) acc ^= 1u;
            if (acc == 0) acc_phase ^= 1u;
        }
        if (lane == 0) bulk_wait_group<0>();  // reduces in flight read this CTA's boxes
        __syncwarp();
    }

    // Neither CTA leaves (or frees TMEM) while the other may still touch its
    // shared memory or TMEM: remote arrivals, peer copies and MMAs all precede
    // this barrier.
    tc_fence_before_sync();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
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
    int max_pairs = 0;  // CTA pairs resident at once
    unsigned int *status = nullptr;  // device address of g_wait_status
    CUcontext primary = nullptr;     // the device's primary context (retained)
    bool attr_set = false;
};

std::mutex g_dev_mu;
DeviceInfo g_dev[64];
std::atomic<int> g_variant{0};  // 0 auto, 1 single CTA, 2 CTA pair, ... (cudair_set_gemm_variant)
std::atomic<int> g_pdl{0};      // 0 plain launch, 1 PDL, 2 PDL with B early (few-row kernel)

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
    // sm_100a code (tcgen05, the arch-specific features) runs on compute
    // capability 10.0 only, not on later 10.x parts.
    if (d.major != 10 || d.minor != 0)
        return set_error(CUDAIR_ERR_UNSUPPORTED,
                         "cudair: device %d has compute capability %d.%d; this build targets sm_100a (10.0)",
                         dev, d.major, d.minor);
    // The library's per-device state (the addresses of its __device__
    // variables, workspaces, streams, events) belongs to one context per
    // device: the primary context, which the runtime and gocudrv use.  A call
    // made with another context current is refused instead of handing its
    // kernels addresses from the primary context.
    const Driver *drv = nullptr;
    int rc = load_driver(&drv);
    if (rc != CUDAIR_OK) return rc;
    if ((rc = ensure_context()) != CUDAIR_OK) return rc;
    if (!d.primary) {
        CUresult r = drv->cuDevicePrimaryCtxRetain(&d.primary, static_cast<CUdevice>(dev));
        if (r != CUDA_SUCCESS) return cu_error(r, "cuDevicePrimaryCtxRetain");
    }
    CUcontext cur = nullptr;
    CUresult r = drv->cuCtxGetCurrent(&cur);
    if (r != CUDA_SUCCESS) return cu_error(r, "cuCtxGetCurrent");
    if (cur != d.primary)
        return set_error(CUDAIR_ERR_UNSUPPORTED,
                         "cudair: the current context is not device %d's primary context; the library "
                         "runs in the primary context only (the one the CUDA runtime and gocudrv use)",
                         dev);
    if (!d.attr_set) {
        const struct {
            const void *fn;
            size_t smem;
        } kernels[] = {
            {reinterpret_cast<const void *>(gemm::gemm_f16f32_kernel<false>), gemm::S_SMEM},
            {reinterpret_cast<const void *>(gemm::gemm_f16f32_kernel<true>), gemm::S_SMEM},
            {reinterpret_cast<const void *>(gemm::gemm_f16f32_pair_kernel<1, false>), gemm::PairCfg<1>::SMEM},
            {reinterpret_cast<const void *>(gemm::gemm_f16f32_pair_kernel<1, true>), gemm::PairCfg<1>::SMEM},
            {reinterpret_cast<const void *>(gemm::gemm_f16f32_pair_kernel<2, false>), gemm::PairCfg<2>::SMEM},
            {reinterpret_cast<const void *>(gemm::gemm_f16f32_pair_kernel<2, true>), gemm::PairCfg<2>::SMEM},
        };
        for (const auto &k : kernels) {
            e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(k.smem));
            if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(gemm)");
        }
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(2 * (d.sm_count / 2), 1, 1);
        cfg.blockDim = dim3(gemm::THREADS, 1, 1);
        cfg.dynamicSmemBytes = gemm::PairCfg<1>::SMEM;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        e = cudaOccupancyMaxActiveClusters(&clusters, gemm::gemm_f16f32_pair_kernel<1, false>, &cfg);
        if (e != cudaSuccess) return cuda_error(e, "cudaOccupancyMaxActiveClusters");
        d.max_pairs = clusters;
        void *sym = nullptr;
        e = cudaGetSymbolAddress(&sym, g_wait_status);
        if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_wait_status)");
        d.status = static_cast<unsigned int *>(sym);
        d.attr_set = true;
    }
    *out = &d;
    return CUDAIR_OK;
}

}  // namespace

int gemm_pdl_mode() { return g_pdl.load(); }

int wait_status_current_device(unsigned int **status) {
    DeviceInfo *d = nullptr;
    int rc = device_info(&d);
    if (rc != CUDAIR_OK) return rc;
    *status = d->status;
    return CUDAIR_OK;
}

int sm_count_current_device(int *count) {
    DeviceInfo *d = nullptr;
    int rc = device_info(&d);
    if (rc != CUDAIR_OK) return rc;
    *count = d->sm_count;
    return CUDAIR_OK;
}

namespace gemm {
// The CTA-pair tile for a shape: 256 x 512 tiles (2) move a quarter fewer
// operand bytes per FLOP, but their accumulator fills TMEM, so each tile's
// epilogue is not overlapped, and they come in half as many tiles.  The choice
// compares the estimated makespan, persistent waves x time per tile, with
// per-tile times fitted on B200 (microseconds, K in elements):
//   256 x 256: 0.00703 K + 3.4     256 x 512: 0.0124 K + 11.6
// (8192^3: 14 waves x 61.0 us against 7 x 113.2 us).
int auto_pair_nb(int64_t M, int64_t N, int64_t K, int pairs) {
    const int64_t mt = (M + P_BM - 1) / P_BM;
    const int64_t w1 = (mt * ((N + 255) / 256) + pairs - 1) / pairs;
    const int64_t w2 = (mt * ((N + 511) / 512) + pairs - 1) / pairs;
    const double t1 = static_cast<double>(w1) * (0.00703 * static_cast<double>(K) + 3.4);
    const double t2 = static_cast<double>(w2) * (0.0124 * static_cast<double>(K) + 11.6);
    return t2 < t1 ? 2 : 1;
}
}  // namespace gemm

namespace {

// Launches one square-tile kernel instance: the single-CTA kernel (nb = 0) or
// the CTA-pair kernel with nb 256-column blocks per tile.
template <bool BT>
cudaError_t launch_square(int nb, const DeviceInfo &dev, const CUtensorMap &tmA, const CUtensorMap &tmB,
                          const CUtensorMap &tmC, float *c, int64_t M, int64_t N, int64_t K,
                          long long ldc, bool bf16, int epi, bool pdl, cudaStream_t stream) {
    const int Mi = static_cast<int>(M), Ni = static_cast<int>(N), Ki = static_cast<int>(K);
    if (nb == 0) {
        const int64_t tiles = ((M + gemm::S_BM - 1) / gemm::S_BM) * ((N + gemm::BN - 1) / gemm::BN);
        const int grid = static_cast<int>(tiles < dev.sm_count ? tiles : dev.sm_count);
        const uint32_t idesc = idesc_f16_f32(gemm::S_BM, gemm::BN, false, !BT, bf16);
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
        cfg.blockDim = dim3(gemm::THREADS, 1, 1);
        cfg.dynamicSmemBytes = gemm::S_SMEM;
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        return cudaLaunchKernelEx(&cfg, gemm::gemm_f16f32_kernel<BT>, tmA, tmB, tmC, c, Mi, Ni, Ki, ldc, idesc,
                                  epi);
    }
    const int tile_n = 256 * nb;
    const int64_t tiles = ((M + gemm::P_BM - 1) / gemm::P_BM) * ((N + tile_n - 1) / tile_n);
    const int pairs = static_cast<int>(tiles < dev.max_pairs ? tiles : dev.max_pairs);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(gemm::THREADS, 1, 1);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    const uint32_t idesc = idesc_f16_f32(gemm::P_BM, 256, false, !BT, bf16);
    if (nb == 2) {
        cfg.dynamicSmemBytes = gemm::PairCfg<2>::SMEM;
        return cudaLaunchKernelEx(&cfg, gemm::gemm_f16f32_pair_kernel<2, BT>, tmA, tmB, tmC, c, Mi, Ni, Ki,
                                  ldc, idesc, epi);
    }
    cfg.dynamicSmemBytes = gemm::PairCfg<1>::SMEM;
    return cudaLaunchKernelEx(&cfg, gemm::gemm_f16f32_pair_kernel<1, BT>, tmA, tmB, tmC, c, Mi, Ni, Ki,
                              ldc, idesc, epi);
}

}  // namespace

// The argument rules of the GEMM entry points; CUDAIR_OK when the call is
// valid (including the no-op sizes).
int gemm_check(const void *a, const void *b, const void *c, int64_t M, int64_t N, int64_t K, int64_t lda,
               int64_t ldb, int64_t ldc, uint32_t flags) {
    constexpr uint32_t kKnown = CUDAIR_GEMM_BF16 | CUDAIR_GEMM_B_T | CUDAIR_GEMM_OVERWRITE | CUDAIR_GEMM_C_F16;
    if (flags & ~kKnown) return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: unknown flags 0x%x", flags);
    const bool bt = flags & CUDAIR_GEMM_B_T;
    const bool overwrite = flags & CUDAIR_GEMM_OVERWRITE, c_f16 = flags & CUDAIR_GEMM_C_F16;
    if (c_f16 && !overwrite)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: a half C is written, not accumulated into: "
                                             "CUDAIR_GEMM_C_F16 needs CUDAIR_GEMM_OVERWRITE");
    if (M < 0 || N < 0 || K < 0)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: negative size M=%lld N=%lld K=%lld",
                         (long long)M, (long long)N, (long long)K);
    if (M == 0 || N == 0 || (K == 0 && !overwrite)) return CUDAIR_OK;  // C = C
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: sizes must fit int32");
    if (!c) return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: nil pointer");
    if (ldc < N)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: leading dimension ldc=%lld too small",
                         (long long)ldc);
    // With K = 0 nothing of A or B is read (a written C becomes zero), so
    // their pointers and pitches are not checked.
    if (K > 0) {
        if (!a || !b) return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: nil pointer");
        if (lda < K || ldb < (bt ? K : N))
            return set_error(CUDAIR_ERR_INVALID,
                             "cudair: gemm: leading dimensions lda=%lld ldb=%lld ldc=%lld too small",
                             (long long)lda, (long long)ldb, (long long)ldc);
        if (lda % 8 || ldb % 8)
            return set_error(CUDAIR_ERR_INVALID,
                             "cudair: gemm: lda=%lld and ldb=%lld must be multiples of 8 (16-byte rows)",
                             (long long)lda, (long long)ldb);
        if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15u)
            return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: A and B must be 16-byte aligned");
    }
    const int64_t c_elem = c_f16 ? 2 : 4;
    // C takes a TMA epilogue when a tensor map can describe it (16-byte
    // aligned base and row pitch); an fp32 C accumulated into also has a
    // scalar path, the written forms do not.
    const bool c_tma = (reinterpret_cast<uintptr_t>(c) & 15u) == 0 && (ldc * c_elem) % 16 == 0;
    if (!c_tma && overwrite)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm: a written C must be 16-byte aligned with a 16-byte row pitch");
    if (reinterpret_cast<uintptr_t>(c) & 3u)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: C must be 4-byte aligned");
    return CUDAIR_OK;
}

int gemm_launch(const void *a, const void *b, void *c, int64_t M, int64_t N, int64_t K, int64_t lda,
                int64_t ldb, int64_t ldc, uint32_t flags, cudaStream_t stream) {
    int rc = gemm_check(a, b, c, M, N, K, lda, ldb, ldc, flags);
    if (rc != CUDAIR_OK) return rc;
    const bool bf16 = flags & CUDAIR_GEMM_BF16, bt = flags & CUDAIR_GEMM_B_T;
    const bool overwrite = flags & CUDAIR_GEMM_OVERWRITE, c_f16 = flags & CUDAIR_GEMM_C_F16;
    if (M == 0 || N == 0 || (K == 0 && !overwrite)) return CUDAIR_OK;  // C = C
    const int64_t c_elem = c_f16 ? 2 : 4;
    const bool c_tma = (reinterpret_cast<uintptr_t>(c) & 15u) == 0 && (ldc * c_elem) % 16 == 0;

    DeviceInfo *dev = nullptr;
    rc = device_info(&dev);
    if (rc != CUDAIR_OK) return rc;
    cudaError_t e;
    if (K == 0) {  // C = 0: the product of an empty sum
        e = cudaMemset2DAsync(c, static_cast<size_t>(ldc * c_elem), 0, static_cast<size_t>(N * c_elem),
                              static_cast<size_t>(M), stream);
        return e == cudaSuccess ? CUDAIR_OK : cuda_error(e, "cudaMemset2DAsync(C)");
    }

    const int variant = g_variant.load();
    // The few-row (stream-K) kernel takes the plain form (fp16, B as stored,
    // fp32 C accumulated into) for M <= 64, and for 64 < M <= 128 up to
    // N = 8192.  Past that its re-reads of A from L2 (one per 128-column
    // tile) cost more than the single-CTA kernel's idle SMs (measured: at
    // M = 128, K = 8192: 51.0 against 54.6 us for N = 8192; at K = 4096,
    // 47.5 against 33.2 us for N = 14336).
    if ((variant == 3 || variant == 6) && flags != 0)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm: the few-row kernels (variants 3 and 6) take only the plain form (flags 0)");
    if (variant == 6 && M > 64)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm: the chunked few-row kernel (variant 6) takes M <= 64, got %lld",
                         (long long)M);
    if (variant == 5 && (flags != 0 || K > 64 * kSmallMaxKBlocks))
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm: the small-problem kernel (variant 5) takes the plain form (flags 0) "
                         "and K <= %d",
                         64 * kSmallMaxKBlocks);
    // It also needs at least one (128-column x 64-k) unit of work per SM: on
    // fewer it leaves SMs idle and pays its fix-up anyway (128^3: 14.1 us
    // against 5.3 us for the single-CTA kernel).
    const int64_t units = ((N + 127) / 128) * ((K + 63) / 64);
    // A problem of one wave of the small-problem kernel's 128 x 64 tiles
    // with K <= 512 takes that kernel: the whole K panel is loaded at once,
    // and neither the pipelined kernels' set-up nor the few-row kernel's
    // split-K fix-up is amortised at that size (128 x 4096 x 512: 5.9 us,
    // against 26.6 us for the few-row kernel and 9.4 us for CTA pairs).
    const int64_t small_tiles = ((M + 127) / 128) * ((N + 63) / 64);
    const bool small_auto = variant == 0 && flags == 0 && K <= 64 * kSmallMaxKBlocks &&
                            small_tiles <= dev->sm_count;
    const bool fewrows_auto = variant == 0 && flags == 0 && !small_auto && (M <= 64 || (M <= 128 && N <= 8192)) &&
                              units >= dev->sm_count;
    const int use_variant = small_auto ? 5 : variant;
    // Fewer units than SMs at M <= 64 (narrow N, long K: a single-CTA tile
    // would stream all of K on one SM) take the chunked kernel when its rule
    // splits K into at least two chunks of eight or more k-blocks, one chunk
    // per CTA (chains of 30 launches: 16 x 128 x 4096 8.65 us against 21.2
    // us; 64 x 128 x 4096 15.2 against 21.3 us; 48 x 512 x 2048 11.0
    // against 16.4 us).
    const bool few_units = variant == 0 && flags == 0 && !small_auto && M <= 64 && units < dev->sm_count;
    // The few-row kernels: with fixed k-chunks handed out at run time where
    // that measured faster (chunked_auto_chunks), else stream-K.
    const int chunks = (fewrows_auto || few_units)
                           ? chunked_auto_chunks(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                                                 dev->sm_count)
                           : 0;
    if (variant == 6 || chunks > 0)
        return gemm_chunked_launch(a, b, static_cast<float *>(c), static_cast<int>(M), static_cast<int>(N),
                                   static_cast<int>(K), lda, ldb, ldc, chunks, dev->sm_count, dev->status,
                                   stream);
    if (variant == 3 || fewrows_auto)
        return gemm_skinny_launch(a, b, static_cast<float *>(c), static_cast<int>(M), static_cast<int>(N),
                                  static_cast<int>(K), lda, ldb, ldc, dev->sm_count, dev->status,
                                  stream);
    // 0 auto, 1 single CTA, 2 CTA pair (256 x 256), 4 CTA pair (256 x 512).
    const bool pair_auto = variant == 0 && M > 128 && dev->max_pairs > 0;
    const int nb = (variant == 4) ? 2
                   : (variant == 2) ? 1
                   : pair_auto ? gemm::auto_pair_nb(M, N, K, dev->max_pairs)
                               : 0;
    const uint32_t in_type = bf16 ? CUDAIR_TENSOR_MAP_BFLOAT16 : CUDAIR_TENSOR_MAP_FLOAT16;
    alignas(64) CUtensorMap tmA, tmB, tmC = {};
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
        const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
        const uint32_t box[2] = {64, 128};
        rc = encode_tiled_internal(&tmA, in_type, 2, reinterpret_cast<uint64_t>(a), dims, strides, box,
                                   nullptr, CUDAIR_INTERLEAVE_NONE, CUDAIR_SWIZZLE_128B,
                                   CUDAIR_L2_PROMOTION_256B, CUDAIR_OOB_FILL_NONE);
        if (rc != CUDAIR_OK) return rc;
    }
    {
        // B as stored: K rows of N (boxes of 64 n x 64 k); B^T: N rows of K
        // (boxes of 64 k x 64 n).  Both boxes are 8 KB.
        const uint64_t dims[2] = {static_cast<uint64_t>(bt ? K : N), static_cast<uint64_t>(bt ? N : K)};
        const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
        const uint32_t box[2] = {64, 64};
        rc = encode_tiled_internal(&tmB, in_type, 2, reinterpret_cast<uint64_t>(b), dims, strides, box,
                                   nullptr, CUDAIR_INTERLEAVE_NONE, CUDAIR_SWIZZLE_128B,
                                   CUDAIR_L2_PROMOTION_256B, CUDAIR_OOB_FILL_NONE);
        if (rc != CUDAIR_OK) return rc;
    }
    const int epi = c_f16 ? gemm::kEpiStoreF16
                    : overwrite ? gemm::kEpiStoreF32
                    : c_tma ? gemm::kEpiReduceF32
                            : gemm::kEpiScalarAdd;
    if (epi != gemm::kEpiScalarAdd) {
        const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
        const uint64_t strides[1] = {static_cast<uint64_t>(ldc * c_elem)};
        const uint32_t box[2] = {c_f16 ? 64u : 32u, 32u};  // 128-byte rows
        rc = encode_tiled_internal(&tmC, c_f16 ? CUDAIR_TENSOR_MAP_FLOAT16 : CUDAIR_TENSOR_MAP_FLOAT32, 2,
                                   reinterpret_cast<uint64_t>(c), dims, strides, box, nullptr,
                                   CUDAIR_INTERLEAVE_NONE, CUDAIR_SWIZZLE_128B, CUDAIR_L2_PROMOTION_NONE,
                                   CUDAIR_OOB_FILL_NONE);
        if (rc != CUDAIR_OK) return rc;
    }
    float *cf = static_cast<float *>(c);
    if (use_variant == 5) return gemm_small_launch(tmA, tmB, cf, M, N, K, ldc, dev->status, stream);
    const bool pdl = g_pdl.load() > 0;
    e = bt ? launch_square<true>(nb, *dev, tmA, tmB, tmC, cf, M, N, K, static_cast<long long>(ldc), bf16, epi,
                                 pdl, stream)
           : launch_square<false>(nb, *dev, tmA, tmB, tmC, cf, M, N, K, static_cast<long long>(ldc), bf16,
                                  epi, pdl, stream);
    if (e != cudaSuccess) return cuda_error(e, nb ? "gemm_f16f32_pair_kernel launch" : "gemm_f16f32_kernel launch");
    return CUDAIR_OK;
}

int gemm_f16f32_launch(const void *a, const void *b, float *c, int64_t M, int64_t N, int64_t K,
                       int64_t lda, int64_t ldb, int64_t ldc, cudaStream_t stream) {
    return gemm_launch(a, b, c, M, N, K, lda, ldb, ldc, 0u, stream);
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
    // Up to n = 384 the one-warp-per-tile kernel has the lowest latency
    // (n = 256: 3.5 us, against 4.9 us for the small-problem tcgen05 kernel
    // and 7.7 us for the pipelined ones); from there to n = 512 the
    // small-problem kernel (n = 512: 5.7 against 9.0 us), which the GEMM's
    // automatic choice takes for K <= 512.
    if (n <= 384 && g_variant.load() == 0) {
        if (!a || !b || !c) return set_error(CUDAIR_ERR_INVALID, "cudair: MatMul16: nil pointer");
        if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15u)
            return set_error(CUDAIR_ERR_INVALID, "cudair: MatMul16: A and B must be 16-byte aligned");
        int sms = 0;
        int rc = sm_count_current_device(&sms);  // the device and context checks
        if (rc != CUDAIR_OK) return rc;
        return matmul16_warp_launch(a, b, c, n, static_cast<cudaStream_t>(stream));
    }
    return gemm_f16f32_launch(a, b, c, n, n, n, n, n, n, static_cast<cudaStream_t>(stream));
}

CUDAIR_API int cudair_gemm_f16f32(const void *a, const void *b, float *c, int64_t M, int64_t N,
                                  int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void *stream) {
    clear_error();
    return gemm_f16f32_launch(a, b, c, M, N, K, lda, ldb, ldc, static_cast<cudaStream_t>(stream));
}

CUDAIR_API int cudair_gemm(const void *a, const void *b, void *c, const float *bias, int64_t M,
                           int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int64_t ldbias,
                           uint32_t flags, void *stream) {
    clear_error();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (bias) {
        // C = A.B + bias: bias is copied into C, and the product added to it.
        if (!(flags & CUDAIR_GEMM_OVERWRITE) || (flags & CUDAIR_GEMM_C_F16))
            return set_error(CUDAIR_ERR_INVALID,
                             "cudair: gemm: a bias needs CUDAIR_GEMM_OVERWRITE and an fp32 C");
        int rc = gemm_check(a, b, c, M, N, K, lda, ldb, ldc, flags);
        if (rc != CUDAIR_OK) return rc;
        if (M == 0 || N == 0) return CUDAIR_OK;
        if (ldbias < N)
            return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: ldbias=%lld must be >= N", (long long)ldbias);
        cudaError_t e = cudaMemcpy2DAsync(c, static_cast<size_t>(ldc) * 4, bias, static_cast<size_t>(ldbias) * 4,
                                          static_cast<size_t>(N) * 4, static_cast<size_t>(M),
                                          cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cuda_error(e, "cudaMemcpy2DAsync(bias -> C)");
        return gemm_launch(a, b, c, M, N, K, lda, ldb, ldc, flags & ~CUDAIR_GEMM_OVERWRITE, s);
    }
    return gemm_launch(a, b, c, M, N, K, lda, ldb, ldc, flags, s);
}

CUDAIR_API int cudair_set_gemm_variant(int variant) {
    clear_error();
    if (variant < 0 || variant > 6)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm variant %d, want 0 (auto), 1 (single CTA), 2 (CTA pair), "
                         "3 (few rows), 4 (CTA pair, 256 x 512 tiles), 5 (small problems, K <= 512) "
                         "or 6 (few rows, chunks handed out at run time, M <= 64)",
                         variant);
    g_variant.store(variant);
    return CUDAIR_OK;
}

CUDAIR_API int cudair_set_gemm_pdl(int mode) {
    clear_error();
    if (mode < 0 || mode > 2)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm PDL mode %d, want 0 (off), 1 (on) or 2 (on, B read early)", mode);
    g_pdl.store(mode);
    return CUDAIR_OK;
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
    if (v) {
        skinny_reset_workspace();
        return set_error(CUDAIR_ERR_TIMEOUT, "cudair: a bounded device wait gave up (status 0x%x)", v);
    }
    return CUDAIR_OK;
}

CUDAIR_API int cudair_wait_timeout_selftest(uint64_t limit_ns, void *stream) {
    clear_error();
    gemm::wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "wait_timeout_selftest launch");
    return CUDAIR_OK;
}
