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
//
// A second kernel below (gemm_chunked_kernel, M <= 64) keeps the swap of
// operands and the ring but replaces the static ranges by fixed k-chunks
// that the CTAs take at run time; chunked_auto_chunks picks it for the
// shapes where it measured faster.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
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


// ---- dynamically scheduled variant: fixed k-chunks handed out by ticket ----
//
// The stream-K kernel above gives every CTA the same share of B.  In a chain
// of launches the CTAs do not start together (a CTA takes an SM when the
// preceding launch's CTA on it exits) and do not stream at the same rate, so
// the last MMAs of one launch spread over several microseconds, and every
// tile split between two late CTAs waits for both.  This variant cuts each
// 128-column n-tile into S fixed k-chunks and hands the chunks out at run
// time: CTA c takes chunk c first (so it may request that chunk's B before
// the dependency wait), then the next ticket of a counter in the workspace,
// one chunk ahead of its loads.  A CTA that started late or streams slowly
// simply takes fewer chunks.  Chunks are numbered k-chunk by k-chunk (every
// tile's first chunk, then every tile's second, ...), so the chunks taken
// last belong to tiles whose other parts were done a wave earlier: the last
// chunk of such a tile finds them published and sums the tile at once from
// its registers, instead of publishing its own part and counting in.
//
// Every chunk's fp32 part is summed into C by the tile's last chunk to
// finish, in chunk order: C + part_0 + ... + part_{S-1}.  The chunk bounds
// depend only on the shape, so the result does not depend on which CTA ran
// which chunk, nor on timing.  As in the stream-K fix-up, the last chunk
// checks the tile's counter first and, when it is last, adds its own part
// straight from its registers.  Every CTA takes exactly one ticket past the
// end, so the CTA that takes the last ticket value resets the counter for the
// next launch, which reads it only after its dependency wait.
constexpr int QDEPTH = 4;             // chunk ids in flight from the producer to the consumers
constexpr int NACC = 4;               // TMEM accumulators: the MMA runs up to three chunks ahead
constexpr uint32_t CH_BAR_BYTES = 512;
constexpr int CH_MAX_MPAD = 64;

__host__ __device__ constexpr int ch_stages_for(int mpad) {
    return static_cast<int>((SMEM_BYTES - 1024 - CH_BAR_BYTES) / (B_STAGE_BYTES + mpad * BK * 2)) < MAX_STAGES
               ? static_cast<int>((SMEM_BYTES - 1024 - CH_BAR_BYTES) / (B_STAGE_BYTES + mpad * BK * 2))
               : MAX_STAGES;
}
__host__ __device__ constexpr size_t ch_smem_for(int mpad) {
    return 1024 + static_cast<size_t>(ch_stages_for(mpad)) * (B_STAGE_BYTES + mpad * BK * 2) + CH_BAR_BYTES;
}
static_assert(ch_smem_for(16) <= SMEM_BYTES && ch_smem_for(CH_MAX_MPAD) <= SMEM_BYTES, "shared memory budget");
static_assert(2 * MAX_STAGES * 8 + (2 * NACC + 1) * 8 + 2 * QDEPTH * 8 + 16 + QDEPTH * 4 + 4 <= CH_BAR_BYTES,
              "barrier area");

// k-blocks [kb0, kb1) of chunk s of S over num_kb k-blocks.
__host__ __device__ __forceinline__ int chunk_kb(int s, int S, int num_kb) {
    return static_cast<int>((static_cast<long long>(s) * num_kb) / S);
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_chunked_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA,
                        float *__restrict__ C, int M, int N, int K, long long ldc, int mpad, int S,
                        unsigned int *__restrict__ counters, unsigned int *__restrict__ sched,
                        float *__restrict__ partials, unsigned int *status, int b_early) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

    const uint32_t a_stage_bytes = static_cast<uint32_t>(mpad) * BK * 2;  // multiple of 1024
    const int STAGES = ch_stages_for(mpad);
    uint8_t *sB = smem;
    uint8_t *sA = smem + STAGES * B_STAGE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sA + STAGES * a_stage_bytes);
    uint64_t *full = bars;
    uint64_t *empty = bars + STAGES;
    uint64_t *acc_full = bars + 2 * STAGES;
    uint64_t *acc_empty = acc_full + NACC;
    uint64_t *drain = acc_empty + NACC;
    uint64_t *q_full = drain + 1;
    uint64_t *q_empty = q_full + QDEPTH;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(q_empty + QDEPTH);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int *last_flag = abort_flag + 1;
    volatile int *q_ring = last_flag + 1;
    volatile int *pf_flag = q_ring + QDEPTH;

    const uint32_t warp = warp_id(), lane = lane_id();
    const int n_tiles = (N + BN_T - 1) / BN_T;
    const int num_kb = (K + BK - 1) / BK;
    const int total = n_tiles * S;
    const int G = static_cast<int>(gridDim.x);
    const int c = static_cast<int>(blockIdx.x);
    const uint32_t tmem_cols = mpad <= 16 ? 64u : mpad <= 32 ? 128u : 256u;  // NACC accumulators of mpad columns

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < NACC; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(drain, 1);
        for (int i = 0; i < QDEPTH; ++i) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 5);  // the MMA thread and the four epilogue warps
        }
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
    if (threadIdx.x == 0) grid_launch_dependents();

    if (warp == 0) {
        // ---------------- TMA producer and scheduler ----------------
        if (lane == 0) {
            const uint64_t policy_b = l2_policy_evict_normal();
            const uint64_t policy_a = l2_policy_evict_last();  // A is re-read by every chunk
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            // Two chunks per tile with more tiles than SMs but fewer than two
            // waves (the decode shape: 112 tiles on 148 CTAs): CTA c takes
            // chunks c and c + G, numbered so that CTA c < 2 n_tiles - G runs
            // both halves of tile c in turn and the other 2 (G - n_tiles) CTAs
            // split the remaining tiles between them.  `canon` maps that order
            // to the chunk ids (s * n_tiles + t) the MMA and the epilogue use,
            // so the bits are those of the ticket order (64 x 14336 x 4096:
            // 32.55 -> 29.94 us; 16 x 14336 x 4096: 24.97 -> 24.90 us).
            const bool pairs = (S == 2 && n_tiles < G && G < 2 * n_tiles);
            const int T1 = 2 * n_tiles - G;
            auto canon = [&](int r) { return (!pairs || r < n_tiles) ? r : (r < G ? T1 + r : n_tiles + r - G); };
            int q_raw = c < total ? c : -1;
            int q = q_raw >= 0 ? canon(q_raw) : -1;
            int kb_start = q >= 0 ? chunk_kb(q / n_tiles, S, num_kb) : 0;
            if (b_early && q >= 0) {
                // B does not depend on the preceding kernel (the caller's
                // promise): the first ring of this CTA's first chunk is
                // requested before the dependency wait, A after it.
                const int t = q % n_tiles, kb1 = chunk_kb(q / n_tiles + 1, S, num_kb);
                const int pre = min(kb1 - kb_start, STAGES);
                const int n0 = t * BN_T, nb = (n0 + 64 < N) ? 2 : 1;
                for (int i = 0; i < pre; ++i) {
                    mbar_arrive_expect_tx(&full[i], nb * B_BOX_BYTES + a_stage_bytes);
                    for (int j = 0; j < nb; ++j)
                        tma_load_2d(sB + i * B_STAGE_BYTES + j * B_BOX_BYTES, &tmB, &full[i], n0 + 64 * j,
                                    (kb_start + i) * BK, policy_b);
                }
                grid_dependency_wait();
                for (int i = 0; i < pre; ++i)
                    tma_load_2d(sA + i * a_stage_bytes, &tmA, &full[i], (kb_start + i) * BK, 0, policy_a);
                issued = static_cast<uint32_t>(pre);
                stage = issued % static_cast<uint32_t>(STAGES);
                phase = (issued == static_cast<uint32_t>(STAGES)) ? 1u : 0u;
                kb_start += pre;
            } else {
                grid_dependency_wait();
            }
            for (int j = 0; ok; ++j) {
                // Hand the chunk (or the end, -1) to the MMA thread and the
                // epilogue.
                const int slot = j % QDEPTH;
                if (!mbar_wait(&q_empty[slot], ((j / QDEPTH) & 1) ^ 1, abort_flag, status, kSiteProducerEmpty)) {
                    ok = false;
                    break;
                }
                q_ring[slot] = q;
                mbar_arrive(&q_full[slot]);
                if (q < 0) break;
                // The next chunk, taken one chunk ahead of its loads.
                const bool grab = !pairs && total > G;
                const unsigned int raw = grab ? atomicAdd(&sched[0], 1u) : 0u;
                const int next = grab ? G + static_cast<int>(raw) : (pairs ? q_raw + G : total);
                const int t = q % n_tiles, kb1 = chunk_kb(q / n_tiles + 1, S, num_kb);
                const int n0 = t * BN_T, nb = (n0 + 64 < N) ? 2 : 1;  // skip a box wholly beyond N
                for (int kb = kb_start; kb < kb1; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, status, kSiteProducerEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], nb * B_BOX_BYTES + a_stage_bytes);
                    for (int jj = 0; jj < nb; ++jj)
                        tma_load_2d(sB + stage * B_STAGE_BYTES + jj * B_BOX_BYTES, &tmB, &full[stage],
                                    n0 + 64 * jj, kb * BK, policy_b);
                    tma_load_2d(sA + stage * a_stage_bytes, &tmA, &full[stage], kb * BK, 0, policy_a);
                    ++issued;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                q_raw = next < total ? next : -1;
                q = q_raw >= 0 ? canon(q_raw) : -1;
                kb_start = q >= 0 ? chunk_kb(q / n_tiles, S, num_kb) : 0;
                // Every CTA takes exactly one ticket past the end, so the one
                // that takes the last value (total - 1) takes the launch's last
                // ticket: it resets the counter for the next launch, which reads
                // it only after its dependency wait.
                if (grab && raw == static_cast<unsigned int>(total - 1)) sched[0] = 0u;
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
            grid_dependency_wait();
            const uint32_t idesc = idesc_f16_f32(BN_T, static_cast<uint32_t>(mpad), true, false);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true, issued_any = false;
            for (int j = 0; ok; ++j) {
                const int slot = j % QDEPTH;
                if (!mbar_wait(&q_full[slot], (j / QDEPTH) & 1, abort_flag, status, kSiteMmaFull)) {
                    ok = false;
                    break;
                }
                const int q = q_ring[slot];
                mbar_arrive(&q_empty[slot]);
                if (q < 0) break;
                const int kb0 = chunk_kb(q / n_tiles, S, num_kb), kb1 = chunk_kb(q / n_tiles + 1, S, num_kb);
                if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, status, kSiteMmaAccEmpty)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t d_tmem = tmem_base + acc * static_cast<uint32_t>(mpad);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, status, kSiteMmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t b_base = smem_u32(sB + stage * B_STAGE_BYTES);
                    const uint32_t a_base = smem_u32(sA + stage * a_stage_bytes);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t b_desc = smem_desc_sw128(b_base + kk * 2048, B_BOX_BYTES, 1024);
                        const uint64_t a_desc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                        umma_f16_ss(d_tmem, b_desc, a_desc, idesc, (kb == kb0 && kk == 0) ? 0u : 1u);
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
                if (++acc == NACC) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok && issued_any) {
                umma_commit(drain);
                int never = 0;
                mbar_wait(drain, 0, &never, status, kSiteDrain);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue and tile sums (warps 2..5) ----------------
        // Each chunk's accumulator is read into registers and handed back to
        // the MMA at once; the memory round trips that follow (the tile
        // counter, the part's visibility, the sum) then delay only this
        // role, not the tensor pipe.  The counter is read when the chunk id
        // arrives, long before the accumulator does.
        grid_dependency_wait();  // C and the workspace may be the preceding kernel's
        const uint32_t qw = warp & 3u;
        const int nl = static_cast<int>(qw * 32 + lane);  // n within the tile
        const bool leader = (warp == 2 && lane == 0);
        const int chunks16 = mpad / 16;  // 1 to 4
        uint32_t acc = 0, acc_phase = 0;
        for (int j = 0;; ++j) {
            const int slot = j % QDEPTH;
            const bool got = mbar_wait(&q_full[slot], (j / QDEPTH) & 1, abort_flag, status, kSiteEpilogueAccFull);
            if (named_bar_or(1, 128, !got || *abort_flag != 0)) break;
            const int q = q_ring[slot];
            if (leader) *pf_flag = 0;
            named_bar_sync(1, 128);  // every thread has read the slot
            if (lane == 0) mbar_arrive(&q_empty[slot]);
            if (q < 0) break;
            const int t = q % n_tiles, s = q / n_tiles;
            const int n = t * BN_T + nl;
            const unsigned int others = static_cast<unsigned int>(S - 1);
            unsigned int pre = 0;
            if (leader && S > 1) pre = ld_relaxed_gpu_u32(&counters[t]);
            // Two chunks per tile at M <= 16: while the accumulator is being
            // computed the leader watches the tile counter, and once the other
            // chunk has published its part every thread loads C and that part,
            // so the tile's sum after the last MMA waits on no memory.
            const bool watch = (S == 2 && chunks16 == 1);
            const float *other_part = partials + (static_cast<size_t>(1 - s) * n_tiles + t) * BN_T * mpad;
            bool known = false;  // leader: the other part is published
            bool have = false;   // this thread holds C and the other part
            float cv[16], pv[16];
            bool ok = true;
            {
                const uint32_t bar_a = smem_u32(&acc_full[acc]);
                const uint64_t t0 = globaltimer_ns();
                uint64_t next_poll = 0;
                for (uint32_t it = 1;; ++it) {
                    if (mbar_try_wait(bar_a, acc_phase)) break;
                    if (watch) {
                        if (leader && !known) {
                            const uint64_t now = globaltimer_ns();
                            if (now >= next_poll) {
                                if (pre == others || ld_relaxed_gpu_u32(&counters[t]) == others) {
                                    __threadfence();  // acquire
                                    known = true;
                                    *pf_flag = 1;
                                }
                                next_poll = now + 500;
                            }
                        }
                        if (!have && *pf_flag != 0) {
                            __threadfence();
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                cv[i] = (i < M && n < N) ? C[static_cast<long long>(i) * ldc + n] : 0.f;
                                pv[i] = (i < M) ? __ldcg(other_part + i * BN_T + nl) : 0.f;
                            }
                            have = true;
                        }
                    }
                    if ((it & 15u) == 0u) {
                        if (*abort_flag) {
                            ok = false;
                            break;
                        }
                        if (globaltimer_ns() - t0 > kWaitLimitNs) {
                            *abort_flag = 1;
                            atomicOr(status, kSiteEpilogueAccFull);
                            ok = false;
                            break;
                        }
                    }
                }
            }
            if (named_bar_or(1, 128, !ok || *abort_flag != 0)) break;
            tc_fence_after_sync();
            const uint32_t t_row = tmem_base + ((qw * 32u) << 16) + acc * static_cast<uint32_t>(mpad);
            // Up to 32 rows the accumulator is read into registers and handed
            // back to the MMA at once.  At 48 and 64 rows it stays in TMEM, is
            // read one 16-row group at a time where it is needed, and is
            // handed back once the chunk's part is published or its tile
            // summed (with four accumulators the MMA still runs up to three
            // chunks ahead).  Every TMEM read below is warp-uniform.
            const bool hold = chunks16 > 2;
            const uint32_t acc_used = acc;
            auto hand_back = [&]() {
                tc_fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[acc_used]);
            };
            uint32_t r[2][16];
            if (!hold) {
                tmem_ld_32x32b_x16(t_row, r[0]);
                if (chunks16 > 1) tmem_ld_32x32b_x16(t_row + 16, r[1]);
                tmem_ld_wait();
                hand_back();
            }
            if (++acc == NACC) {
                acc = 0;
                acc_phase ^= 1u;
            }
            // This thread's 16 accumulator values of row group jj.
            auto own_group = [&](int jj, uint32_t (&g)[16]) {
                if (hold) {
                    tmem_ld_32x32b_x16(t_row + 16u * static_cast<uint32_t>(jj), g);
                    tmem_ld_wait();
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) g[i] = (jj == 0) ? r[0][i] : r[1][i];
                }
            };
            if (S == 1) {
#pragma unroll
                for (int jj = 0; jj < CH_MAX_MPAD / 16; ++jj) {
                    if (jj >= chunks16 || 16 * jj >= M) break;
                    uint32_t g[16];
                    own_group(jj, g);
                    if (n < N) {
                        float v[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            v[i] = (16 * jj + i < M) ? C[static_cast<long long>(16 * jj + i) * ldc + n] : 0.f;
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (16 * jj + i < M)
                                C[static_cast<long long>(16 * jj + i) * ldc + n] = v[i] + __uint_as_float(g[i]);
                    }
                }
                if (hold) hand_back();
                continue;
            }
            // The early read may predate the other chunks' counts: read again
            // now (one load, against a publish, fence and count otherwise).
            if (leader) {
                if (!known && pre != others) pre = ld_relaxed_gpu_u32(&counters[t]);
                *last_flag = (known || pre == others) ? 1 : 0;
            }
            named_bar_sync(1, 128);
            bool last = *last_flag != 0;
            if (!last) {
                float *part = partials + static_cast<size_t>(q) * BN_T * mpad;
#pragma unroll
                for (int jj = 0; jj < CH_MAX_MPAD / 16; ++jj) {
                    if (jj >= chunks16) break;
                    uint32_t g[16];
                    own_group(jj, g);
#pragma unroll
                    for (int i = 0; i < 16; ++i) part[(16 * jj + i) * BN_T + nl] = __uint_as_float(g[i]);
                }
                // The part is published by one release: the barrier orders
                // every thread's stores before the leader's fence and count.
                named_bar_sync(1, 128);
                if (leader) {
                    __threadfence();
                    const unsigned int prev = atomicAdd(&counters[t], 1u);
                    *last_flag = (prev == others) ? 1 : 0;
                }
                named_bar_sync(1, 128);
                last = *last_flag != 0;
            }
            if (last && watch) {
                if (!have) {
                    __threadfence();  // acquire: the other part is visible from here
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        cv[i] = (i < M && n < N) ? C[static_cast<long long>(i) * ldc + n] : 0.f;
                        pv[i] = (i < M) ? __ldcg(other_part + i * BN_T + nl) : 0.f;
                    }
                }
                // C + part 0 + part 1, the order of the general sum below.
                if (n < N) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float own = __uint_as_float(r[0][i]);
                        float v = cv[i];
                        v += (s == 0) ? own : pv[i];
                        v += (s == 0) ? pv[i] : own;
                        if (i < M) C[static_cast<long long>(i) * ldc + n] = v;
                    }
                }
                if (leader) counters[t] = 0u;
            } else if (last) {
                __threadfence();  // acquire: the other chunks' parts are visible from here
                // Sixteen rows at a time: C, then the parts in chunk order,
                // four loaded together (this chunk's own from registers).
#pragma unroll
                for (int jj = 0; jj < CH_MAX_MPAD / 16; ++jj) {
                    if (jj >= chunks16 || 16 * jj >= M) break;
                    uint32_t g[16];
                    own_group(jj, g);
                    if (n >= N) continue;
                    float v[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        v[i] = (16 * jj + i < M) ? C[static_cast<long long>(16 * jj + i) * ldc + n] : 0.f;
                    for (int sb = 0; sb < S; sb += 4) {
                        float pv[4][16];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const int ss = sb + k;
                            if (ss >= S || ss == s) continue;
                            const float *pc = partials + (static_cast<size_t>(ss) * n_tiles + t) * BN_T * mpad;
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                pv[k][i] = (16 * jj + i < M) ? __ldcg(pc + (16 * jj + i) * BN_T + nl) : 0.f;
                        }
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const int ss = sb + k;
                            if (ss >= S) break;
#pragma unroll
                            for (int i = 0; i < 16; ++i) v[i] += (ss == s) ? __uint_as_float(g[i]) : pv[k][i];
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        if (16 * jj + i < M) C[static_cast<long long>(16 * jj + i) * ldc + n] = v[i];
                }
                if (leader) counters[t] = 0u;
            }
            if (hold) hand_back();
            named_bar_sync(1, 128);  // last_flag is reused by the next chunk
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

// Tile counters, the chunked variant's ticket counter (in a 1 KiB block), then
// the partial sums: two slots (128 x M fp32) per CTA for up to 160 CTAs at
// M = 128, or one slot per chunk of the chunked variant: 21.25 MB.
constexpr size_t kSchedBytes = 1024;
constexpr size_t kWorkspaceBytes =
    skinny::COUNTER_BYTES + kSchedBytes + 160u * 2u * skinny::BN_T * skinny::MAX_M * sizeof(float);

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
        e = cudaFuncSetAttribute(skinny::gemm_chunked_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(skinny::SMEM_BYTES));
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(chunked)");
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
    const long long slots_fit = static_cast<long long>(ws->bytes - skinny::COUNTER_BYTES - kSchedBytes) /
                                (2LL * skinny::BN_T * mpad * static_cast<long long>(sizeof(float)));
    long long g = T < sm_count ? T : sm_count;
    if (g > slots_fit) g = slots_fit;
    const int grid = static_cast<int>(g);
    unsigned int *counters = static_cast<unsigned int *>(ws->ptr);
    float *partials =
        reinterpret_cast<float *>(static_cast<uint8_t *>(ws->ptr) + skinny::COUNTER_BYTES + kSchedBytes);
    cudaError_t e = launch_skinny(grid, skinny::smem_for(mpad), stream, gemm_pdl_mode(), tmB, tmA, c, M, N,
                                  K, static_cast<long long>(ldc), mpad, counters, partials, status);
    if (e != cudaSuccess) return cuda_error(e, "gemm_skinny_kernel launch");
    return CUDAIR_OK;
}

// The automatic choice takes the chunked kernel up to this many rows (all the
// kernel runs).  At 33 to 64 rows, chains of 30 launches against stream-K:
// 64 x 14336 x 4096 32.3 against 34.0 us (S = 2), 33 x 14336 x 4096 28.2
// against 30.9, 40 x 8192 x 8192 29.6 against 34.6, 64 x 4096 x 4096 16.6
// against 21.8 (S = 4), 64 x 2048 x 8192 20.5 (S = 4) against 27.8.  With
// more 128-column tiles than SMs it lost there (160, 192 and 256 tiles at
// M = 64: 44.2, 48.1, 61.3 against 40.9, 46.9, 59.4 us), so above 32 rows
// those shapes keep stream-K.
constexpr int kChunkedAutoMaxM = skinny::CH_MAX_MPAD;

// The automatic choice between the two few-row kernels, from measurements on
// a B200 (148 SMs) of M = 1, 16 and 32 with N from 1024 to 57344 and K from
// 4096 to 28672, each kernel in a chain of 20-30 launches with B requested
// early.  Returns the chunks per n-tile for the chunked kernel, or 0 for the
// stream-K kernel (M > 64, or K under four k-blocks per chunk).
//   * At most half as many 128-column tiles as SMs: G / n_tiles chunks per
//     tile (at most one per eight k-blocks), so every CTA runs at most one
//     chunk and every tile has equal parts (8-16 % faster than stream-K at 8
//     to 64 tiles).
//   * More tiles: the chunks run in waves of G, and a wave that is only
//     partly full leaves the HBM to fewer SMs.  The count S in 2..4 (2..3 at
//     M > 16) whose waves are fullest, n_tiles * S / (ceil(n_tiles * S / G) * G),
//     wins, a smaller S when two are within 0.02 of each other.  That picked
//     the measured best, or one within 2 %, at every tile count from 80 to
//     448; against stream-K it is 3-12 % faster, except at M = 32 with 160
//     or 256 tiles (1-4 % slower).
int chunked_auto_chunks(int M, int N, int K, int sm_count) {
    const int mpad = (M + 15) / 16 * 16;
    if (mpad > kChunkedAutoMaxM || sm_count < 2) return 0;
    const long long G = sm_count;
    const long long n_tiles = (N + skinny::BN_T - 1) / skinny::BN_T;
    const long long max_s = ((K + skinny::BK - 1) / skinny::BK) / 4;  // chunks of at least four k-blocks
    if (2 * n_tiles <= G) {
        // Chunks of at least eight k-blocks here: shorter ones cost more in
        // their parts' sum than they gain in SMs (16 x 128 x 4096: 8.65 us
        // with 8 chunks, 9.1 with 16; 64 x 128 x 4096: 15.2 against 20.5;
        // 32 x 296 x 2048: 9.5 with 4 chunks against 9.9 with 8).  Above
        // four, a multiple of four: the tile's sum loads the parts four at a
        // time (1 x 1024 x 16384: 13.7 us with 16 chunks, 15.3 with 18;
        // 16 x 2048 x 8192: 11.9 with 8, 13.6 with 9).
        long long S = std::min(G / n_tiles, static_cast<long long>((K + skinny::BK - 1) / skinny::BK) / 8);
        if (S > 4) S -= S % 4;
        return S >= 2 ? static_cast<int>(S) : 0;
    }
    if (mpad > 32 && n_tiles > G) return 0;
    int best = 0;
    double best_fill = 0.0;
    for (long long S = 2; S <= (mpad <= 16 ? 4 : 3) && S <= max_s; ++S) {
        const long long total = n_tiles * S;
        const double fill = static_cast<double>(total) / static_cast<double>(((total + G - 1) / G) * G);
        if (fill > best_fill + 0.02) {
            best_fill = fill;
            best = static_cast<int>(S);
        }
    }
    return best;
}

// Chunks per n-tile for a launch of the chunked kernel: `chunks` when > 0,
// else the automatic count (two where the automatic rule would run
// stream-K); CUDAIR_FEWROWS_CHUNKS, when set, overrides both.  At most one
// chunk per k-block and no more chunks than the partial slots hold.
int chunked_chunks(int chunks, int M, int N, int K, int grid, size_t partial_bytes) {
    const int mpad = (M + 15) / 16 * 16;
    const int n_tiles = (N + skinny::BN_T - 1) / skinny::BN_T;
    const int num_kb = (K + skinny::BK - 1) / skinny::BK;
    long long S = chunks > 0 ? chunks : chunked_auto_chunks(M, N, K, grid);
    if (S <= 0) S = 2;
    if (const char *env = std::getenv("CUDAIR_FEWROWS_CHUNKS")) {
        const long long v = std::atoll(env);
        if (v > 0) S = v;
    }
    if (S > num_kb) S = num_kb;
    const long long fit =
        static_cast<long long>(partial_bytes / (static_cast<size_t>(skinny::BN_T) * mpad * sizeof(float))) / n_tiles;
    if (S > fit) S = fit;
    return S < 1 ? 1 : static_cast<int>(S);
}

int gemm_chunked_launch(const void *a, const void *b, float *c, int M, int N, int K, int64_t lda,
                        int64_t ldb, int64_t ldc, int chunks, int sm_count, unsigned int *status,
                        cudaStream_t stream) {
    if (M < 1 || M > skinny::CH_MAX_MPAD)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm: the chunked few-row kernel takes 1 <= M <= %d, got %d",
                         skinny::CH_MAX_MPAD, M);
    const int n_tiles = (N + skinny::BN_T - 1) / skinny::BN_T;
    if (n_tiles > skinny::MAX_TILES)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: N = %d too large for the few-row kernel", N);
    Workspace *ws = nullptr;
    int rc = workspace(&ws);
    if (rc != CUDAIR_OK) return rc;
    const int mpad = (M + 15) / 16 * 16;
    const size_t partial_bytes = ws->bytes - skinny::COUNTER_BYTES - kSchedBytes;
    if (static_cast<size_t>(n_tiles) * skinny::BN_T * mpad * sizeof(float) > partial_bytes)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm: N = %d too large for the chunked kernel", N);

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
    const int S = chunked_chunks(chunks, M, N, K, sm_count, partial_bytes);
    const long long total = static_cast<long long>(n_tiles) * S;
    const int grid = static_cast<int>(total < sm_count ? total : sm_count);
    uint8_t *base = static_cast<uint8_t *>(ws->ptr);
    unsigned int *counters = reinterpret_cast<unsigned int *>(base);
    unsigned int *sched = reinterpret_cast<unsigned int *>(base + skinny::COUNTER_BYTES);
    float *partials = reinterpret_cast<float *>(base + skinny::COUNTER_BYTES + kSchedBytes);

    const int pdl = gemm_pdl_mode();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(skinny::THREADS, 1, 1);
    cfg.dynamicSmemBytes = skinny::ch_smem_for(mpad);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl > 0) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, skinny::gemm_chunked_kernel, tmB, tmA, c, M, N, K,
                                       static_cast<long long>(ldc), mpad, S, counters, sched, partials, status,
                                       pdl == 2 ? 1 : 0);
    if (e != cudaSuccess) return cuda_error(e, "gemm_chunked_kernel launch");
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
