// sm100.cuh - hand-written sm_100a device primitives: mbarriers with bounded
// waits, TMA tensor copies, tcgen05 MMA / TMEM, and the shared-memory matrix
// descriptors the tensor cores read.
//
// These are the device-side operations of the reference's cuda/mbarrier.go
// (MBarrier Init / ArriveExpectTx / WaitParity, FenceMBarrierInit,
// FenceProxyAsyncShared: mbarrier.go:59-170), cuda/tma.go
// (CpAsyncBulkTensor2D: tma.go:80-98) and the tensor-core path that
// cuda/mma.go covers for mma.sync, rebuilt on Blackwell's tcgen05.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace cudair {

// ---- status word of the bounded waits --------------------------------------

// One bit per wait site that gave up.  Read (and cleared) by the host through
// cudair_wait_status().
enum WaitSite : uint32_t {
    kSiteProducerEmpty = 1u << 0,
    kSiteMmaFull = 1u << 1,
    kSiteMmaAccEmpty = 1u << 2,
    kSiteEpilogueAccFull = 1u << 3,
    kSiteDrain = 1u << 4,
    kSiteSelfTest = 1u << 5,
};

// Default limit of one wait: far above any legitimate wait in these kernels
// (a whole 65536x8192x8192 GEMM takes milliseconds), far below a watchdog.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ----------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// Makes the initialised barriers visible to the async proxy and the cluster.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `bar` with the given parity to complete, giving up
// when *abort (shared memory, set by any role that gave up) becomes non-zero
// or after limit_ns.  On a timeout it raises *abort, ORs `site` into the
// device status word and returns false; the caller then unwinds.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          unsigned int *status, uint32_t site,
                                          uint64_t limit_ns = kWaitLimitNs) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(a, parity)) return true;
        if ((it & 15u) == 0u) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                *abort = 1;
                atomicOr(status, site);
                return false;
            }
        }
    }
}

// ---- TMA (cp.async.bulk.tensor) -------------------------------------------

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2D tile load global -> shared, completing `bytes` of tx on `bar`.  x is the
// innermost coordinate; callers keep x * element size a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t x, int32_t y, uint64_t cache_hint) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(cache_hint)
        : "memory");
}

// 2D tile reduce-add shared -> global: L2 adds the box element-wise into the
// tensor (fp32 add, round to nearest); elements outside the tensor are
// skipped.  x (innermost) * element size must be a multiple of 16 bytes and
// neither coordinate may be negative.  Tracked by the bulk-group mechanism.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, uint32_t smem_src,
                                                  int32_t x, int32_t y, uint64_t cache_hint) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group.L2::cache_hint"
        " [%0, {%2, %3}], [%1], %4;" ::"l"(reinterpret_cast<uint64_t>(map)),
        "r"(smem_src), "r"(x), "r"(y), "l"(cache_hint)
        : "memory");
}
// 2D tile store shared -> global (elements outside the tensor are skipped);
// the same coordinate rules as the reduce above.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t smem_src, int32_t x,
                                             int32_t y, uint64_t cache_hint) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group.L2::cache_hint"
        " [%0, {%2, %3}], [%1], %4;" ::"l"(reinterpret_cast<uint64_t>(map)),
        "r"(smem_src), "r"(x), "r"(y), "l"(cache_hint)
        : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N of this thread's committed bulk groups are still
// reading their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until at most N of this thread's committed bulk groups are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

// Load with acquire semantics at GPU scope: the writes another CTA made
// before its release (a fence, then the update of this word) are visible to
// this thread's later loads.
__device__ __forceinline__ unsigned int ld_acquire_gpu_u32(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Relaxed load at GPU scope: it orders nothing, so the thread does not wait
// for it until it uses the value.  A caller that then reads what another CTA
// published follows it with a fence (acquire) before those reads.
__device__ __forceinline__ unsigned int ld_relaxed_gpu_u32(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Programmatic dependent launch.  griddepcontrol.wait returns once the grids
// this one depends on have completed and their memory is visible (at once
// when the launch had no such dependency); launch_dependents lets the next
// kernel in the stream be launched before this one ends.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// L2 eviction-priority policies for the cache hints above.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---- tcgen05: tensor memory -------------------------------------------------

// Warp-wide.  Writes the TMEM base address of ncols columns (power of two,
// >= 32) to *dst in shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- tcgen05: MMA -------------------------------------------------------------

// D[tmem] (+)= A[smem desc] . B[smem desc], kind::f16 (fp16/bf16 in, fp32 acc),
// issued by one thread.  accumulate == 0 overwrites D.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on `bar` when every tcgen05.mma this thread issued before it
// has completed (their smem reads and TMEM writes).
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// Instruction descriptor for kind::f16 with fp16 (or, with bf16, bfloat16)
// A and B and fp32 D.
//   bits 4-5 D format (1 = f32), 7-9 A format (0 = f16, 1 = bf16), 10-12 B
//   format, 15 A major (0 = K), 16 B major (1 = MN), 17-22 N/8, 24-28 M/16.
__host__ __device__ constexpr uint32_t idesc_f16_f32(uint32_t M, uint32_t N, bool a_mn_major,
                                                     bool b_mn_major, bool bf16 = false) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
           ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) | ((N >> 3) << 17) |
           ((M >> 4) << 24);
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile:
//   bits 0-13 start address >> 4, 16-29 leading byte offset >> 4,
//   32-45 stride byte offset >> 4, 46-47 version (1 on sm_100),
//   49-51 base offset (0: tiles are 1024-byte aligned), 61-63 layout
//   (2 = SWIZZLE_128B).
// K-major: rows of 128 bytes (64 fp16 along K), 8-row groups `sbo` apart; the
//   leading offset is unused (1).
// MN-major: 128-byte rows hold 64 consecutive M/N values of one k; `lbo` is
//   the distance between 64-wide M/N blocks and `sbo` between 8-row k groups.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// ---- tcgen05: TMEM -> registers ---------------------------------------------

// Each thread of the warp reads 32 consecutive 32-bit columns of its own TMEM
// lane (lane = warp's quarter * 32 + lane id) starting at taddr.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
        "[%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// Named barrier over `count` threads (a multiple of 32) with id `id` (1..15).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Named barrier that also ORs a predicate over the `count` threads: every
// thread gets the same answer, so a decision to stop that any one thread
// takes (or any thread sees in a flag that other roles may raise at any
// moment) is taken by all of them together, and none is left waiting at a
// later barrier for threads that have left.
__device__ __forceinline__ bool named_bar_or(uint32_t id, uint32_t count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(pred ? 1u : 0u), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- thread-block clusters and CTA pairs ---------------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// The shared::cluster address of the variable at local shared address
// `saddr` in the CTA of rank `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

// Arrive (release, cluster scope) on an mbarrier given by its shared::cluster
// address, which may be in another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}

__device__ __forceinline__ void st_shared_cluster_u32(uint32_t cluster_addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// All threads of all CTAs of the cluster.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
                 ::: "memory");
}

// 2D tile load for a CTA pair: the data lands in this CTA's shared memory and
// completes its bytes on the mbarrier at shared::cluster address `bar_cluster`,
// which may belong to the peer CTA of the pair.  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const CUtensorMap *map,
                                                 uint32_t bar_cluster, int32_t x, int32_t y,
                                                 uint64_t cache_hint) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "l"(cache_hint)
        : "memory");
}

// TMEM allocation shared by a CTA pair: one warp of each CTA (same warp id)
// issues it with the same destination slot.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// D (+)= A . B across a CTA pair, issued by one thread of the even CTA:
// M = 256 with rows 0-127 from this CTA's shared memory and 128-255 from the
// peer's (same descriptor), N split the same way for B; each CTA's TMEM
// receives its own 128 rows of D.
__device__ __forceinline__ void umma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc,
                                                 uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on the mbarrier at the same shared-memory offset in every CTA
// of cta_mask when all prior tcgen05.mma of this thread have completed.
__device__ __forceinline__ void umma_commit_pair_multicast(uint64_t *bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}

// Local-only commit of a CTA pair's MMAs (used to drain while unwinding).
__device__ __forceinline__ void umma_commit_pair_local(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void spin_ns(uint64_t ns) {
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < ns) __nanosleep(1000);
}

// ---- misc ------------------------------------------------------------------

__device__ __forceinline__ uint32_t warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

}  // namespace cudair
