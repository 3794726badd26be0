// module_demos.cuh - the remaining entry points of the reference's hopper,
// vecadd and tensor example packages and the wmma GEMMs of its advanced
// package, with the reference's names and parameter ABI, so the module is a
// drop-in for those packages' tests (TestHopper, TestTensorMap, TestLaunchEx,
// TestTensor, the Wmma case of TestAdvanced, the vecadd run program).
//
// Every wait on an mbarrier here is bounded (kDemoWaitNs); a wait that runs
// out gives up and the kernel returns, leaving its outputs unwritten, which
// the caller's check then reports.  None of these kernels traps.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <mma.h>
#include <stdint.h>

namespace cudair_demo {

constexpr int kBlock = 256;                     // the reference's blockSize (hopper.go:10)
constexpr uint64_t kDemoWaitNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint32_t s_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait_parity(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(s_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded phase wait; false when it gave up.
__device__ __forceinline__ bool mbar_wait_parity(uint64_t *bar, uint32_t parity) {
    const uint64_t t0 = now_ns();
    while (!mbar_try_wait_parity(bar, parity))
        if (now_ns() - t0 > kDemoWaitNs) return false;
    return true;
}

}  // namespace cudair_demo

// ---- hopper package (examples/hopper/hopper.go) ------------------------------

// Clusters of two blocks: each block fills its shared tile with
// block*1000 + tid and reads its partner's through distributed shared
// memory; info[block] = rank + 10*size + 100*clusterID + 1000*numClusters
// (hopper.go:16-35).  256 threads per block.
extern "C" __global__ void __cluster_dims__(2, 1, 1) ClusterExchange(int *out, int *info) {
    using namespace cudair_demo;
    __shared__ int tile[kBlock];
    const int tid = threadIdx.x, b = blockIdx.x;
    if (tid < kBlock) tile[tid] = b * 1000 + tid;
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    uint32_t rank, size, cid, ncl;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(size));
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(cid));
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(ncl));
    if (tid < kBlock) {
        uint32_t remote;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(s_addr(&tile[tid])), "r"(rank ^ 1u));
        int v;
        asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(remote) : "memory");
        out[static_cast<int64_t>(b) * blockDim.x + tid] = v;
    }
    if (tid == 0) info[b] = static_cast<int>(rank + 10 * size + 100 * cid + 1000 * ncl);
    // No block leaves while its partner may still read its tile.
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// mbarrier as a block barrier: every thread deposits in[i] in shared memory,
// arrives, waits for the phase; thread 0 then sums the block
// (hopper.go:42-64).
extern "C" __global__ void MBarrierSum(const int *in, int *out) {
    using namespace cudair_demo;
    __shared__ uint64_t bar;
    __shared__ int vals[kBlock];
    const int tid = threadIdx.x;
    if (tid == 0) {
        mbar_init(&bar, blockDim.x);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid < kBlock) vals[tid] = in[static_cast<int64_t>(blockIdx.x) * blockDim.x + tid];
    uint64_t token;
    asm volatile("mbarrier.arrive.shared::cta.b64 %0, [%1];" : "=l"(token) : "r"(s_addr(&bar)) : "memory");
    bool ok = false;
    const uint64_t t0 = now_ns();
    while (!ok && now_ns() - t0 <= kDemoWaitNs) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.test_wait.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(s_addr(&bar)), "l"(token)
            : "memory");
        ok = done != 0;
    }
    // Every thread has finished polling before the barrier is invalidated.
    __syncthreads();
    if (tid == 0 && ok) {
        int s = 0;
        for (int k = 0; k < kBlock; ++k) s += vals[k];
        out[blockIdx.x] = s;
        asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(s_addr(&bar)) : "memory");
    }
}

// Bulk copies (TMA without a tensor map): each block copies its 1 KiB slice
// of in to shared memory completing on an mbarrier, doubles it, and copies it
// back to out with a bulk store (hopper.go:71-100).  n is a multiple of 256.
extern "C" __global__ void TmaDouble(const int *in, int *out, int n) {
    using namespace cudair_demo;
    __shared__ __align__(128) int tile[kBlock];
    __shared__ uint64_t bar;
    __shared__ int landed;
    const int tid = threadIdx.x;
    const int base = blockIdx.x * kBlock;
    if (base >= n) return;  // the whole block, before any barrier
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s_addr(&bar)),
                     "r"(static_cast<uint32_t>(kBlock * sizeof(int)))
                     : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                s_addr(tile)),
            "l"(in + base), "r"(static_cast<uint32_t>(kBlock * sizeof(int))), "r"(s_addr(&bar))
            : "memory");
        landed = mbar_wait_parity(&bar, 0) ? 1 : 0;
        // A wait that gave up leaves the copy in flight, writing this block's
        // shared memory: wait for it once more (bounded) before the block
        // leaves.
        if (!landed) mbar_wait_parity(&bar, 0);
    }
    // One thread decides for the block, so the barrier below is reached by
    // every thread and the early return is the whole block's.
    __syncthreads();
    if (!landed) return;
    if (tid < kBlock) tile[tid] *= 2;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> async proxy
    __syncthreads();
    if (tid == 0) {
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(out + base),
                     "r"(s_addr(tile)), "r"(static_cast<uint32_t>(kBlock * sizeof(int)))
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
}

// leader[i] = the lane elect.sync picks in the warp, elected[i] = 1 in that
// lane only (hopper.go:104-115).
extern "C" __global__ void Elect(int *leader, int *elected) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    uint32_t l, e;
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\telect.sync r|p, 0xffffffff;\n\t"
        "mov.u32 %0, r;\n\tselp.u32 %1, 1, 0, p;\n\t}"
        : "=r"(l), "=r"(e));
    leader[i] = static_cast<int>(l);
    elected[i] = static_cast<int>(e);
}

// Programmatic dependent launch: wait for the prerequisite grid, write
// out[i] = i, let dependents launch (hopper.go:119-127).
extern "C" __global__ void GridDep(int *out) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    out[i] = i;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("fence.acq_rel.cluster;" ::: "memory");
}

// One 32 x 32 fp32 tile through two TMA tensor maps that live in global
// memory: block (bx, by) loads the tile at (32 bx, 32 by), doubles it in
// shared memory and stores it at the same coordinates of the second tensor;
// edges follow the maps' out-of-bounds rules (hopper.go:136-176).
extern "C" __global__ void TensorTileDouble(const CUtensorMap *src, const CUtensorMap *dst) {
    using namespace cudair_demo;
    constexpr int kTile = 32;
    __shared__ __align__(128) float t[kTile * kTile];
    __shared__ uint64_t bar;
    const int tid = threadIdx.x;
    const int x0 = blockIdx.x * kTile, y0 = blockIdx.y * kTile;  // x0 * 4 B: 16-byte aligned
    __shared__ int landed;
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s_addr(&bar)),
                     "r"(static_cast<uint32_t>(sizeof(t)))
                     : "memory");
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%2, %3}], [%4];" ::"r"(s_addr(t)),
            "l"(reinterpret_cast<uint64_t>(src)), "r"(x0), "r"(y0), "r"(s_addr(&bar))
            : "memory");
        landed = mbar_wait_parity(&bar, 0) ? 1 : 0;
        // As in TmaDouble: a load still in flight is waited for (bounded)
        // before the block leaves.
        if (!landed) mbar_wait_parity(&bar, 0);
    }
    __syncthreads();
    if (!landed) return;  // the whole block: every thread read the flag after the barrier
    for (int i = tid; i < kTile * kTile; i += blockDim.x) t[i] *= 2.0f;
    __syncthreads();
    if (tid == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                         reinterpret_cast<uint64_t>(dst)),
                     "r"(x0), "r"(y0), "r"(s_addr(t))
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
}

// The cluster shape comes only from the launch attribute (no
// __cluster_dims__): block b writes its rank + 100 * cluster size
// (hopper.go:178-187).
extern "C" __global__ void ClusterRankRuntime(int *out) {
    if (threadIdx.x != 0) return;
    uint32_t rank, size;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(size));
    out[blockIdx.x] = static_cast<int>(rank + 100 * size);
}

// ldmatrix / stmatrix round trips on four 8x8 fp16 matrices (hopper.go:230-275):
// out[0:256] after stmatrix.x4 (the tile unchanged), out[256:512] after
// stmatrix.x4.trans (each matrix transposed), out[512:640] after
// stmatrix.x2.trans of the first two, out[640:704] after x1.trans of the first.
extern "C" __global__ void StMatrixRoundTrip(const __half *in, __half *out) {
    __shared__ __align__(16) __half t[4 * 64];
    const int lane = threadIdx.x & 31;
    if (threadIdx.x >= 32) return;
    for (int i = lane; i < 4 * 64; i += 32) t[i] = in[i];
    __syncwarp();
    const uint32_t row = cudair_demo::s_addr(&t[lane * 8]);
    uint32_t v4[4], v2[2], v1;
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v4[0]), "=r"(v4[1]), "=r"(v4[2]), "=r"(v4[3]) : "r"(row));
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(v2[0]), "=r"(v2[1]) : "r"(row));
    asm volatile("ldmatrix.sync.aligned.m8n8.x1.shared.b16 {%0}, [%1];" : "=r"(v1) : "r"(row));
    __syncwarp();
    asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(row), "r"(v4[0]),
                 "r"(v4[1]), "r"(v4[2]), "r"(v4[3])
                 : "memory");
    __syncwarp();
    for (int i = lane; i < 4 * 64; i += 32) out[i] = t[i];
    __syncwarp();
    asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(row),
                 "r"(v4[0]), "r"(v4[1]), "r"(v4[2]), "r"(v4[3])
                 : "memory");
    __syncwarp();
    for (int i = lane; i < 4 * 64; i += 32) out[4 * 64 + i] = t[i];
    __syncwarp();
    asm volatile("stmatrix.sync.aligned.m8n8.x2.trans.shared.b16 [%0], {%1, %2};" ::"r"(row), "r"(v2[0]),
                 "r"(v2[1])
                 : "memory");
    __syncwarp();
    for (int i = lane; i < 2 * 64; i += 32) out[8 * 64 + i] = t[i];
    __syncwarp();
    asm volatile("stmatrix.sync.aligned.m8n8.x1.trans.shared.b16 [%0], {%1};" ::"r"(row), "r"(v1) : "memory");
    __syncwarp();
    for (int i = lane; i < 64; i += 32) out[10 * 64 + i] = t[i];
}

// ---- tensor package: mma.sync m16n8k16 matmuls (examples/tensor/tensor.go:9-100) ----
//
// The reference's launch contract for these is one warp per 16 x 8 tile of
// C (LaunchConfig1D((n/16)*(n/8)*32, 128)), a shape tcgen05 cannot take (its
// smallest MMA has 64 rows and is issued for a whole CTA), so they keep the
// warp-level m16n8k16 instruction.  Fragments are read straight from global
// memory: lane l holds rows g = l/4 and g+8, columns 2t, 2t+1 (+8) of A
// (t = l%4), k-rows 2t, 2t+1 (+8) of column g of B, and rows g, g+8, columns
// 2t, 2t+1 of C.

namespace cudair_tensor {

__device__ __forceinline__ uint32_t pack2(uint16_t lo, uint16_t hi) {
    return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

struct Tile {
    int row, col;  // 16-row block, 8-column block
    bool ok;
};

// The 16 x 8 tile of C this warp owns.  ok is false (the warp returns
// without writing) past the last tile, and for every warp when n is not a
// positive multiple of 16 and of kstep or the block is not whole warps: the
// fragments would run past the rows, and a .sync.aligned instruction needs
// all 32 lanes of a warp.
__device__ __forceinline__ Tile tile_of_warp(int n, int kstep = 16) {
    Tile t{0, 0, false};
    if (n <= 0 || n % 16 != 0 || n % kstep != 0 || (blockDim.x & 31) != 0) return t;
    const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t warp = gid / 32;
    const int tiles = n / 8;
    t.row = static_cast<int>(warp / tiles);
    t.col = static_cast<int>(warp % tiles);
    t.ok = warp / tiles < n / 16;
    return t;
}

// A fragment of the 16 x 16 tile at p (row-major, leading dimension n).
__device__ __forceinline__ void frag_a(uint32_t (&a)[4], const uint16_t *p, int n) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    a[0] = *reinterpret_cast<const uint32_t *>(p + g * n + 2 * t);
    a[1] = *reinterpret_cast<const uint32_t *>(p + (g + 8) * n + 2 * t);
    a[2] = *reinterpret_cast<const uint32_t *>(p + g * n + 2 * t + 8);
    a[3] = *reinterpret_cast<const uint32_t *>(p + (g + 8) * n + 2 * t + 8);
}

// B fragment of the 16 x 8 tile at p, B row-major (k-rows, leading dimension n).
__device__ __forceinline__ void frag_b_rows(uint32_t (&b)[2], const uint16_t *p, int n) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    b[0] = pack2(p[(2 * t) * n + g], p[(2 * t + 1) * n + g]);
    b[1] = pack2(p[(2 * t + 8) * n + g], p[(2 * t + 9) * n + g]);
}

// B fragment read column-major: element (k, j) at p[j * n + k].
__device__ __forceinline__ void frag_b_cols(uint32_t (&b)[2], const uint16_t *p, int n) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    b[0] = *reinterpret_cast<const uint32_t *>(p + g * n + 2 * t);
    b[1] = *reinterpret_cast<const uint32_t *>(p + g * n + 2 * t + 8);
}

__device__ __forceinline__ void mma_f16_f32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void mma_bf16_f32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void mma_f16_f16(uint32_t (&d)[2], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f16.f16.f16.f16 {%0, %1}, {%2, %3, %4, %5}, {%6, %7}, {%0, %1};"
        : "+r"(d[0]), "+r"(d[1])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void load_acc(float (&d)[4], const float *p, int n) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    d[0] = p[g * n + 2 * t];
    d[1] = p[g * n + 2 * t + 1];
    d[2] = p[(g + 8) * n + 2 * t];
    d[3] = p[(g + 8) * n + 2 * t + 1];
}

__device__ __forceinline__ void store_acc(float *p, int n, const float (&d)[4]) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    p[g * n + 2 * t] = d[0];
    p[g * n + 2 * t + 1] = d[1];
    p[(g + 8) * n + 2 * t] = d[2];
    p[(g + 8) * n + 2 * t + 1] = d[3];
}

}  // namespace cudair_tensor

// C = A.B, fp16 inputs, fp32 accumulate (tensor.go:15-29).
extern "C" __global__ void MmaF16(const uint16_t *a, const uint16_t *b, float *c, int n) {
    using namespace cudair_tensor;
    const Tile tl = tile_of_warp(n);
    if (!tl.ok) return;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < n; k += 16) {
        uint32_t fa[4], fb[2];
        frag_a(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        frag_b_rows(fb, b + static_cast<int64_t>(k) * n + tl.col * 8, n);
        mma_f16_f32(acc, fa, fb);
    }
    store_acc(c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 8, n, acc);
}

// C = A.B + Bias, the accumulator loaded from bias (tensor.go:31-47).
extern "C" __global__ void MmaF16Bias(const uint16_t *a, const uint16_t *b, const float *bias, float *c,
                                      int n) {
    using namespace cudair_tensor;
    const Tile tl = tile_of_warp(n);
    if (!tl.ok) return;
    float acc[4];
    load_acc(acc, bias + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 8, n);
    for (int k = 0; k < n; k += 16) {
        uint32_t fa[4], fb[2];
        frag_a(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        frag_b_rows(fb, b + static_cast<int64_t>(k) * n + tl.col * 8, n);
        mma_f16_f32(acc, fa, fb);
    }
    store_acc(c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 8, n, acc);
}

// C = A.Bt^T with bt row-major, so B is read column-major (tensor.go:49-64).
extern "C" __global__ void MmaF16Trans(const uint16_t *a, const uint16_t *bt, float *c, int n) {
    using namespace cudair_tensor;
    const Tile tl = tile_of_warp(n);
    if (!tl.ok) return;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < n; k += 16) {
        uint32_t fa[4], fb[2];
        frag_a(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        frag_b_cols(fb, bt + static_cast<int64_t>(tl.col) * 8 * n + k, n);
        mma_f16_f32(acc, fa, fb);
    }
    store_acc(c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 8, n, acc);
}

// C = A.B accumulating in fp16 (tensor.go:66-81).
extern "C" __global__ void MmaF16Half(const uint16_t *a, const uint16_t *b, uint16_t *c, int n) {
    using namespace cudair_tensor;
    const Tile tl = tile_of_warp(n);
    if (!tl.ok) return;
    uint32_t acc[2] = {0u, 0u};
    for (int k = 0; k < n; k += 16) {
        uint32_t fa[4], fb[2];
        frag_a(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        frag_b_rows(fb, b + static_cast<int64_t>(k) * n + tl.col * 8, n);
        mma_f16_f16(acc, fa, fb);
    }
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    uint16_t *p = c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 8;
    *reinterpret_cast<uint32_t *>(p + g * n + 2 * t) = acc[0];
    *reinterpret_cast<uint32_t *>(p + (g + 8) * n + 2 * t) = acc[1];
}

// C = A.B with bfloat16 inputs (tensor.go:83-98).
extern "C" __global__ void MmaBF16(const uint16_t *a, const uint16_t *b, float *c, int n) {
    using namespace cudair_tensor;
    const Tile tl = tile_of_warp(n);
    if (!tl.ok) return;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < n; k += 16) {
        uint32_t fa[4], fb[2];
        frag_a(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        frag_b_rows(fb, b + static_cast<int64_t>(k) * n + tl.col * 8, n);
        mma_bf16_f32(acc, fa, fb);
    }
    store_acc(c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 8, n, acc);
}

// ---- tensor package: tf32 and int8 mma.sync, ldmatrix (examples/tensor/tensor.go:100-238) ----
//
// Same contract as the m16n8k16 family: one warp per 16 x 8 tile of C,
// fragments read from global memory.  g = l/4, t = l%4 for lane l.
//   m16n8k8 tf32:  A a0 (g, t), a1 (g+8, t), a2 (g, t+4), a3 (g+8, t+4);
//                  B b0 (k t, col g), b1 (k t+4, col g).
//   m16n8k32 int8: A a0 row g cols 4t..4t+3, a1 row g+8, a2 row g cols
//                  16+4t.., a3 row g+8 cols 16+4t.. (four bytes a register,
//                  the lowest column in the low byte); B b0 k-rows 4t..4t+3
//                  of column g, b1 k-rows 16+4t.. (lowest k in the low byte).
// The accumulators keep the m16n8k16 layout (rows g, g+8, columns 2t, 2t+1).

namespace cudair_tensor {

// float32 -> tf32, round to nearest with ties away from zero (cvt.rna).
__device__ __forceinline__ uint32_t to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ void frag_a_tf32(uint32_t (&a)[4], const float *p, int n) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    a[0] = to_tf32(p[g * n + t]);
    a[1] = to_tf32(p[(g + 8) * n + t]);
    a[2] = to_tf32(p[g * n + t + 4]);
    a[3] = to_tf32(p[(g + 8) * n + t + 4]);
}

// B row-major (k-rows, leading dimension n).
__device__ __forceinline__ void frag_b_tf32_rows(uint32_t (&b)[2], const float *p, int n) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    b[0] = to_tf32(p[t * n + g]);
    b[1] = to_tf32(p[(t + 4) * n + g]);
}

// B column-major: element (k, j) at p[j * n + k].
__device__ __forceinline__ void frag_b_tf32_cols(uint32_t (&b)[2], const float *p, int n) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    b[0] = to_tf32(p[g * n + t]);
    b[1] = to_tf32(p[g * n + t + 4]);
}

__device__ __forceinline__ void mma_tf32_f32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t word_at(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

__device__ __forceinline__ void frag_a_i8(uint32_t (&a)[4], const uint8_t *p, int n) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    a[0] = word_at(p + g * n + 4 * t);
    a[1] = word_at(p + (g + 8) * n + 4 * t);
    a[2] = word_at(p + g * n + 16 + 4 * t);
    a[3] = word_at(p + (g + 8) * n + 16 + 4 * t);
}

// B row-major: the four k-rows of a register sit n bytes apart.
__device__ __forceinline__ void frag_b_i8_rows(uint32_t (&b)[2], const uint8_t *p, int n) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint8_t *q = p + (16 * r + 4 * t) * n + g;
        b[r] = static_cast<uint32_t>(q[0]) | (static_cast<uint32_t>(q[n]) << 8) |
               (static_cast<uint32_t>(q[2 * n]) << 16) | (static_cast<uint32_t>(q[3 * n]) << 24);
    }
}

// B column-major: element (k, j) at p[j * n + k], so a register is one word.
__device__ __forceinline__ void frag_b_i8_cols(uint32_t (&b)[2], const uint8_t *p, int n) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    b[0] = word_at(p + g * n + 4 * t);
    b[1] = word_at(p + g * n + 16 + 4 * t);
}

__device__ __forceinline__ void mma_s8_s32(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void mma_u8_s32_sat(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.satfinite.s32.u8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void store_acc_i32(int32_t *p, int n, const int (&d)[4]) {
    const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
    p[g * n + 2 * t] = d[0];
    p[g * n + 2 * t + 1] = d[1];
    p[(g + 8) * n + 2 * t] = d[2];
    p[(g + 8) * n + 2 * t + 1] = d[3];
}

__device__ __forceinline__ bool aligned_to(const void *p, uintptr_t bytes) {
    return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0;
}

}  // namespace cudair_tensor

// C = A.B, float32 inputs rounded to tf32, k steps of 8 (tensor.go:102-117).
extern "C" __global__ void MmaTF32(const float *a, const float *b, float *c, int n) {
    using namespace cudair_tensor;
    const Tile tl = tile_of_warp(n);
    if (!tl.ok) return;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < n; k += 8) {
        uint32_t fa[4], fb[2];
        frag_a_tf32(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        frag_b_tf32_rows(fb, b + static_cast<int64_t>(k) * n + tl.col * 8, n);
        mma_tf32_f32(acc, fa, fb);
    }
    store_acc(c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 8, n, acc);
}

// C = A.Bt^T with bt row-major, B read column-major (tensor.go:119-134).
extern "C" __global__ void MmaTF32Trans(const float *a, const float *bt, float *c, int n) {
    using namespace cudair_tensor;
    const Tile tl = tile_of_warp(n);
    if (!tl.ok) return;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < n; k += 8) {
        uint32_t fa[4], fb[2];
        frag_a_tf32(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        frag_b_tf32_cols(fb, bt + static_cast<int64_t>(tl.col) * 8 * n + k, n);
        mma_tf32_f32(acc, fa, fb);
    }
    store_acc(c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 8, n, acc);
}

// C = A.B with signed bytes, int32 accumulate, k steps of 32
// (tensor.go:138-153).  n is a multiple of 32; a and b are 4-byte aligned.
extern "C" __global__ void MmaS8(const int8_t *a, const int8_t *b, int32_t *c, int n) {
    using namespace cudair_tensor;
    const Tile tl = tile_of_warp(n, 32);
    if (!tl.ok || !aligned_to(a, 4)) return;
    const uint8_t *au = reinterpret_cast<const uint8_t *>(a);
    const uint8_t *bu = reinterpret_cast<const uint8_t *>(b);
    int acc[4] = {0, 0, 0, 0};
    for (int k = 0; k < n; k += 32) {
        uint32_t fa[4], fb[2];
        frag_a_i8(fa, au + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        frag_b_i8_rows(fb, bu + static_cast<int64_t>(k) * n + tl.col * 8, n);
        mma_s8_s32(acc, fa, fb);
    }
    store_acc_i32(c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 8, n, acc);
}

// C = A.B with unsigned bytes, B read column-major from a row-major bt,
// .satfinite accumulation (tensor.go:155-171).  n is a multiple of 32; a and
// bt are 4-byte aligned.
extern "C" __global__ void MmaU8(const uint8_t *a, const uint8_t *bt, int32_t *c, int n) {
    using namespace cudair_tensor;
    const Tile tl = tile_of_warp(n, 32);
    if (!tl.ok || !aligned_to(a, 4) || !aligned_to(bt, 4)) return;
    int acc[4] = {0, 0, 0, 0};
    for (int k = 0; k < n; k += 32) {
        uint32_t fa[4], fb[2];
        frag_a_i8(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        frag_b_i8_cols(fb, bt + static_cast<int64_t>(tl.col) * 8 * n + k, n);
        mma_u8_s32_sat(acc, fa, fb);
    }
    store_acc_i32(c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 8, n, acc);
}

// Copies four 8 x 8 half matrices (in, 256 halves back to back) into shared
// memory and reads them with ldmatrix .x4, .x4.trans, .x2 and .x1, lane l
// giving the address of row l; out[lane*4 + i] is register i of .x4,
// out[128 + lane*4 + i] of .x4.trans, out[256 + lane*2 + i] of .x2,
// out[384 + lane] of .x1 (tensor.go:177-205).  Launched as one warp
// (LaunchConfig1D(32, 32)); larger blocks write the same values again.
extern "C" __global__ void LdMatrixRegs(const uint16_t *in, uint32_t *out) {
    using cudair_demo::s_addr;
    __shared__ __align__(16) uint16_t tile[4 * 64];
    if ((blockDim.x & 31) != 0) return;  // .sync.aligned needs whole warps
    for (int i = threadIdx.x; i < 4 * 64; i += blockDim.x) tile[i] = in[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const uint32_t row = s_addr(&tile[lane * 8]);
    uint32_t v4[4], v4t[4], v2[2], v1;
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v4[0]), "=r"(v4[1]), "=r"(v4[2]), "=r"(v4[3])
                 : "r"(row));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v4t[0]), "=r"(v4t[1]), "=r"(v4t[2]), "=r"(v4t[3])
                 : "r"(row));
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(v2[0]), "=r"(v2[1]) : "r"(row));
    asm volatile("ldmatrix.sync.aligned.m8n8.x1.shared.b16 {%0}, [%1];" : "=r"(v1) : "r"(row));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[lane * 4 + i] = v4[i];
        out[32 * 4 + lane * 4 + i] = v4t[i];
    }
    out[2 * 32 * 4 + lane * 2] = v2[0];
    out[2 * 32 * 4 + lane * 2 + 1] = v2[1];
    out[3 * 32 * 4 + lane] = v1;
}

// One 16 x 16 by 16 x 8 fp16 product with both operands staged in shared
// memory and loaded by ldmatrix: .x4 over rows l%16, columns 8*(l/16) of A
// gives the four 8 x 8 blocks in A-fragment order, .x2.trans over rows l%16
// of B gives the B fragment (tensor.go:211-233).  c is 16 x 8, row-major.
extern "C" __global__ void MmaLdMatrix(const uint16_t *a, const uint16_t *b, float *c) {
    using namespace cudair_tensor;
    using cudair_demo::s_addr;
    __shared__ __align__(16) uint16_t at[16 * 16];
    __shared__ __align__(16) uint16_t bt[16 * 8];
    if ((blockDim.x & 31) != 0) return;
    for (int i = threadIdx.x; i < 16 * 16; i += blockDim.x) at[i] = a[i];
    for (int i = threadIdx.x; i < 16 * 8; i += blockDim.x) bt[i] = b[i];
    __syncthreads();
    if (threadIdx.x >= 32) return;  // one warp computes the product
    const int lane = threadIdx.x;
    uint32_t fa[4], fb[2];
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(fa[0]), "=r"(fa[1]), "=r"(fa[2]), "=r"(fa[3])
                 : "r"(s_addr(&at[(lane % 16) * 16 + 8 * (lane / 16)])));
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
                 : "=r"(fb[0]), "=r"(fb[1])
                 : "r"(s_addr(&bt[(lane % 16) * 8])));
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    mma_f16_f32(acc, fa, fb);
    store_acc(c, 8, acc);
}

// ---- wmma: tensor package (bf16, tf32, s8, u8; examples/tensor/tensor.go:238-330) and the
// advanced package's fp16 Wmma / WmmaTrans ----
//
// The reference's contract is one warp per 16 x 16 tile of C
// (LaunchConfig1D((n/16)*(n/16)*32, 128)).  wmma fragment loads want 32-byte
// aligned tiles: bf16 and tf32 tiles are (k steps of 16 and 8 elements are 32
// bytes), so those load from global memory; an int8 k step is 16 bytes, so
// the int8 kernels stage each 16 x 16 operand tile in a 32-byte aligned
// shared block of their own warp and load the fragment from there.  Every
// kernel returns without writing unless n is a positive multiple of 16, the
// block is whole warps and the buffers are 32-byte aligned.

namespace cudair_tensor {

struct Tile16 {
    int row, col;
    bool ok;
};

__device__ __forceinline__ Tile16 tile16_of_warp(int n) {
    Tile16 t{0, 0, false};
    if (n <= 0 || n % 16 != 0 || (blockDim.x & 31) != 0) return t;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const int tiles = n / 16;
    t.row = static_cast<int>(warp / tiles);
    t.col = static_cast<int>(warp % tiles);
    t.ok = warp / tiles < tiles;
    return t;
}

__device__ __forceinline__ bool aligned32(const void *p, const void *q, const void *r, const void *s = nullptr) {
    const uintptr_t m = reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(q) |
                        reinterpret_cast<uintptr_t>(r) | reinterpret_cast<uintptr_t>(s);
    return (m & 31u) == 0;
}

// Copies the 16 x 16 byte tile at p (leading dimension n) into the 256-byte
// shared block s (leading dimension 16); the warp's two lanes per row move 8
// bytes each.
__device__ __forceinline__ void stage_bytes(uint8_t *s, const uint8_t *p, int n) {
    const int l = threadIdx.x & 31, r = l >> 1, h = (l & 1) * 8;
    *reinterpret_cast<uint2 *>(s + r * 16 + h) = *reinterpret_cast<const uint2 *>(p + static_cast<int64_t>(r) * n + h);
}

}  // namespace cudair_tensor

// C = A.B + Bias, bfloat16 inputs, float accumulate (tensor.go:241-256).
extern "C" __global__ void WmmaBF16(const __nv_bfloat16 *a, const __nv_bfloat16 *b, const float *bias, float *c,
                                    int n) {
    using namespace cudair_tensor;
    namespace w = nvcuda::wmma;
    const Tile16 tl = tile16_of_warp(n);
    if (!tl.ok || !aligned32(a, b, c, bias)) return;
    const int64_t rc = static_cast<int64_t>(tl.row) * 16 * n + tl.col * 16;
    w::fragment<w::accumulator, 16, 16, 16, float> acc;
    w::load_matrix_sync(acc, bias + rc, n, w::mem_row_major);
    for (int k = 0; k < n; k += 16) {
        w::fragment<w::matrix_a, 16, 16, 16, __nv_bfloat16, w::row_major> fa;
        w::fragment<w::matrix_b, 16, 16, 16, __nv_bfloat16, w::row_major> fb;
        w::load_matrix_sync(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        w::load_matrix_sync(fb, b + static_cast<int64_t>(k) * n + tl.col * 16, n);
        w::mma_sync(acc, fa, fb, acc);
    }
    w::store_matrix_sync(c + rc, acc, n, w::mem_row_major);
}

// C = A.Bt^T with bt row-major, B read column-major (tensor.go:258-273).
extern "C" __global__ void WmmaBF16Trans(const __nv_bfloat16 *a, const __nv_bfloat16 *bt, float *c, int n) {
    using namespace cudair_tensor;
    namespace w = nvcuda::wmma;
    const Tile16 tl = tile16_of_warp(n);
    if (!tl.ok || !aligned32(a, bt, c)) return;
    w::fragment<w::accumulator, 16, 16, 16, float> acc;
    w::fill_fragment(acc, 0.f);
    for (int k = 0; k < n; k += 16) {
        w::fragment<w::matrix_a, 16, 16, 16, __nv_bfloat16, w::row_major> fa;
        w::fragment<w::matrix_b, 16, 16, 16, __nv_bfloat16, w::col_major> fb;
        w::load_matrix_sync(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        w::load_matrix_sync(fb, bt + static_cast<int64_t>(tl.col) * 16 * n + k, n);
        w::mma_sync(acc, fa, fb, acc);
    }
    w::store_matrix_sync(c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 16, acc, n, w::mem_row_major);
}

// C = A.B + Bias with fp16 inputs, the MatMul16 element types on wmma
// (examples/advanced/advanced.go:11-27).
extern "C" __global__ void Wmma(const __half *a, const __half *b, const float *bias, float *c, int n) {
    using namespace cudair_tensor;
    namespace w = nvcuda::wmma;
    const Tile16 tl = tile16_of_warp(n);
    if (!tl.ok || !aligned32(a, b, c, bias)) return;
    const int64_t rc = static_cast<int64_t>(tl.row) * 16 * n + tl.col * 16;
    w::fragment<w::accumulator, 16, 16, 16, float> acc;
    w::load_matrix_sync(acc, bias + rc, n, w::mem_row_major);
    for (int k = 0; k < n; k += 16) {
        w::fragment<w::matrix_a, 16, 16, 16, __half, w::row_major> fa;
        w::fragment<w::matrix_b, 16, 16, 16, __half, w::row_major> fb;
        w::load_matrix_sync(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        w::load_matrix_sync(fb, b + static_cast<int64_t>(k) * n + tl.col * 16, n);
        w::mma_sync(acc, fa, fb, acc);
    }
    w::store_matrix_sync(c + rc, acc, n, w::mem_row_major);
}

// C = A.Bt^T with bt row-major (B read column-major), zero accumulator, and
// C stored column-major: c[j*n + i] = C[i][j] (examples/advanced/advanced.go:29-46).
extern "C" __global__ void WmmaTrans(const __half *a, const __half *bt, float *c, int n) {
    using namespace cudair_tensor;
    namespace w = nvcuda::wmma;
    const Tile16 tl = tile16_of_warp(n);
    if (!tl.ok || !aligned32(a, bt, c)) return;
    w::fragment<w::accumulator, 16, 16, 16, float> acc;
    w::fill_fragment(acc, 0.f);
    for (int k = 0; k < n; k += 16) {
        w::fragment<w::matrix_a, 16, 16, 16, __half, w::row_major> fa;
        w::fragment<w::matrix_b, 16, 16, 16, __half, w::col_major> fb;
        w::load_matrix_sync(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        w::load_matrix_sync(fb, bt + static_cast<int64_t>(tl.col) * 16 * n + k, n);
        w::mma_sync(acc, fa, fb, acc);
    }
    w::store_matrix_sync(c + static_cast<int64_t>(tl.col) * 16 * n + tl.row * 16, acc, n, w::mem_col_major);
}

// C = A.B, float32 inputs rounded to tf32, m16n16k8 so k steps of 8
// (tensor.go:275-291).
extern "C" __global__ void WmmaTF32(const float *a, const float *b, float *c, int n) {
    using namespace cudair_tensor;
    namespace w = nvcuda::wmma;
    const Tile16 tl = tile16_of_warp(n);
    if (!tl.ok || !aligned32(a, b, c)) return;
    w::fragment<w::accumulator, 16, 16, 8, float> acc;
    w::fill_fragment(acc, 0.f);
    for (int k = 0; k < n; k += 8) {
        w::fragment<w::matrix_a, 16, 16, 8, w::precision::tf32, w::row_major> fa;
        w::fragment<w::matrix_b, 16, 16, 8, w::precision::tf32, w::row_major> fb;
        w::load_matrix_sync(fa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        w::load_matrix_sync(fb, b + static_cast<int64_t>(k) * n + tl.col * 16, n);
        for (int i = 0; i < fa.num_elements; ++i) fa.x[i] = w::__float_to_tf32(fa.x[i]);
        for (int i = 0; i < fb.num_elements; ++i) fb.x[i] = w::__float_to_tf32(fb.x[i]);
        w::mma_sync(acc, fa, fb, acc);
    }
    w::store_matrix_sync(c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 16, acc, n, w::mem_row_major);
}

// C = A.B with signed bytes and int32 accumulate (tensor.go:293-308).
extern "C" __global__ void WmmaS8(const int8_t *a, const int8_t *b, int32_t *c, int n) {
    using namespace cudair_tensor;
    namespace w = nvcuda::wmma;
    __shared__ __align__(32) uint8_t stage[32][2][256];  // per warp: A tile, B tile
    const Tile16 tl = tile16_of_warp(n);
    if (!tl.ok || !aligned32(a, b, c)) return;
    uint8_t *sa = stage[threadIdx.x >> 5][0], *sb = stage[threadIdx.x >> 5][1];
    const uint8_t *au = reinterpret_cast<const uint8_t *>(a), *bu = reinterpret_cast<const uint8_t *>(b);
    w::fragment<w::accumulator, 16, 16, 16, int> acc;
    w::fill_fragment(acc, 0);
    for (int k = 0; k < n; k += 16) {
        stage_bytes(sa, au + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        stage_bytes(sb, bu + static_cast<int64_t>(k) * n + tl.col * 16, n);
        __syncwarp();
        w::fragment<w::matrix_a, 16, 16, 16, signed char, w::row_major> fa;
        w::fragment<w::matrix_b, 16, 16, 16, signed char, w::row_major> fb;
        w::load_matrix_sync(fa, reinterpret_cast<const signed char *>(sa), 16);
        w::load_matrix_sync(fb, reinterpret_cast<const signed char *>(sb), 16);
        __syncwarp();  // the next step's staging overwrites the blocks
        w::mma_sync(acc, fa, fb, acc);
    }
    w::store_matrix_sync(c + static_cast<int64_t>(tl.row) * 16 * n + tl.col * 16, acc, n, w::mem_row_major);
}

// C = A.Bt^T + Bias with unsigned bytes, the accumulator loaded from bias and
// B read column-major from a row-major bt (tensor.go:310-326).
extern "C" __global__ void WmmaU8(const uint8_t *a, const uint8_t *bt, const int32_t *bias, int32_t *c, int n) {
    using namespace cudair_tensor;
    namespace w = nvcuda::wmma;
    __shared__ __align__(32) uint8_t stage[32][2][256];
    const Tile16 tl = tile16_of_warp(n);
    if (!tl.ok || !aligned32(a, bt, c, bias)) return;
    uint8_t *sa = stage[threadIdx.x >> 5][0], *sb = stage[threadIdx.x >> 5][1];
    const int64_t rc = static_cast<int64_t>(tl.row) * 16 * n + tl.col * 16;
    w::fragment<w::accumulator, 16, 16, 16, int> acc;
    w::load_matrix_sync(acc, bias + rc, n, w::mem_row_major);
    for (int k = 0; k < n; k += 16) {
        stage_bytes(sa, a + static_cast<int64_t>(tl.row) * 16 * n + k, n);
        // rows col*16.. of bt are the columns of B: staged with leading
        // dimension 16 they are a column-major 16 x 16 block
        stage_bytes(sb, bt + static_cast<int64_t>(tl.col) * 16 * n + k, n);
        __syncwarp();
        w::fragment<w::matrix_a, 16, 16, 16, unsigned char, w::row_major> fa;
        w::fragment<w::matrix_b, 16, 16, 16, unsigned char, w::col_major> fb;
        w::load_matrix_sync(fa, sa, 16);
        w::load_matrix_sync(fb, sb, 16);
        __syncwarp();
        w::mma_sync(acc, fa, fb, acc);
    }
    w::store_matrix_sync(c + rc, acc, n, w::mem_row_major);
}
