// host_gemm.cu - the entry points that take host buffers: the flows of the
// reference's tests (copy the inputs to the device, launch, copy the result
// back) as single calls whose copies overlap the kernels.  GEMM first:
// C = A.B + C as in the MatMul16 test (advanced_test.go:466-483); VecAdd
// (main_test.go:31-48) and the square MatMul16 call follow at the end.
//
// C is cut into tiles of rows x columns.  Three streams carry the work:
//   in       H2D, in order: for each column block j, the columns of B it
//            needs, then for each row block i the rows of A (on the first
//            column pass only) and tile (i, j) of C;
//   caller   the GEMM of tile (i, j) once its inputs have landed;
//   out      D2H of tile (i, j) of C once its GEMM is done.
// So tile t+1 crosses the host link while tile t is multiplied and tile t-1
// travels back, and the step costs about its bytes at the link's duplex
// speed instead of H2D + GEMM + D2H in series.  Tiles in both dimensions
// matter when B comes from the host: the first tile of C can return after
// one column block of B and one row block of A (at 8192^3 with 2048 x 2048
// tiles, 80 MiB) instead of after all of B, so the copies out start early
// and the step takes the link's duplex time (8192^3: 11.66 -> 10.93 ms of
// copies).  The caller's stream waits for the last copy out, so
// synchronising that stream covers the whole call.
//
// The caller owns every buffer; the library keeps two streams and a set of
// events per device, created on first use.
#include <cuda_runtime.h>

#include <mutex>

#include "cudair_internal.h"

namespace cudair {
namespace {

constexpr int kMaxBlocks = 64;
// Tiles per side of C when B comes from the host (see the tiling rule in
// cudair_gemm_f16f32_host).
#ifndef CUDAIR_HOST_TILES
#define CUDAIR_HOST_TILES 4
#endif
constexpr int kTilesPerSide = CUDAIR_HOST_TILES;

struct HostPipe {
    cudaStream_t in = nullptr, out = nullptr;
    cudaEvent_t start = nullptr;
    cudaEvent_t block_in[kMaxBlocks], block_done[kMaxBlocks], block_out[kMaxBlocks];
    bool ready = false;
};

std::mutex g_pipe_mu;
HostPipe g_pipe[64];

int make_event(cudaEvent_t *e) {
    cudaError_t r = cudaEventCreateWithFlags(e, cudaEventDisableTiming);
    return r == cudaSuccess ? CUDAIR_OK : cuda_error(r, "cudaEventCreateWithFlags");
}

// The pipe of the current device; called with g_pipe_mu held.
int pipe_for_current_device(HostPipe **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return set_error(CUDAIR_ERR_INVALID, "cudair: device index %d out of range", dev);
    HostPipe &p = g_pipe[dev];
    if (!p.ready) {
        if ((e = cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking)) != cudaSuccess)
            return cuda_error(e, "cudaStreamCreateWithFlags");
        if ((e = cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking)) != cudaSuccess)
            return cuda_error(e, "cudaStreamCreateWithFlags");
        int rc = make_event(&p.start);
        for (int i = 0; i < kMaxBlocks && rc == CUDAIR_OK; ++i) {
            rc = make_event(&p.block_in[i]);
            if (rc == CUDAIR_OK) rc = make_event(&p.block_done[i]);
            if (rc == CUDAIR_OK) rc = make_event(&p.block_out[i]);
        }
        if (rc != CUDAIR_OK) return rc;
        p.ready = true;
    }
    *out = &p;
    return CUDAIR_OK;
}

// rows x row_bytes between buffers with pitches dpitch / spitch.
cudaError_t copy_rows(void *dst, size_t dpitch, const void *src, size_t spitch, size_t row_bytes,
                      size_t rows, cudaMemcpyKind kind, cudaStream_t s) {
    if (dpitch == row_bytes && spitch == row_bytes)
        return cudaMemcpyAsync(dst, src, row_bytes * rows, kind, s);
    return cudaMemcpy2DAsync(dst, dpitch, src, spitch, row_bytes, rows, kind, s);
}

}  // namespace
}  // namespace cudair

using namespace cudair;

CUDAIR_API int cudair_gemm_f16f32_host(const void *a_host, const void *b_host, float *c_host,
                                       int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                                       int64_t ldc, void *a_dev, void *b_dev, float *c_dev,
                                       int64_t rows_per_block, void *stream) {
    clear_error();
    if (M < 0 || N < 0 || K < 0)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm_host: negative size M=%lld N=%lld K=%lld",
                         (long long)M, (long long)N, (long long)K);
    if (M == 0 || N == 0) return CUDAIR_OK;  // C has no elements
    // b_host may be NULL: B is then already in b_dev (replicated on the
    // device, e.g. over NVLink), and only A and C cross the host link.
    if (!a_host || !c_host || !a_dev || !b_dev || !c_dev)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm_host: nil pointer");
    if (lda < K || ldb < N || ldc < N)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm_host: host leading dimensions lda=%lld ldb=%lld ldc=%lld too small",
                         (long long)lda, (long long)ldb, (long long)ldc);
    if (K % 8 || N % 8)
        return set_error(CUDAIR_ERR_INVALID,
                         "cudair: gemm_host: K=%lld and N=%lld must be multiples of 8 (the device "
                         "copies are dense, with 16-byte rows)",
                         (long long)K, (long long)N);
    if (rows_per_block < 0)
        return set_error(CUDAIR_ERR_INVALID, "cudair: gemm_host: rows_per_block = %lld",
                         (long long)rows_per_block);
    // Tiles of whole 256-row pair tiles.  By default, with B from the host
    // and N >= 4096, about 4 x 4 tiles (the first copy out starts early);
    // otherwise full-width row blocks, about sixteen, so the copy out of the
    // last block (the part of the call nothing overlaps) stays short.  An
    // explicit rows_per_block asks for full-width row blocks of that height.
    // At most kMaxBlocks tiles.
    // Block boundaries along M (rows) and N (columns).
    int64_t rbnd[kMaxBlocks + 1], cbnd[kMaxBlocks + 1];
    auto even = [](int64_t L, int64_t blk, int64_t *b) -> int {
        int nb = 0;
        b[0] = 0;
        for (int64_t x = 0; x < L; x += blk) b[++nb] = (x + blk < L) ? x + blk : L;
        return nb;
    };
    int row_blocks = 0, col_blocks = 0;
    if (rows_per_block == 0 && b_host && K > 0 && N >= 4096 && M >= 1024) {
        // Even 2D tiles.  Finer ones (6 x 6, 8 x 8) and a short first and
        // last block were measured slower or equal at 8192^3.
        row_blocks = even(M, ((M + kTilesPerSide - 1) / kTilesPerSide + 255) / 256 * 256, rbnd);
        col_blocks = even(N, ((N + kTilesPerSide - 1) / kTilesPerSide + 255) / 256 * 256, cbnd);
    } else {
        int64_t rb = rows_per_block > 0 ? rows_per_block : (M + 15) / 16;
        rb = (rb + 255) / 256 * 256;
        if ((M + rb - 1) / rb > kMaxBlocks) rb = ((M + kMaxBlocks - 1) / kMaxBlocks + 255) / 256 * 256;
        row_blocks = even(M, rb, rbnd);
        col_blocks = even(N, N, cbnd);
    }

    int sms = 0;
    int rc = sm_count_current_device(&sms);  // device and primary-context checks
    if (rc != CUDAIR_OK) return rc;
    std::lock_guard<std::mutex> lk(g_pipe_mu);  // the events are shared per device
    HostPipe *p = nullptr;
    if ((rc = pipe_for_current_device(&p)) != CUDAIR_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
#define CUDAIR_TRY(call, what)                                 \
    do {                                                       \
        if ((e = (call)) != cudaSuccess) return cuda_error(e, what); \
    } while (0)

    // Nothing is copied in before earlier work on the caller's stream (which
    // may still read these device buffers) is done.
    CUDAIR_TRY(cudaEventRecord(p->start, s), "cudaEventRecord");
    CUDAIR_TRY(cudaStreamWaitEvent(p->in, p->start, 0), "cudaStreamWaitEvent");
    CUDAIR_TRY(cudaStreamWaitEvent(p->out, p->start, 0), "cudaStreamWaitEvent");
    const size_t a_row = static_cast<size_t>(K) * 2, b_row = static_cast<size_t>(N) * 2,
                 c_row = static_cast<size_t>(N) * 4;
    int t = 0;
    for (int j = 0; j < col_blocks; ++j) {
        const int64_t n0 = cbnd[j], cols = cbnd[j + 1] - cbnd[j];
        if (K > 0 && b_host)
            CUDAIR_TRY(copy_rows(static_cast<uint8_t *>(b_dev) + static_cast<size_t>(n0) * 2, b_row,
                                 static_cast<const uint8_t *>(b_host) + static_cast<size_t>(n0) * 2,
                                 static_cast<size_t>(ldb) * 2, static_cast<size_t>(cols) * 2,
                                 static_cast<size_t>(K), cudaMemcpyHostToDevice, p->in),
                       "H2D of B");
        for (int i = 0; i < row_blocks; ++i, ++t) {
            const int64_t r0 = rbnd[i], rows = rbnd[i + 1] - rbnd[i];
            uint8_t *a_blk = static_cast<uint8_t *>(a_dev) + static_cast<size_t>(r0) * a_row;
            float *c_tile = c_dev + static_cast<size_t>(r0) * N + n0;
            float *c_host_tile = c_host + static_cast<size_t>(r0) * ldc + n0;
            if (K > 0 && j == 0)
                CUDAIR_TRY(copy_rows(a_blk, a_row,
                                     static_cast<const uint8_t *>(a_host) + static_cast<size_t>(r0) * lda * 2,
                                     static_cast<size_t>(lda) * 2, a_row, static_cast<size_t>(rows),
                                     cudaMemcpyHostToDevice, p->in),
                           "H2D of a block of A");
            CUDAIR_TRY(copy_rows(c_tile, c_row, c_host_tile, static_cast<size_t>(ldc) * 4,
                                 static_cast<size_t>(cols) * 4, static_cast<size_t>(rows),
                                 cudaMemcpyHostToDevice, p->in),
                       "H2D of a tile of C");
            // Everything the tile's GEMM reads (B's columns, A's rows, the
            // tile of C) was copied earlier on the in-stream.
            CUDAIR_TRY(cudaEventRecord(p->block_in[t], p->in), "cudaEventRecord");
            CUDAIR_TRY(cudaStreamWaitEvent(s, p->block_in[t], 0), "cudaStreamWaitEvent");
            rc = gemm_f16f32_launch(a_blk, static_cast<uint8_t *>(b_dev) + static_cast<size_t>(n0) * 2, c_tile,
                                    rows, cols, K, K, N, N, s);
            if (rc != CUDAIR_OK) return rc;
            CUDAIR_TRY(cudaEventRecord(p->block_done[t], s), "cudaEventRecord");
            CUDAIR_TRY(cudaStreamWaitEvent(p->out, p->block_done[t], 0), "cudaStreamWaitEvent");
            CUDAIR_TRY(copy_rows(c_host_tile, static_cast<size_t>(ldc) * 4, c_tile, c_row,
                                 static_cast<size_t>(cols) * 4, static_cast<size_t>(rows),
                                 cudaMemcpyDeviceToHost, p->out),
                       "D2H of a tile of C");
            CUDAIR_TRY(cudaEventRecord(p->block_out[t], p->out), "cudaEventRecord");
        }
    }
    CUDAIR_TRY(cudaStreamWaitEvent(s, p->block_out[t - 1], 0), "cudaStreamWaitEvent");
#undef CUDAIR_TRY
    return CUDAIR_OK;
}

// =============================================================================
// VecAdd from host buffers: the flow of the reference's TestVecAdd
// (main_test.go:31-48: upload a and b, launch VecAdd, copy out back) as one
// call.  The vectors are cut into chunks; chunk i+1 is copied in on the
// in-stream while chunk i is added on the caller's stream and chunk i-1 is
// copied out on the out-stream.
// =============================================================================
CUDAIR_API int cudair_vecadd_host(const float *a_host, const float *b_host, float *out_host, int32_t n,
                                  float *a_dev, float *b_dev, float *out_dev, int32_t chunk,
                                  void *stream) {
    clear_error();
    if (n < 0 || chunk < 0)
        return set_error(CUDAIR_ERR_INVALID, "cudair: vecadd_host: n = %d, chunk = %d", n, chunk);
    if (n == 0) return CUDAIR_OK;
    if (!a_host || !b_host || !out_host || !a_dev || !b_dev || !out_dev)
        return set_error(CUDAIR_ERR_INVALID, "cudair: vecadd_host: nil pointer");
    // By default about sixteen chunks of at least 2^20 elements; a chunk is
    // a multiple of 4 elements, so every chunk keeps the buffers' 16-byte
    // alignment; at most kMaxBlocks chunks.
    int64_t ch = chunk;
    if (ch == 0) ch = ((static_cast<int64_t>(n) + 15) / 16 < (1 << 20)) ? (1 << 20) : (static_cast<int64_t>(n) + 15) / 16;
    ch = (ch + 3) / 4 * 4;
    if ((n + ch - 1) / ch > kMaxBlocks) ch = ((n + kMaxBlocks - 1) / kMaxBlocks + 3) / 4 * 4;
    const int chunks = static_cast<int>((n + ch - 1) / ch);

    int sms = 0;
    int rc = sm_count_current_device(&sms);  // device and primary-context checks
    if (rc != CUDAIR_OK) return rc;
    std::lock_guard<std::mutex> lk(g_pipe_mu);
    HostPipe *p = nullptr;
    if ((rc = pipe_for_current_device(&p)) != CUDAIR_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
#define CUDAIR_TRY(call, what)                                       \
    do {                                                             \
        if ((e = (call)) != cudaSuccess) return cuda_error(e, what); \
    } while (0)
    CUDAIR_TRY(cudaEventRecord(p->start, s), "cudaEventRecord");
    CUDAIR_TRY(cudaStreamWaitEvent(p->in, p->start, 0), "cudaStreamWaitEvent");
    CUDAIR_TRY(cudaStreamWaitEvent(p->out, p->start, 0), "cudaStreamWaitEvent");
    for (int i = 0; i < chunks; ++i) {
        const int64_t i0 = i * ch, len = (n - i0 < ch) ? n - i0 : ch;
        const size_t bytes = static_cast<size_t>(len) * 4;
        CUDAIR_TRY(cudaMemcpyAsync(a_dev + i0, a_host + i0, bytes, cudaMemcpyHostToDevice, p->in), "H2D of a");
        CUDAIR_TRY(cudaMemcpyAsync(b_dev + i0, b_host + i0, bytes, cudaMemcpyHostToDevice, p->in), "H2D of b");
        CUDAIR_TRY(cudaEventRecord(p->block_in[i], p->in), "cudaEventRecord");
        CUDAIR_TRY(cudaStreamWaitEvent(s, p->block_in[i], 0), "cudaStreamWaitEvent");
        rc = cudair_vecadd(a_dev + i0, b_dev + i0, out_dev + i0, static_cast<int32_t>(len), s);
        if (rc != CUDAIR_OK) return rc;
        CUDAIR_TRY(cudaEventRecord(p->block_done[i], s), "cudaEventRecord");
        CUDAIR_TRY(cudaStreamWaitEvent(p->out, p->block_done[i], 0), "cudaStreamWaitEvent");
        CUDAIR_TRY(cudaMemcpyAsync(out_host + i0, out_dev + i0, bytes, cudaMemcpyDeviceToHost, p->out),
                   "D2H of out");
        CUDAIR_TRY(cudaEventRecord(p->block_out[i], p->out), "cudaEventRecord");
    }
    CUDAIR_TRY(cudaStreamWaitEvent(s, p->block_out[chunks - 1], 0), "cudaStreamWaitEvent");
#undef CUDAIR_TRY
    return CUDAIR_OK;
}

// =============================================================================
// MatMul16 from host buffers: advanced_test.go:466-483 (copy A, B and C in,
// launch MatMul16, copy C back) as one call on the caller's stream.  Up to
// n = 512 the copies and cudair_matmul16's one launch run in order (the
// copies are a few microseconds each and there is nothing to overlap); above
// that the pipelined cudair_gemm_f16f32_host takes over.
// =============================================================================
CUDAIR_API int cudair_matmul16_host(const void *a_host, const void *b_host, float *c_host, int32_t n,
                                    void *a_dev, void *b_dev, float *c_dev, void *stream) {
    clear_error();
    if (n < 0 || (n & 15) != 0)
        return set_error(CUDAIR_ERR_INVALID, "cudair: MatMul16: n = %d, want a non-negative multiple of 16", n);
    if (n == 0) return CUDAIR_OK;
    if (!a_host || !b_host || !c_host || !a_dev || !b_dev || !c_dev)
        return set_error(CUDAIR_ERR_INVALID, "cudair: matmul16_host: nil pointer");
    if (n > 512)
        return cudair_gemm_f16f32_host(a_host, b_host, c_host, n, n, n, n, n, n, a_dev, b_dev, c_dev, 0, stream);
    int sms = 0;
    int rc = sm_count_current_device(&sms);  // device and primary-context checks
    if (rc != CUDAIR_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t h = static_cast<size_t>(n) * n * 2, f = static_cast<size_t>(n) * n * 4;
    cudaError_t e;
    if ((e = cudaMemcpyAsync(a_dev, a_host, h, cudaMemcpyHostToDevice, s)) != cudaSuccess)
        return cuda_error(e, "H2D of A");
    if ((e = cudaMemcpyAsync(b_dev, b_host, h, cudaMemcpyHostToDevice, s)) != cudaSuccess)
        return cuda_error(e, "H2D of B");
    if ((e = cudaMemcpyAsync(c_dev, c_host, f, cudaMemcpyHostToDevice, s)) != cudaSuccess)
        return cuda_error(e, "H2D of C");
    if ((rc = cudair_matmul16(a_dev, b_dev, c_dev, n, stream)) != CUDAIR_OK) return rc;
    if ((e = cudaMemcpyAsync(c_host, c_dev, f, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
        return cuda_error(e, "D2H of C");
    return CUDAIR_OK;
}
