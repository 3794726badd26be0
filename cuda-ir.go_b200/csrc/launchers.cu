// launchers.cu - the module kernels (module_kernels.cuh) compiled into the
// library, the C-ABI launchers for VecAdd and ReduceF32, and the B
// replication primitives of the row-sharded multi-GPU GEMM.
#include <cuda_runtime.h>
#include <string.h>

#include "cudair_internal.h"
#include "module_kernels.cuh"

using namespace cudair;

namespace {

constexpr int kStreamThreads = 512;

// The grid of the streaming kernels (VecAdd, Saxpy, Square): one chunk of
// 512 x V 16-byte vectors per block (V = vectors per thread: 1 for VecAdd and
// Saxpy, 2 for Square), as many blocks as chunks.
int stream_grid(int32_t n, int vectors_per_thread, unsigned *blocks_out) {
    int sms = 0;
    int rc = sm_count_current_device(&sms);  // refuses a device other than sm_100
    if (rc != CUDAIR_OK) return rc;
    const int64_t vec_work = (static_cast<int64_t>(n) + 3) / 4;
    const int64_t chunk = static_cast<int64_t>(kStreamThreads) * vectors_per_thread;
    int64_t blocks = (vec_work + chunk - 1) / chunk;
    if (blocks < 1) blocks = 1;
    *blocks_out = static_cast<unsigned>(blocks);
    return CUDAIR_OK;
}

}  // namespace

CUDAIR_API int cudair_vecadd(const float *a, const float *b, float *out, int32_t n, void *stream) {
    clear_error();
    if (n < 0) return set_error(CUDAIR_ERR_INVALID, "cudair: VecAdd: n = %d", n);
    if (n == 0) return CUDAIR_OK;
    if (!a || !b || !out) return set_error(CUDAIR_ERR_INVALID, "cudair: VecAdd: nil pointer");
    unsigned blocks = 0;
    int rc = stream_grid(n, cudair_detail::kVecAddV, &blocks);
    if (rc != CUDAIR_OK) return rc;
    VecAdd<<<blocks, kStreamThreads, 0, static_cast<cudaStream_t>(stream)>>>(a, b, out, n);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "VecAdd launch");
    return CUDAIR_OK;
}

// The reference-launch MatMul16 (one warp per 16 x 16 tile of C), launched
// by the library for small n, where it beats the pipelined kernels' fixed
// cost (n = 256: 3.6 against 7.8 us per launch).
int cudair::matmul16_warp_launch(const void *a, const void *b, float *c, int n, cudaStream_t stream) {
    const dim3 grid(static_cast<unsigned>(n / 16), static_cast<unsigned>(n / 16), 1);
    MatMul16<<<grid, 32, 0, stream>>>(static_cast<const __half *>(a), static_cast<const __half *>(b), c, n);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "MatMul16 launch");
    return CUDAIR_OK;
}

CUDAIR_API int cudair_saxpy(float alpha, const float *x, float *y, int32_t n, void *stream) {
    clear_error();
    if (n < 0) return set_error(CUDAIR_ERR_INVALID, "cudair: Saxpy: n = %d", n);
    if (n == 0) return CUDAIR_OK;
    if (!x || !y) return set_error(CUDAIR_ERR_INVALID, "cudair: Saxpy: nil pointer");
    unsigned blocks = 0;
    int rc = stream_grid(n, cudair_detail::kVecAddV, &blocks);
    if (rc != CUDAIR_OK) return rc;
    Saxpy<<<blocks, kStreamThreads, 0, static_cast<cudaStream_t>(stream)>>>(alpha, x, y, n);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "Saxpy launch");
    return CUDAIR_OK;
}

CUDAIR_API int cudair_square(float *x, int32_t n, void *stream) {
    clear_error();
    if (n < 0) return set_error(CUDAIR_ERR_INVALID, "cudair: Square: n = %d", n);
    if (n == 0) return CUDAIR_OK;
    if (!x) return set_error(CUDAIR_ERR_INVALID, "cudair: Square: nil pointer");
    unsigned blocks = 0;
    int rc = stream_grid(n, cudair_detail::kSquareV, &blocks);
    if (rc != CUDAIR_OK) return rc;
    Square<<<blocks, kStreamThreads, 0, static_cast<cudaStream_t>(stream)>>>(x, n);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "Square launch");
    return CUDAIR_OK;
}

CUDAIR_API int cudair_reduce_f32(const float *in, float *out, int32_t n, void *stream) {
    clear_error();
    if (n < 0 || n % 32 != 0)
        return set_error(CUDAIR_ERR_INVALID, "cudair: ReduceF32: n = %d, want a multiple of 32", n);
    if (n == 0) return CUDAIR_OK;
    if (!in || !out) return set_error(CUDAIR_ERR_INVALID, "cudair: ReduceF32: nil pointer");
    int sms = 0;
    int rc = sm_count_current_device(&sms);  // also refuses a device other than sm_100
    if (rc != CUDAIR_OK) return rc;
    // The kernel reads one element per launched thread, so the launch covers
    // exactly n threads: 256-thread blocks when they divide n, else warps.
    const int threads = (n % 256 == 0) ? 256 : 32;
    ReduceF32<<<n / threads, threads, 0, static_cast<cudaStream_t>(stream)>>>(in, out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "ReduceF32 launch");
    return CUDAIR_OK;
}

// ---- B replication for the row-sharded GEMM -----------------------------------

CUDAIR_API int cudair_ipc_export(const void *dev_ptr, void *handle_out, uint64_t *offset_out) {
    clear_error();
    if (!dev_ptr || !handle_out || !offset_out)
        return set_error(CUDAIR_ERR_INVALID, "cudair: ipc_export: nil pointer");
    static_assert(sizeof(cudaIpcMemHandle_t) == CUDAIR_IPC_HANDLE_BYTES, "IPC handle size");
    // The handle names the whole allocation that holds dev_ptr (a caching
    // allocator hands out pieces of larger blocks), and the importer maps
    // that allocation's base: report where dev_ptr sits inside it.
    const Driver *d = nullptr;
    int rc = load_driver(&d);
    if (rc != CUDAIR_OK) return rc;
    if ((rc = ensure_context()) != CUDAIR_OK) return rc;
    CUdeviceptr base = 0;
    size_t size = 0;
    CUresult r = d->cuMemGetAddressRange(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr));
    if (r != CUDA_SUCCESS) return cu_error(r, "cuMemGetAddressRange");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    if (e != cudaSuccess) return cuda_error(e, "cudaIpcGetMemHandle");
    memcpy(handle_out, &h, sizeof(h));
    *offset_out = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
    return CUDAIR_OK;
}

CUDAIR_API int cudair_ipc_open(const void *handle, void **dev_ptr_out) {
    clear_error();
    if (!handle || !dev_ptr_out) return set_error(CUDAIR_ERR_INVALID, "cudair: ipc_open: nil pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_error(e, "cudaIpcOpenMemHandle");
    return CUDAIR_OK;
}

CUDAIR_API int cudair_ipc_close(void *dev_ptr) {
    clear_error();
    if (!dev_ptr) return CUDAIR_OK;
    cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    if (e != cudaSuccess) return cuda_error(e, "cudaIpcCloseMemHandle");
    return CUDAIR_OK;
}

CUDAIR_API int cudair_peer_copy(void *dst, const void *src, size_t bytes, void *stream) {
    clear_error();
    if (bytes == 0) return CUDAIR_OK;
    if (!dst || !src) return set_error(CUDAIR_ERR_INVALID, "cudair: peer_copy: nil pointer");
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice,
                                    static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyAsync(peer)");
    return CUDAIR_OK;
}
