// cudair_internal.h - shared declarations of the host side of
// libcudair_b200.so (not part of the public C ABI; see include/cudair_b200.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cudair_b200.h"

#define CUDAIR_API extern "C" __attribute__((visibility("default")))

namespace cudair {

// ---- errors (thread-local last error, like errno) --------------------------

void clear_error();
// Formats the message, stores it as the thread's last error, returns code.
int set_error(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
// "op: cudaErrorX (text)" from a runtime error.
int cuda_error(cudaError_t e, const char *op);
// "op: CUDA_ERROR_X (text)" from a driver result, as cudaresult.Error prints.
int cu_error(CUresult r, const char *op);

// ---- the CUDA driver entry points bound at run time -------------------------

// Bound once from libcuda.so.1 (dlopen; the candidates of the reference's
// host/driver_notwindows.go:15-19), so the library needs no link-time
// dependency on the driver and reports a missing symbol as an error.
struct Driver {
    CUresult (*cuInit)(unsigned int);
    CUresult (*cuGetErrorName)(CUresult, const char **);
    CUresult (*cuGetErrorString)(CUresult, const char **);
    CUresult (*cuCtxGetCurrent)(CUcontext *);
    CUresult (*cuCtxSetCurrent)(CUcontext);
    CUresult (*cuCtxSynchronize)(void);
    CUresult (*cuDevicePrimaryCtxRetain)(CUcontext *, CUdevice);
    CUresult (*cuModuleLoadData)(CUmodule *, const void *);
    CUresult (*cuModuleUnload)(CUmodule);
    CUresult (*cuModuleGetFunction)(CUfunction *, CUmodule, const char *);
    CUresult (*cuLaunchKernelEx)(const CUlaunchConfig *, CUfunction, void **, void **);
    CUresult (*cuMemGetAddressRange)(CUdeviceptr *, size_t *, CUdeviceptr);
    CUresult (*cuTensorMapEncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                       const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                       const cuuint32_t *, CUtensorMapInterleave,
                                       CUtensorMapSwizzle, CUtensorMapL2promotion,
                                       CUtensorMapFloatOOBfill);
};

// Opens the driver and binds the entry points once; thread-safe.
int load_driver(const Driver **out);

// Makes a context current on this thread if none is: the current device's
// primary context, through the runtime (the context gocudrv's Primary() uses).
int ensure_context();

// ---- internal entry points ---------------------------------------------------

// Encodes a tensor map without the EncodeTiled validation (callers inside the
// library pass known-good descriptors).
int encode_tiled_internal(CUtensorMap *out, uint32_t data_type, uint32_t rank,
                          uint64_t global_address, const uint64_t *global_dim,
                          const uint64_t *global_strides, const uint32_t *box_dim,
                          const uint32_t *element_strides, uint32_t interleave, uint32_t swizzle,
                          uint32_t l2_promotion, uint32_t oob_fill);

// Both also check the device (compute capability 10.0) and that the current
// context is the device's primary context, where the library's per-device
// state (symbol addresses, workspaces, streams, events) lives.
int sm_count_current_device(int *count);
// Device address of the bounded-wait status word on the current device.
int wait_status_current_device(unsigned int **status);

int gemm_skinny_launch(const void *a, const void *b, float *c, int M, int N, int K, int64_t lda,
                       int64_t ldb, int64_t ldc, int sm_count, unsigned int *status,
                       cudaStream_t stream);
// The chunked few-row variant (M <= 64): fixed k-chunks per n-tile handed
// out at run time; same operands and result rules as gemm_skinny_launch.
// chunks > 0 sets the chunks per n-tile, 0 picks them automatically.
int gemm_chunked_launch(const void *a, const void *b, float *c, int M, int N, int K, int64_t lda,
                        int64_t ldb, int64_t ldc, int chunks, int sm_count, unsigned int *status,
                        cudaStream_t stream);
// Chunks per n-tile if the chunked kernel is the faster few-row kernel for
// this shape, else 0 (the stream-K kernel).
int chunked_auto_chunks(int M, int N, int K, int sm_count);
int skinny_reset_workspace();
// The programmatic-dependent-launch mode of the few-row GEMM
// (cudair_set_gemm_pdl): 0 off, 1 on, 2 on with B requested early.
int gemm_pdl_mode();

// The one-warp-per-tile MatMul16 (square n, a multiple of 16; row-major, ld = n).
int matmul16_warp_launch(const void *a, const void *b, float *c, int n, cudaStream_t stream);

// The small-problem kernel (gemm_small_sm100.cu): one 128 x 64 tile of C per
// CTA, the whole K panel (K <= 64 * kSmallMaxKBlocks) loaded at once.  Takes
// the tensor maps the square-tile kernels use (A: box 64 k x 128 rows, B:
// box 64 n x 64 k, 128-byte swizzle) and the plain form only.
constexpr int kSmallMaxKBlocks = 8;
int gemm_small_launch(const CUtensorMap &tmA, const CUtensorMap &tmB, float *c, int64_t M, int64_t N,
                      int64_t K, int64_t ldc, unsigned int *status, cudaStream_t stream);

int gemm_f16f32_launch(const void *a, const void *b, float *c, int64_t M, int64_t N, int64_t K,
                       int64_t lda, int64_t ldb, int64_t ldc, cudaStream_t stream);

}  // namespace cudair
