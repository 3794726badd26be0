/*
 * cudair_b200.h - the C ABI of the B200 (sm_100a) build of cuda-ir.go's
 * MatMul16 / VecAdd path.
 *
 * Two things replace the reference's compiled kernels and host helpers:
 *
 *  1. A kernel module image (cudair_kernels.cubin, sm_100a) whose entry
 *     points keep the reference's names and parameter ABI, so a caller that
 *     loads a module and launches "MatMul16" / "VecAdd" / "ReduceF32" by name
 *     (gocudrv ctx.LoadModule + Function.Launch) runs them unchanged:
 *       MatMul16(const __half* a, const __half* b, float* c, int32 n)
 *           examples/hopper/hopper.go:201 (launched as in advanced_test.go:477)
 *       VecAdd(const float* a, const float* b, float* out, int32 n)
 *           examples/vecadd/vecadd.go:6   (launched as in main_test.go:37)
 *       ReduceF32(const float* in, float* out)
 *           examples/blackwell/blackwell.go:8
 *     Each cuda.Buf[T] parameter is one 8-byte device pointer and int32 is
 *     4 bytes, the layout the reference's compiler gives them
 *     (build.go:809-820).
 *
 *  2. This shared library (libcudair_b200.so): the reference's host/ helpers
 *     (tensor maps, module loading, cuLaunchKernelEx launches) and launchers
 *     for the tuned sm_100a kernels, all behind plain C types.
 *
 * Conventions: every function returns CUDAIR_OK (0) or an error code; the
 * message of the calling thread's last error is cudair_last_error().  Device
 * pointers are passed as plain pointers / uint64_t.  A NULL stream is the
 * legacy default stream.  Calls run in the current device's primary context
 * (the context gocudrv and the CUDA runtime use), making it current when no
 * context is; a call made while another context is current returns
 * CUDAIR_ERR_UNSUPPORTED, since the library's per-device state lives in the
 * primary context.  No function allocates device memory unless its comment
 * says so; the caller owns every buffer.
 */
#ifndef CUDAIR_B200_H
#define CUDAIR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- errors ------------------------------------------------------------ */

enum {
    CUDAIR_OK = 0,
    CUDAIR_ERR_INVALID = 1,   /* argument validation failed (nothing launched) */
    CUDAIR_ERR_DRIVER = 2,    /* libcuda could not be opened / a symbol is missing */
    CUDAIR_ERR_CUDA = 3,      /* a CUDA driver or runtime call failed */
    CUDAIR_ERR_TIMEOUT = 4,   /* a bounded device-side wait gave up (see cudair_wait_status) */
    CUDAIR_ERR_UNSUPPORTED = 5 /* the device is not sm_100 */
};

/* Message of the calling thread's last failed call ("" if none).  Replaces
 * the error values of host/driver.go:108-113 and the "host: EncodeTiled: ..."
 * strings of host/tensormap.go:228-253, which it reproduces verbatim. */
const char *cudair_last_error(void);

/* Library version string. */
const char *cudair_version(void);

/* ---- tensor maps (host/tensormap.go) ----------------------------------- */

/* Enum values are CUtensorMap*'s, as in host/tensormap.go:37-108. */
enum {
    CUDAIR_TENSOR_MAP_UINT8 = 0, CUDAIR_TENSOR_MAP_UINT16 = 1,
    CUDAIR_TENSOR_MAP_UINT32 = 2, CUDAIR_TENSOR_MAP_INT32 = 3,
    CUDAIR_TENSOR_MAP_UINT64 = 4, CUDAIR_TENSOR_MAP_INT64 = 5,
    CUDAIR_TENSOR_MAP_FLOAT16 = 6, CUDAIR_TENSOR_MAP_FLOAT32 = 7,
    CUDAIR_TENSOR_MAP_FLOAT64 = 8, CUDAIR_TENSOR_MAP_BFLOAT16 = 9,
    CUDAIR_TENSOR_MAP_FLOAT32_FTZ = 10, CUDAIR_TENSOR_MAP_TFLOAT32 = 11,
    CUDAIR_TENSOR_MAP_TFLOAT32_FTZ = 12
};
enum { CUDAIR_INTERLEAVE_NONE = 0, CUDAIR_INTERLEAVE_16B = 1, CUDAIR_INTERLEAVE_32B = 2 };
enum { CUDAIR_SWIZZLE_NONE = 0, CUDAIR_SWIZZLE_32B = 1, CUDAIR_SWIZZLE_64B = 2, CUDAIR_SWIZZLE_128B = 3 };
enum { CUDAIR_L2_PROMOTION_NONE = 0, CUDAIR_L2_PROMOTION_64B = 1,
       CUDAIR_L2_PROMOTION_128B = 2, CUDAIR_L2_PROMOTION_256B = 3 };
enum { CUDAIR_OOB_FILL_NONE = 0, CUDAIR_OOB_FILL_NAN = 1 };

#define CUDAIR_TENSOR_MAP_BYTES 128

/*
 * Encodes a tiled TMA tensor map into out (128 bytes, 64-byte aligned).
 * Replaces host.EncodeTiled / host.EncodeTiledPtr (host/tensormap.go:167-224)
 * with the same validation and messages (validate, :228-253): rank 1..5,
 * n_box_dim == rank, n_global_strides == rank-1, n_element_strides == rank
 * when element_strides is non-NULL, a 16-byte aligned pointer, box entries
 * 1..256 and strides that are multiples of 16.  buffer_elem_size is the
 * element size of the buffer the pointer came from (EncodeTiled's check,
 * :171-174), or 0 to skip that check (EncodeTiledPtr).  element_strides may
 * be NULL (all 1).  The arrays are innermost dimension first.
 * Validation runs before the driver is touched, so it also works on a host
 * without a GPU.
 */
int cudair_encode_tiled(void *out, uint32_t data_type, uint32_t rank,
                        uint64_t global_address,
                        const uint64_t *global_dim,
                        const uint64_t *global_strides, uint32_t n_global_strides,
                        const uint32_t *box_dim, uint32_t n_box_dim,
                        const uint32_t *element_strides, uint32_t n_element_strides,
                        uint32_t interleave, uint32_t swizzle,
                        uint32_t l2_promotion, uint32_t oob_fill,
                        uint32_t buffer_elem_size);

/* ---- modules and attribute launches (host/launchex.go) ----------------- */

typedef struct cudair_module_s *cudair_module;
typedef struct cudair_function_s *cudair_function;

/* Loads a module image (cubin or NUL-terminated PTX) into the current
 * context.  Replaces host.LoadModule (host/launchex.go:45-70). */
int cudair_module_load(const void *image, size_t len, cudair_module *out);
/* Replaces Module.Close (host/launchex.go:73-80). */
int cudair_module_unload(cudair_module m);
/* Replaces Module.Function (host/launchex.go:83-101). */
int cudair_module_function(cudair_module m, const char *name, cudair_function *out);

/*
 * Launches f with cuLaunchKernelEx and the attributes of host.LaunchAttrs
 * (host/launchex.go:105-120, ids of :144-148): cluster_dim (NULL or all-zero
 * adds none), cooperative, programmatic stream serialisation.  params is the
 * usual void** array of pointers to each parameter's bytes.  A NULL stream
 * synchronises the context afterwards, as Function.LaunchEx does
 * (host/launchex.go:175-219).
 */
int cudair_launch_ex(cudair_function f, const uint32_t grid[3],
                     const uint32_t block[3], uint32_t shared_mem_bytes,
                     void *stream, const uint32_t cluster_dim[3],
                     int cooperative, int programmatic_stream_serialization,
                     void **params);

/* Synchronises the current context (gocudrv ctx.Synchronize). */
int cudair_ctx_synchronize(void);

/* ---- tuned launchers for the hot path ----------------------------------- */

/*
 * C = A.B + C for n x n row-major matrices: fp16 A and B, fp32 C updated in
 * place, fp32 accumulation.  Same operands as MatMul16 (hopper.go:201); this
 * launcher runs the sm_100a tcgen05/TMA kernel on a persistent grid instead
 * of the reference's one-warp-per-16x16-tile launch when n > 384: the
 * small-problem kernel (whole K panel by TMA, one 128 x 64 tile per CTA) up
 * to n = 512, the persistent CTA-pair kernels above; for n <= 384 it
 * launches the warp-per-tile kernel itself, whose latency is the lowest
 * there (n = 256: 3.5 us).  n must be a multiple of 16 (the reference's own
 * requirement) and the pointers 16-byte aligned.
 * Asynchronous on stream.
 */
int cudair_matmul16(const void *a, const void *b, float *c, int32_t n, void *stream);

/*
 * General form of the same GEMM: C (M x N, row stride ldc) += A (M x K,
 * row stride lda) . B (K x N, row stride ldb), strides in elements.  Needs
 * lda, ldb multiples of 8 and ldc a multiple of 4 (16-byte rows), 16-byte
 * aligned pointers.  M, N or K of 0 is a no-op.  Asynchronous on stream.
 */
int cudair_gemm_f16f32(const void *a, const void *b, float *c,
                       int64_t M, int64_t N, int64_t K,
                       int64_t lda, int64_t ldb, int64_t ldc, void *stream);

/*
 * The GEMM family of the reference's examples/tensor package (tensor.go:15-98:
 * MmaF16, MmaF16Bias, MmaF16Trans, MmaF16Half, MmaBF16, each an n x n matmul
 * of one warp per 16 x 8 tile) on the tuned tcgen05 kernels, for any
 * M x N x K:
 *   flags 0                      C (fp32) += A . B, as cudair_gemm_f16f32
 *   CUDAIR_GEMM_OVERWRITE        C = A . B                          (MmaF16)
 *   ... with bias != NULL        C = A . B + bias (bias M x N fp32, pitch
 *                                ldbias; copied into C, then added to)
 *                                                              (MmaF16Bias)
 *   CUDAIR_GEMM_B_T              b holds B^T: N x K row-major, pitch ldb >= K
 *                                                             (MmaF16Trans)
 *   CUDAIR_GEMM_C_F16 | OVERWRITE  C is fp16 (pitch ldc in halves): the
 *                                fp32 product rounded once to half  (MmaF16Half)
 *   CUDAIR_GEMM_BF16             A and B are bfloat16                (MmaBF16)
 * Flags combine.  A written C (OVERWRITE) needs a 16-byte aligned base and a
 * 16-byte row pitch.  MmaF16Half accumulates in half; here the sum is kept
 * in fp32 and rounded once, which is identical whenever the half sums are
 * exact (the reference's tests) and closer to the exact product otherwise.
 * Other rules as cudair_gemm_f16f32.  Asynchronous on stream.
 */
#define CUDAIR_GEMM_BF16 0x1u
#define CUDAIR_GEMM_B_T 0x2u
#define CUDAIR_GEMM_OVERWRITE 0x4u
#define CUDAIR_GEMM_C_F16 0x8u
int cudair_gemm(const void *a, const void *b, void *c, const float *bias,
                int64_t M, int64_t N, int64_t K,
                int64_t lda, int64_t ldb, int64_t ldc, int64_t ldbias,
                uint32_t flags, void *stream);

/*
 * Selects the GEMM kernel variant for subsequent calls in this process:
 * 0 = automatic (few-row kernel when M <= 64, and when M <= 128 with
 * N <= 8192, given one 128-column x 64-k unit of work per SM, in its
 * chunked form (6) for M <= 64 where the tile count fills the SMs with
 * whole waves of chunks, its stream-K form (3) otherwise; the chunked form
 * also for M <= 64 with fewer such units than SMs when K splits into at
 * least two chunks of eight 64-k blocks (narrow N, long K); the
 * small-problem kernel when K <= 512 and its 128 x 64 tiles fit one wave;
 * single CTAs with 128 x 256 tiles for the rest of M <= 128; else CTA pairs
 * with 256 x 256 or 256 x 512 tiles, whichever a makespan estimate for the
 * shape favours), 1 = single CTA, 2 = CTA pair with 256 x 256 tiles,
 * 3 = few-row kernel (M <= 128 only), 4 = CTA pair with 256 x 512 tiles,
 * 5 = small-problem kernel (K <= 512; one 128 x 64 tile of C per CTA, the
 * whole K panel loaded at once), 6 = few-row kernel with fixed k-chunks
 * handed out to the SMs at run time (M <= 64).  All variants compute the
 * same result within fp32 rounding; the choice only affects speed.
 *
 * The few-row kernel (B as the MMA's 128-row side, K split evenly over all
 * SMs) keeps its partial sums and tile counters in a 21.25 MB per-device
 * workspace that the library allocates, zeroes and synchronises on its first
 * use on a device (make that call before any stream capture).  Its calls on
 * one device must not overlap in time: issue them on one stream, or order the
 * streams with events, as with a single cuBLAS workspace.
 */
int cudair_set_gemm_variant(int variant);

/*
 * Programmatic dependent launch for the GEMM kernels (the
 * ProgrammaticStreamSerialization launch attribute of the reference's
 * host.LaunchAttrs, host/launchex.go:105-148), for chains of GEMMs on one
 * stream such as a decode step.  mode 0 (default): a plain launch.  mode 1:
 * the launch may begin while the preceding kernel in the stream finishes; the
 * kernel sets up and then waits for that kernel (griddepcontrol.wait) before
 * it reads A, B, C or its workspace.  mode 2: as 1, and the few-row kernel
 * requests the first stages of B before the wait (the square-tile kernels
 * treat it as 1).  The caller promises that the preceding kernel does not
 * write B (weights).  Results are identical in all modes.  Applies to
 * subsequent GEMM calls (cudair_gemm_f16f32, cudair_gemm, cudair_matmul16
 * above n = 512) in this process.
 */
int cudair_set_gemm_pdl(int mode);

/*
 * C = A.B + C from host buffers: the flow of the reference's MatMul16 test
 * (advanced_test.go:466-483, which copies A, B and C to the device with
 * gocudrv CopyFrom, launches MatMul16 and copies C back with CopyTo) as one
 * call.  a_host (M x K fp16, pitch lda), b_host (K x N fp16, pitch ldb) and
 * c_host (M x N fp32, pitch ldc) are host memory (page-locked for the copies
 * to overlap); b_host may be NULL when b_dev already holds B (replicated on
 * the device, e.g. by a peer copy or an all-gather over NVLink, ordered
 * before the call on `stream`).  a_dev, b_dev and c_dev are the caller's device buffers for
 * dense copies (pitches K, N and N; 16-byte aligned), so K and N must be
 * multiples of 8.  C is cut into tiles, and tile t+1 is copied in while tile
 * t is multiplied (cudair_gemm_f16f32, the automatic choice) and tile t-1 is
 * copied out, on two library-owned streams per device.  rows_per_block > 0
 * gives full-width row blocks of that many rows (rounded up to 256).  With 0,
 * B from the host, N >= 4096 and M >= 1024, C is cut into about 4 x 4 tiles:
 * B then crosses the link one column block at a time, so the first tile can
 * travel back early.  Otherwise 0 gives about 16 full-width row blocks.  The call is
 * asynchronous: `stream` waits for the last copy out, so synchronising it
 * means C is back in c_host.  Allocates nothing.
 */
int cudair_gemm_f16f32_host(const void *a_host, const void *b_host, float *c_host,
                            int64_t M, int64_t N, int64_t K,
                            int64_t lda, int64_t ldb, int64_t ldc,
                            void *a_dev, void *b_dev, float *c_dev,
                            int64_t rows_per_block, void *stream);

/*
 * MatMul16 from host buffers: the whole flow of the reference's MatMul16
 * test (advanced_test.go:466-483: CopyFrom of A, B and C, the launch, CopyTo
 * of C) as one call.  a_host, b_host (n x n fp16) and c_host (n x n fp32)
 * are host memory (page-locked for asynchronous copies); a_dev, b_dev and
 * c_dev are the caller's device buffers of the same sizes.  Up to n = 512
 * the three copies in, cudair_matmul16 and the copy out run in order on
 * `stream`; above that the call is cudair_gemm_f16f32_host.  Asynchronous:
 * once `stream` is synchronised, c_host holds C = A.B + C.  Allocates
 * nothing.
 */
int cudair_matmul16_host(const void *a_host, const void *b_host, float *c_host, int32_t n,
                         void *a_dev, void *b_dev, float *c_dev, void *stream);

/*
 * The few-row GEMM (1 <= M <= 64, N <= 524288) without any device
 * allocation.  No counterpart in the reference: it serves hosts that must not
 * allocate device memory themselves, because another allocator owns all of
 * it (a framework's caching allocator, a pool reserved at start-up) or
 * because allocating after start-up is forbidden (cudaMalloc may synchronise
 * the device and stall other streams).  Operands, layout rules and results
 * are those of cudair_gemm_f16f32 (up to fp32 rounding order).  Its scratch
 * space is a fixed 4 MiB + 16 KiB array in the library's device image, held
 * on every GPU that loads the library until exit; sizes beyond the maximum
 * return CUDAIR_ERR_INVALID.  The runtime reserves the array when it loads
 * the image on a device; under lazy module loading (the default since CUDA
 * 12.2) that is the first use, normally this entry's first call on the
 * device.  So make one call per device at start-up, before any stream
 * capture (or set CUDA_MODULE_LOADING=EAGER): that first call looks up the
 * array's address and sets the kernel's shared-memory limit, and no later
 * call reserves anything.  Every call clears the tile counters it uses and
 * then launches.  All calls share the array: calls that overlap on the GPU
 * race.
 */
int cudair_gemm_f16f32_noalloc(const void *a, const void *b, float *c,
                               int64_t M, int64_t N, int64_t K,
                               int64_t lda, int64_t ldb, int64_t ldc, void *stream);

/*
 * out[i] = a[i] + b[i] for i < n (fp32, round-to-nearest: bit-exact with a
 * CPU add).  Same operands as VecAdd (vecadd.go:6); the launcher runs one
 * block per chunk of 512 16-byte vectors, so the hardware hands chunks to SMs
 * as they finish.  Any alignment is accepted.  Asynchronous.
 */
int cudair_vecadd(const float *a, const float *b, float *out, int32_t n, void *stream);

/*
 * VecAdd from host buffers: the flow of the reference's TestVecAdd
 * (main_test.go:31-48: upload a and b, launch VecAdd, copy out back) as one
 * call.  a_host, b_host, out_host are host memory (page-locked for the copies
 * to overlap); a_dev, b_dev, out_dev are the caller's device buffers of n
 * floats.  The vectors travel in chunks of `chunk` elements (0: about
 * sixteen chunks of at least 2^20 elements; at most 64 chunks): chunk i+1 is
 * copied in on a library-owned stream while chunk i is added on `stream` and
 * chunk i-1 is copied out on another.  Asynchronous: once `stream` is
 * synchronised, out_host holds a + b, bit-exact.  Allocates nothing.
 */
int cudair_vecadd_host(const float *a_host, const float *b_host, float *out_host, int32_t n,
                       float *a_dev, float *b_dev, float *out_dev, int32_t chunk, void *stream);

/*
 * The rest of the vecadd package (vecadd.go:13-28), streamed like VecAdd in
 * chunks: y[i] = alpha * x[i] + y[i] (product and sum rounded
 * separately, as the reference's check computes them) and x[i] = x[i] * x[i]
 * in place.  Any alignment.  Asynchronous.
 */
int cudair_saxpy(float alpha, const float *x, float *y, int32_t n, void *stream);
int cudair_square(float *x, int32_t n, void *stream);

/*
 * Per-warp min and max of n floats: out[2w], out[2w+1] for warp w
 * (blackwell.go:8-17, redux.sync.{min,max}.f32).  n must be a multiple of 32.
 */
int cudair_reduce_f32(const float *in, float *out, int32_t n, void *stream);

/* ---- seeded synthetic operands -------------------------------------------- */

enum { CUDAIR_FILL_F32 = 0, CUDAIR_FILL_F16 = 1 };
enum { CUDAIR_FILL_UNIFORM = 0, CUDAIR_FILL_NORMAL = 1 };

/*
 * Writes elements offset .. offset + n - 1 of the seeded stream `seed` to
 * out (n contiguous fp32 or fp16 values, out_type CUDAIR_FILL_F32 / _F16):
 * element i comes from the word splitmix64(seed * 0x9E3779B97F4A7C15 + i)
 * alone, as
 *   CUDAIR_FILL_UNIFORM  U(p0, p1): p0 + (p1 - p0) * (w >> 40) * 2^-24 in fp32
 *   CUDAIR_FILL_NORMAL   N(p0, p1): Box-Muller on two 24-bit uniforms of w
 *                        in double, rounded to fp32
 * and, for fp16, the fp32 value rounded to nearest even.  Every step is a
 * correctly rounded IEEE operation in a fixed order (the logarithm and
 * cosine by short series), so the values are bit for bit those of the CPU
 * restatement of the same steps.  No counterpart in the reference, whose
 * tests build their inputs on the host: this generates the benchmark's and
 * the tests' seeded operands where they live, a rank's slice of a matrix
 * included (offset = its first element).  Asynchronous on stream.
 */
int cudair_fill(void *out, uint32_t out_type, uint32_t dist, int64_t n, uint64_t seed,
                int64_t offset, double p0, double p1, void *stream);

/* ---- failure detection ----------------------------------------------------- */

/*
 * Every mbarrier wait inside the library's pipelined kernels is bounded.  A
 * wait that gives up sets a bit in a device status word (which site gave up)
 * and the kernel unwinds without trapping.  cudair_wait_status synchronises
 * the current device, reads the word into *status (0 = no timeout) and, if
 * clear != 0, zeroes it.  It returns CUDAIR_ERR_TIMEOUT when a bit was set.
 */
int cudair_wait_status(uint32_t *status, int clear);

/*
 * Self-test of the bounded wait: launches one CTA that waits on an mbarrier
 * no one arrives on, with a limit of limit_ns nanoseconds.  The kernel gives
 * up, records the timeout and returns, so the context stays usable.
 */
int cudair_wait_timeout_selftest(uint64_t limit_ns, void *stream);

/* ---- multi-GPU: B replication by peer copy ----------------------------- */

#define CUDAIR_IPC_HANDLE_BYTES 64

/* Exports the device allocation holding dev_ptr for other processes
 * (cudaIpcGetMemHandle) and stores dev_ptr's byte offset inside that
 * allocation in *offset_out: the importer maps the allocation's base, so the
 * data starts at the mapped pointer + offset. */
int cudair_ipc_export(const void *dev_ptr, void *handle_out, uint64_t *offset_out);
/* Maps another process's allocation into this one (cudaIpcOpenMemHandle);
 * *dev_ptr_out is the allocation's base. */
int cudair_ipc_open(const void *handle, void **dev_ptr_out);
/* Unmaps it (cudaIpcCloseMemHandle). */
int cudair_ipc_close(void *dev_ptr);
/* Copies bytes from a peer GPU's memory into local memory over NVLink
 * (cudaMemcpyAsync device-to-device on stream).  No kernel ever reads peer
 * memory; the peer copy lands in local HBM first. */
int cudair_peer_copy(void *dst, const void *src, size_t bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* CUDAIR_B200_H */
