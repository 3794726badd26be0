/*
 * A C caller of libcudair_b200.so, the way a host program in any language
 * binds the C ABI (a Go program through purego does the same dlopen/dlsym):
 * the MatMul16 test flow of advanced_test.go:456-483 (n = 64 and 256, the
 * reference's integer generator, an exact comparison with a CPU loop) through
 * cudair_gemm_f16f32_host, the tuned kernel on device buffers
 * (cudair_matmul16), VecAdd on the 2^20 ramp of main_test.go:26-60, and the
 * error path.  Prints "ok" and exits 0 on success.
 *
 *   gcc -O2 matmul16_client.c -o matmul16_client -ldl -lcudart -L<cuda lib>
 *   ./matmul16_client path/to/libcudair_b200.so
 */
#include <dlfcn.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

typedef int (*gemm_host_fn)(const void *, const void *, float *, int64_t, int64_t, int64_t, int64_t,
                            int64_t, int64_t, void *, void *, float *, int64_t, void *);
typedef int (*matmul16_fn)(const void *, const void *, float *, int32_t, void *);
typedef int (*vecadd_fn)(const float *, const float *, float *, int32_t, void *);
typedef const char *(*last_error_fn)(void);
typedef const char *(*version_fn)(void);

static last_error_fn last_error;

#define CHECK(cond, ...)                      \
    do {                                      \
        if (!(cond)) {                        \
            fprintf(stderr, __VA_ARGS__);     \
            fprintf(stderr, "\n");            \
            exit(1);                          \
        }                                     \
    } while (0)

/* Small integers (|x| <= 3) are exact in half: sign, exponent, mantissa. */
static uint16_t half_of_small_int(int v) {
    if (v == 0) return 0;
    uint16_t sign = v < 0 ? 0x8000u : 0;
    unsigned a = (unsigned)(v < 0 ? -v : v);
    int e = 0;
    while ((a >> e) > 1) ++e;
    uint16_t mant = (uint16_t)(((a << (10 - e)) & 0x3FFu));
    return (uint16_t)(sign | ((uint16_t)(e + 15) << 10) | mant);
}

static void run_matmul16(int n, gemm_host_fn gemm_host, matmul16_fn matmul16) {
    size_t nn = (size_t)n * n;
    uint16_t *a = malloc(nn * 2), *b = malloc(nn * 2);
    float *c = malloc(nn * 4), *c2 = malloc(nn * 4), *want = malloc(nn * 4);
    CHECK(a && b && c && c2 && want, "out of memory");
    /* advanced_test.go:459-463: af = (i+2j)%7-3, bf = (3i+j)%5-2, c = j-i */
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < n; ++j) {
            a[(size_t)i * n + j] = half_of_small_int((i + 2 * j) % 7 - 3);
            b[(size_t)i * n + j] = half_of_small_int((3 * i + j) % 5 - 2);
            c[(size_t)i * n + j] = c2[(size_t)i * n + j] = (float)(j - i);
        }
    /* The reference's CPU model: want[i][j] = c[i][j] + sum_k af[i][k] bf[k][j]. */
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < n; ++j) {
            float s = (float)(j - i);
            for (int k = 0; k < n; ++k) s += (float)((i + 2 * k) % 7 - 3) * (float)((3 * k + j) % 5 - 2);
            want[(size_t)i * n + j] = s;
        }
    void *da, *db, *dc;
    CHECK(cudaMalloc(&da, nn * 2) == cudaSuccess && cudaMalloc(&db, nn * 2) == cudaSuccess &&
              cudaMalloc(&dc, nn * 4) == cudaSuccess,
          "cudaMalloc failed");
    /* 1: host buffers in, C back in host memory. */
    int rc = gemm_host(a, b, c, n, n, n, n, n, n, da, db, dc, 0, NULL);
    CHECK(rc == 0, "cudair_gemm_f16f32_host: %s", last_error());
    CHECK(cudaDeviceSynchronize() == cudaSuccess, "sync failed");
    for (size_t i = 0; i < nn; ++i) CHECK(c[i] == want[i], "gemm_host n=%d: C[%zu] = %g, want %g", n, i, c[i], want[i]);
    /* 2: the tuned MatMul16 on device buffers the caller filled. */
    CHECK(cudaMemcpy(dc, c2, nn * 4, cudaMemcpyHostToDevice) == cudaSuccess, "copy failed");
    rc = matmul16(da, db, (float *)dc, n, NULL);
    CHECK(rc == 0, "cudair_matmul16: %s", last_error());
    CHECK(cudaMemcpy(c2, dc, nn * 4, cudaMemcpyDeviceToHost) == cudaSuccess, "copy back failed");
    for (size_t i = 0; i < nn; ++i) CHECK(c2[i] == want[i], "matmul16 n=%d: C[%zu] = %g, want %g", n, i, c2[i], want[i]);
    cudaFree(da);
    cudaFree(db);
    cudaFree(dc);
    free(a), free(b), free(c), free(c2), free(want);
}

int main(int argc, char **argv) {
    CHECK(argc == 2, "usage: %s libcudair_b200.so", argv[0]);
    void *h = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
    CHECK(h, "dlopen: %s", dlerror());
    last_error = (last_error_fn)dlsym(h, "cudair_last_error");
    version_fn version = (version_fn)dlsym(h, "cudair_version");
    gemm_host_fn gemm_host = (gemm_host_fn)dlsym(h, "cudair_gemm_f16f32_host");
    matmul16_fn matmul16 = (matmul16_fn)dlsym(h, "cudair_matmul16");
    vecadd_fn vecadd = (vecadd_fn)dlsym(h, "cudair_vecadd");
    CHECK(last_error && version && gemm_host && matmul16 && vecadd, "missing symbol: %s", dlerror());
    printf("%s\n", version());

    run_matmul16(64, gemm_host, matmul16);
    run_matmul16(256, gemm_host, matmul16);

    /* VecAdd on the 2^20 ramp of main_test.go:26-60: a = 0.5 i, b = 1000 - i. */
    const int vn = 1 << 20;
    float *va = malloc((size_t)vn * 4), *vb = malloc((size_t)vn * 4), *vo = malloc((size_t)vn * 4);
    CHECK(va && vb && vo, "out of memory");
    for (int i = 0; i < vn; ++i) va[i] = 0.5f * (float)i, vb[i] = 1000.0f - (float)i;
    float *dva, *dvb, *dvo;
    CHECK(cudaMalloc((void **)&dva, (size_t)vn * 4) == cudaSuccess &&
              cudaMalloc((void **)&dvb, (size_t)vn * 4) == cudaSuccess &&
              cudaMalloc((void **)&dvo, (size_t)vn * 4) == cudaSuccess,
          "cudaMalloc failed");
    cudaMemcpy(dva, va, (size_t)vn * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dvb, vb, (size_t)vn * 4, cudaMemcpyHostToDevice);
    CHECK(vecadd(dva, dvb, dvo, vn, NULL) == 0, "cudair_vecadd: %s", last_error());
    CHECK(cudaMemcpy(vo, dvo, (size_t)vn * 4, cudaMemcpyDeviceToHost) == cudaSuccess, "copy back failed");
    for (int i = 0; i < vn; ++i) CHECK(vo[i] == va[i] + vb[i], "VecAdd: out[%d] = %g", i, vo[i]);

    /* The error path: a thread-local message, no crash. */
    CHECK(matmul16(dva, dvb, dvo, 17, NULL) != 0, "n = 17 accepted");
    CHECK(strstr(last_error(), "multiple of 16") != NULL, "message: %s", last_error());

    cudaFree(dva), cudaFree(dvb), cudaFree(dvo);
    free(va), free(vb), free(vo);
    printf("ok\n");
    return 0;
}
