// driver.cpp - error reporting and the run-time binding of the CUDA driver
// entry points the library calls directly.
//
// Follows the reference's host/driver.go: the driver library is opened once
// (loadDriver, driver.go:69-91) from the same candidate paths
// (driver_notwindows.go:15-19), a missing symbol becomes an error rather than
// a crash (register, driver.go:96-104), and a failing CUresult is reported
// with the call's name (check, driver.go:108-113).
#include <dlfcn.h>
#include <stdarg.h>
#include <stdio.h>

#include <mutex>
#include <string>

#include "cudair_internal.h"

namespace cudair {

namespace {
thread_local std::string t_last_error;
}

void clear_error() { t_last_error.clear(); }

int set_error(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int cuda_error(cudaError_t e, const char *op) {
    return set_error(CUDAIR_ERR_CUDA, "%s: %s (%s)", op, cudaGetErrorName(e),
                     cudaGetErrorString(e));
}

namespace {

const char *const kDriverCandidates[] = {
    "libcuda.so.1",
    "/usr/lib/x86_64-linux-gnu/libcuda.so.1",
    "/usr/lib/wsl/lib/libcuda.so.1",
};

std::once_flag g_once;
Driver g_drv;
int g_drv_rc = CUDAIR_OK;
std::string g_drv_err;

template <class F>
bool bind(void *h, F &fp, const char *name) {
    void *s = dlsym(h, name);
    if (!s) {
        g_drv_rc = CUDAIR_ERR_DRIVER;
        g_drv_err = std::string("host: bind ") + name + ": symbol not found (CUDA driver too old?)";
        return false;
    }
    fp = reinterpret_cast<F>(s);
    return true;
}

void open_driver() {
    void *h = nullptr;
    std::string errs;
    for (const char *p : kDriverCandidates) {
        h = dlopen(p, RTLD_NOW | RTLD_GLOBAL);
        if (h) break;
        const char *e = dlerror();
        if (!errs.empty()) errs += "; ";
        errs += std::string(p) + ": " + (e ? e : "dlopen failed");
    }
    if (!h) {
        g_drv_rc = CUDAIR_ERR_DRIVER;
        g_drv_err = "host: open CUDA driver: " + errs;
        return;
    }
    bind(h, g_drv.cuInit, "cuInit") && bind(h, g_drv.cuGetErrorName, "cuGetErrorName") &&
        bind(h, g_drv.cuGetErrorString, "cuGetErrorString") &&
        bind(h, g_drv.cuCtxGetCurrent, "cuCtxGetCurrent") &&
        bind(h, g_drv.cuCtxSetCurrent, "cuCtxSetCurrent") &&
        bind(h, g_drv.cuCtxSynchronize, "cuCtxSynchronize") &&
        bind(h, g_drv.cuDevicePrimaryCtxRetain, "cuDevicePrimaryCtxRetain") &&
        bind(h, g_drv.cuModuleLoadData, "cuModuleLoadData") &&
        bind(h, g_drv.cuModuleUnload, "cuModuleUnload") &&
        bind(h, g_drv.cuModuleGetFunction, "cuModuleGetFunction") &&
        bind(h, g_drv.cuLaunchKernelEx, "cuLaunchKernelEx") &&
        bind(h, g_drv.cuMemGetAddressRange, "cuMemGetAddressRange_v2") &&
        bind(h, g_drv.cuTensorMapEncodeTiled, "cuTensorMapEncodeTiled");
    if (g_drv_rc == CUDAIR_OK) {
        CUresult r = g_drv.cuInit(0);
        if (r != CUDA_SUCCESS) {
            g_drv_rc = CUDAIR_ERR_DRIVER;
            g_drv_err = "host: cuInit failed with CUresult " + std::to_string(static_cast<int>(r));
        }
    }
}

}  // namespace

int load_driver(const Driver **out) {
    std::call_once(g_once, open_driver);
    if (g_drv_rc != CUDAIR_OK) return set_error(g_drv_rc, "%s", g_drv_err.c_str());
    *out = &g_drv;
    return CUDAIR_OK;
}

int cu_error(CUresult r, const char *op) {
    const char *name = "CUDA_ERROR_UNKNOWN", *text = "";
    if (g_drv.cuGetErrorName) g_drv.cuGetErrorName(r, &name);
    if (g_drv.cuGetErrorString) g_drv.cuGetErrorString(r, &text);
    return set_error(CUDAIR_ERR_CUDA, "%s: %s (%s)", op, name ? name : "?", text ? text : "");
}

int ensure_context() {
    const Driver *d = nullptr;
    int rc = load_driver(&d);
    if (rc != CUDAIR_OK) return rc;
    CUcontext c = nullptr;
    CUresult r = d->cuCtxGetCurrent(&c);
    if (r != CUDA_SUCCESS) return cu_error(r, "cuCtxGetCurrent");
    if (c) return CUDAIR_OK;
    cudaError_t e = cudaFree(nullptr);  // makes the primary context current
    if (e != cudaSuccess) return cuda_error(e, "cudaFree(0)");
    return CUDAIR_OK;
}

}  // namespace cudair

CUDAIR_API const char *cudair_last_error(void) { return cudair::t_last_error.c_str(); }

CUDAIR_API const char *cudair_version(void) { return "cudair-b200 0.1.0 (sm_100a)"; }

CUDAIR_API int cudair_ctx_synchronize(void) {
    using namespace cudair;
    clear_error();
    const Driver *d = nullptr;
    int rc = load_driver(&d);
    if (rc != CUDAIR_OK) return rc;
    if ((rc = ensure_context()) != CUDAIR_OK) return rc;
    CUresult r = d->cuCtxSynchronize();
    if (r != CUDA_SUCCESS) return cu_error(r, "cuCtxSynchronize");
    return CUDAIR_OK;
}
