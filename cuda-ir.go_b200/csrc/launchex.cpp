// launchex.cpp - loading a kernel module and launching its entry points with
// cuLaunchKernelEx launch attributes: the C-ABI counterpart of the
// reference's host/launchex.go (LoadModule :45, Close :73, Function :83,
// LaunchAttrs :105-120, LaunchExOn :184-219).
#include <string.h>

#include <string>

#include "cudair_internal.h"

struct cudair_module_s {
    CUmodule raw;
};

struct cudair_function_s {
    CUfunction raw;
    std::string name;
};

CUDAIR_API int cudair_module_load(const void *image, size_t len, cudair_module *out) {
    using namespace cudair;
    clear_error();
    if (out == nullptr) return set_error(CUDAIR_ERR_INVALID, "host: LoadModule: nil output");
    *out = nullptr;
    if (image == nullptr || len == 0)
        return set_error(CUDAIR_ERR_INVALID, "host: LoadModule: empty PTX");
    const Driver *d = nullptr;
    int rc = load_driver(&d);
    if (rc != CUDAIR_OK) return rc;
    if ((rc = ensure_context()) != CUDAIR_OK) return rc;
    // cuModuleLoadData wants a NUL-terminated string for PTX text
    // (host/launchex.go:52-55); a cubin/fatbin image is passed as is.
    std::string copy;
    const void *img = image;
    const unsigned char *bytes = static_cast<const unsigned char *>(image);
    const bool is_elf = len >= 4 && bytes[0] == 0x7f && bytes[1] == 'E' && bytes[2] == 'L' && bytes[3] == 'F';
    if (!is_elf && bytes[len - 1] != 0) {
        copy.assign(static_cast<const char *>(image), len);
        img = copy.c_str();
    }
    CUmodule m = nullptr;
    CUresult r = d->cuModuleLoadData(&m, img);
    if (r != CUDA_SUCCESS) return cu_error(r, "host: LoadModule: cuModuleLoadData");
    *out = new cudair_module_s{m};
    return CUDAIR_OK;
}

CUDAIR_API int cudair_module_unload(cudair_module m) {
    using namespace cudair;
    clear_error();
    if (m == nullptr || m->raw == nullptr) return CUDAIR_OK;
    const Driver *d = nullptr;
    int rc = load_driver(&d);
    if (rc != CUDAIR_OK) return rc;
    CUmodule raw = m->raw;
    m->raw = nullptr;
    delete m;
    CUresult r = d->cuModuleUnload(raw);
    if (r != CUDA_SUCCESS) return cu_error(r, "cuModuleUnload");
    return CUDAIR_OK;
}

CUDAIR_API int cudair_module_function(cudair_module m, const char *name, cudair_function *out) {
    using namespace cudair;
    clear_error();
    if (out == nullptr) return set_error(CUDAIR_ERR_INVALID, "host: Function: nil output");
    *out = nullptr;
    if (m == nullptr || m->raw == nullptr)
        return set_error(CUDAIR_ERR_INVALID, "host: Function: module is closed");
    if (name == nullptr) return set_error(CUDAIR_ERR_INVALID, "host: Function: nil name");
    const Driver *d = nullptr;
    int rc = load_driver(&d);
    if (rc != CUDAIR_OK) return rc;
    CUfunction f = nullptr;
    CUresult r = d->cuModuleGetFunction(&f, m->raw, name);
    if (r != CUDA_SUCCESS) {
        std::string op = std::string("host: Function ") + name + ": cuModuleGetFunction";
        return cu_error(r, op.c_str());
    }
    *out = new cudair_function_s{f, name};
    return CUDAIR_OK;
}

CUDAIR_API int cudair_launch_ex(cudair_function f, const uint32_t grid[3], const uint32_t block[3],
                                uint32_t shared_mem_bytes, void *stream,
                                const uint32_t cluster_dim[3], int cooperative,
                                int programmatic_stream_serialization, void **params) {
    using namespace cudair;
    clear_error();
    if (f == nullptr || f->raw == nullptr)
        return set_error(CUDAIR_ERR_INVALID, "host: LaunchEx: nil function");
    if (grid == nullptr || block == nullptr || grid[0] == 0 || block[0] == 0)
        return set_error(CUDAIR_ERR_INVALID, "host: LaunchEx %s: empty launch config",
                         f->name.c_str());
    const Driver *d = nullptr;
    int rc = load_driver(&d);
    if (rc != CUDAIR_OK) return rc;
    if ((rc = ensure_context()) != CUDAIR_OK) return rc;

    auto max1 = [](uint32_t v) { return v == 0 ? 1u : v; };
    // The attribute array of LaunchAttrs.attributes (host/launchex.go:152-173):
    // cluster shape (id 4), cooperative (id 2), programmatic stream
    // serialisation (id 6).
    CUlaunchAttribute attrs[3];
    memset(attrs, 0, sizeof(attrs));
    unsigned n_attrs = 0;
    if (cluster_dim != nullptr && (cluster_dim[0] | cluster_dim[1] | cluster_dim[2]) != 0) {
        attrs[n_attrs].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
        attrs[n_attrs].value.clusterDim.x = cluster_dim[0];
        attrs[n_attrs].value.clusterDim.y = cluster_dim[1];
        attrs[n_attrs].value.clusterDim.z = cluster_dim[2];
        ++n_attrs;
    }
    if (cooperative) {
        attrs[n_attrs].id = CU_LAUNCH_ATTRIBUTE_COOPERATIVE;
        attrs[n_attrs].value.cooperative = 1;
        ++n_attrs;
    }
    if (programmatic_stream_serialization) {
        attrs[n_attrs].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
        attrs[n_attrs].value.programmaticStreamSerializationAllowed = 1;
        ++n_attrs;
    }
    CUlaunchConfig cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDimX = grid[0];
    cfg.gridDimY = max1(grid[1]);
    cfg.gridDimZ = max1(grid[2]);
    cfg.blockDimX = block[0];
    cfg.blockDimY = max1(block[1]);
    cfg.blockDimZ = max1(block[2]);
    cfg.sharedMemBytes = shared_mem_bytes;
    cfg.hStream = static_cast<CUstream>(stream);
    cfg.attrs = n_attrs ? attrs : nullptr;
    cfg.numAttrs = n_attrs;

    std::string op = "host: LaunchEx " + f->name + ": cuLaunchKernelEx";
    CUresult r = d->cuLaunchKernelEx(&cfg, f->raw, params, nullptr);
    if (r != CUDA_SUCCESS) return cu_error(r, op.c_str());
    if (stream == nullptr) {
        // A nil stream waits for the context, as Function.LaunchEx does.
        r = d->cuCtxSynchronize();
        if (r != CUDA_SUCCESS) {
            op = "host: LaunchEx " + f->name + ": cuCtxSynchronize";
            return cu_error(r, op.c_str());
        }
    }
    return CUDAIR_OK;
}
