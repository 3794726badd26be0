// tensormap.cpp - TMA tensor maps: the C-ABI counterpart of the reference's
// host.EncodeTiled / EncodeTiledPtr (host/tensormap.go:165-253).
//
// The validation rules and their messages are the reference's, because the
// driver reports all of them only as CUDA_ERROR_INVALID_VALUE.  The checks
// run before the driver is opened, so a caller without a GPU still gets the
// precise message.
#include <string.h>

#include "cudair_internal.h"

namespace cudair {

namespace {

// Element size of a CUtensorMapDataType; 0 for an unknown type
// (TensorMapDataType.size, host/tensormap.go:54-67).
int data_type_size(uint32_t t) {
    switch (t) {
    case CUDAIR_TENSOR_MAP_UINT8:
        return 1;
    case CUDAIR_TENSOR_MAP_UINT16:
    case CUDAIR_TENSOR_MAP_FLOAT16:
    case CUDAIR_TENSOR_MAP_BFLOAT16:
        return 2;
    case CUDAIR_TENSOR_MAP_UINT32:
    case CUDAIR_TENSOR_MAP_INT32:
    case CUDAIR_TENSOR_MAP_FLOAT32:
    case CUDAIR_TENSOR_MAP_FLOAT32_FTZ:
    case CUDAIR_TENSOR_MAP_TFLOAT32:
    case CUDAIR_TENSOR_MAP_TFLOAT32_FTZ:
        return 4;
    case CUDAIR_TENSOR_MAP_UINT64:
    case CUDAIR_TENSOR_MAP_INT64:
    case CUDAIR_TENSOR_MAP_FLOAT64:
        return 8;
    }
    return 0;
}

// TiledTensor.validate (host/tensormap.go:228-253).
int validate(uint32_t rank, uint64_t ptr, const uint64_t *global_strides,
             uint32_t n_global_strides, const uint32_t *box_dim, uint32_t n_box_dim,
             const uint32_t *element_strides, uint32_t n_element_strides) {
    if (rank < 1 || rank > 5)
        return set_error(CUDAIR_ERR_INVALID, "host: EncodeTiled: rank %u, want 1..5", rank);
    if (n_box_dim != rank)
        return set_error(CUDAIR_ERR_INVALID, "host: EncodeTiled: %u BoxDim for rank %u", n_box_dim,
                         rank);
    if (n_global_strides != rank - 1)
        return set_error(CUDAIR_ERR_INVALID,
                         "host: EncodeTiled: %u GlobalStrides for rank %u, want %u",
                         n_global_strides, rank, rank - 1);
    if (element_strides != nullptr && n_element_strides != rank)
        return set_error(CUDAIR_ERR_INVALID, "host: EncodeTiled: %u ElementStrides for rank %u",
                         n_element_strides, rank);
    if (ptr % 16 != 0)
        return set_error(CUDAIR_ERR_INVALID,
                         "host: EncodeTiled: device pointer %#llx is not 16-byte aligned",
                         static_cast<unsigned long long>(ptr));
    for (uint32_t i = 0; i < n_box_dim; ++i)
        if (box_dim[i] < 1 || box_dim[i] > 256)
            return set_error(CUDAIR_ERR_INVALID, "host: EncodeTiled: BoxDim[%u] = %u, want 1..256",
                             i, box_dim[i]);
    for (uint32_t i = 0; i < n_global_strides; ++i)
        if (global_strides[i] % 16 != 0)
            return set_error(CUDAIR_ERR_INVALID,
                             "host: EncodeTiled: GlobalStrides[%u] = %llu, want a multiple of 16",
                             i, static_cast<unsigned long long>(global_strides[i]));
    return CUDAIR_OK;
}

}  // namespace

int encode_tiled_internal(CUtensorMap *out, uint32_t data_type, uint32_t rank,
                          uint64_t global_address, const uint64_t *global_dim,
                          const uint64_t *global_strides, const uint32_t *box_dim,
                          const uint32_t *element_strides, uint32_t interleave, uint32_t swizzle,
                          uint32_t l2_promotion, uint32_t oob_fill) {
    const Driver *d = nullptr;
    int rc = load_driver(&d);
    if (rc != CUDAIR_OK) return rc;
    cuuint32_t ones[5] = {1, 1, 1, 1, 1};
    // A rank-1 tensor has no strides; the driver ignores the pointer then
    // (host/tensormap.go:196-201).
    cuuint64_t zero_stride[1] = {0};
    CUresult r = d->cuTensorMapEncodeTiled(
        out, static_cast<CUtensorMapDataType>(data_type), rank,
        reinterpret_cast<void *>(global_address), global_dim,
        rank > 1 ? global_strides : zero_stride, box_dim,
        element_strides ? element_strides : ones, static_cast<CUtensorMapInterleave>(interleave),
        static_cast<CUtensorMapSwizzle>(swizzle), static_cast<CUtensorMapL2promotion>(l2_promotion),
        static_cast<CUtensorMapFloatOOBfill>(oob_fill));
    if (r != CUDA_SUCCESS) return cu_error(r, "cuTensorMapEncodeTiled");
    return CUDAIR_OK;
}

}  // namespace cudair

CUDAIR_API int cudair_encode_tiled(void *out, uint32_t data_type, uint32_t rank,
                                   uint64_t global_address, const uint64_t *global_dim,
                                   const uint64_t *global_strides, uint32_t n_global_strides,
                                   const uint32_t *box_dim, uint32_t n_box_dim,
                                   const uint32_t *element_strides, uint32_t n_element_strides,
                                   uint32_t interleave, uint32_t swizzle, uint32_t l2_promotion,
                                   uint32_t oob_fill, uint32_t buffer_elem_size) {
    using namespace cudair;
    clear_error();
    if (out == nullptr) return set_error(CUDAIR_ERR_INVALID, "host: EncodeTiled: nil output");
    if (reinterpret_cast<uintptr_t>(out) % 64 != 0)
        return set_error(CUDAIR_ERR_INVALID,
                         "host: EncodeTiled: output descriptor is not 64-byte aligned");
    if (global_address == 0) return set_error(CUDAIR_ERR_INVALID, "host: EncodeTiled: nil buffer");
    // EncodeTiled's element-size check (host/tensormap.go:171-174).
    const int want = data_type_size(data_type);
    if (buffer_elem_size != 0 && want != 0 && static_cast<int>(buffer_elem_size) != want)
        return set_error(CUDAIR_ERR_INVALID,
                         "host: EncodeTiled: buffer element is %u bytes, DataType is %d",
                         buffer_elem_size, want);
    if (global_dim == nullptr || box_dim == nullptr ||
        (n_global_strides > 0 && global_strides == nullptr))
        return set_error(CUDAIR_ERR_INVALID, "host: EncodeTiled: nil dimension array");
    int rc = validate(rank, global_address, global_strides, n_global_strides, box_dim, n_box_dim,
                      element_strides, n_element_strides);
    if (rc != CUDAIR_OK) return rc;
    alignas(64) CUtensorMap m;
    memset(&m, 0, sizeof(m));
    rc = encode_tiled_internal(&m, data_type, rank, global_address, global_dim, global_strides,
                               box_dim, element_strides, interleave, swizzle, l2_promotion,
                               oob_fill);
    if (rc != CUDAIR_OK) return rc;
    memcpy(out, &m, sizeof(m));
    return CUDAIR_OK;
}
