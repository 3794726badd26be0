"""The C-ABI library on CPU: it loads, exports every function the header
declares, and rejects bad arguments with the reference's messages before it
touches the driver (TestTensorMap/Encode, hostapi_test.go:503-535, is the
model for the tensor-map cases)."""
import ctypes

import pytest


def test_library_exports_every_header_function(cudair):
    from cudair import _lib
    names = _lib.header_functions()
    assert len(names) >= 18
    for n in names:
        assert hasattr(cudair.lib(), n), f"{n} declared in include/cudair_b200.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


# The ctypes table the Python wrapper binds must match the C declarations in
# include/cudair_b200.h parameter by parameter: pointer or scalar, and for a
# scalar its width and signedness.
_C_SCALARS = {"int": (4, "i"), "int32_t": (4, "i"), "int64_t": (8, "i"), "uint32_t": (4, "u"),
              "uint64_t": (8, "u"), "size_t": (8, "u"), "float": (4, "f"),
              "double": (8, "f")}
_C_HANDLES = {"cudair_module", "cudair_function"}  # typedef'd struct pointers


def _c_kind(decl):
    decl = decl.strip()
    if "*" in decl or "[" in decl:
        return "ptr"
    typ = decl.replace("const ", "").split()[0]
    return "ptr" if typ in _C_HANDLES else _C_SCALARS[typ]


def _ctypes_kind(ct):
    if ct in (ctypes.c_void_p, ctypes.c_char_p) or issubclass(ct, ctypes._Pointer):
        return "ptr"
    if ct is ctypes.c_float:
        return (4, "f")
    if ct is ctypes.c_double:
        return (8, "f")
    return (ctypes.sizeof(ct), "i" if ct(-1).value < 0 else "u")


def test_ctypes_signatures_match_the_header(cudair):
    import re
    from cudair import _lib
    text = re.sub(r"/\*.*?\*/", "", open(_lib.HEADER_PATH).read(), flags=re.S)
    decls = {m.group(2): (m.group(1).strip(), m.group(3))
             for m in re.finditer(r"([A-Za-z_][\w \t\*]*?)\b(cudair_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text)}
    assert set(decls) == set(_lib.SIGNATURES), set(decls) ^ set(_lib.SIGNATURES)
    for name, (ret, params) in decls.items():
        restype, argtypes = _lib.SIGNATURES[name]
        assert (ret == "int") == (restype is ctypes.c_int), name
        cparams = [] if params.strip() == "void" else [p for p in params.split(",")]
        assert len(cparams) == len(argtypes), (name, len(cparams), len(argtypes))
        for i, (cp, ct) in enumerate(zip(cparams, argtypes)):
            assert _c_kind(cp) == _ctypes_kind(ct), (name, i, cp, ct)


def test_module_image_has_reference_entry_points(cudair):
    from cudair import host
    img = host.KernelsImage()
    assert img[:4] == b"\x7fELF"
    for name in (b"MatMul16", b"VecAdd", b"ReduceF32"):
        assert name + b"\x00" in img, name


BASE = dict(GlobalDim=[64, 64], GlobalStrides=[64 * 4], BoxDim=[32, 32])
PTR = 0x7F0000000000  # a 16-byte aligned address; never dereferenced on CPU


def _encode(cudair, ptr=PTR, elem=4, **over):
    from cudair import host
    d = host.TiledTensor(DataType=host.TensorMapFloat32, **{**BASE, **over})
    return host.EncodeTiledPtr(ptr, d, _elem_size=elem)


@pytest.mark.parametrize("mutate,message", [
    (dict(GlobalStrides=[64 * 4 + 4]), "host: EncodeTiled: GlobalStrides[0] = 260, want a multiple of 16"),
    (dict(BoxDim=[512, 32]), "host: EncodeTiled: BoxDim[0] = 512, want 1..256"),
    (dict(GlobalStrides=[256, 256]), "host: EncodeTiled: 2 GlobalStrides for rank 2, want 1"),
    (dict(BoxDim=[32]), "host: EncodeTiled: 1 BoxDim for rank 2"),
    (dict(GlobalDim=[1] * 6, GlobalStrides=[16] * 5, BoxDim=[1] * 6), "host: EncodeTiled: rank 6, want 1..5"),
    (dict(ElementStrides=[1]), "host: EncodeTiled: 1 ElementStrides for rank 2"),
])
def test_encode_tiled_rejects_bad_descriptors(cudair, mutate, message):
    with pytest.raises(cudair.CudairError) as e:
        _encode(cudair, **mutate)
    assert e.value.code == 1
    assert str(e.value) == message


def test_encode_tiled_rejects_element_size_mismatch(cudair):
    from cudair import host
    d = host.TiledTensor(DataType=host.TensorMapFloat16, **BASE)
    with pytest.raises(cudair.CudairError) as e:
        host.EncodeTiledPtr(PTR, d, _elem_size=4)
    assert str(e.value) == "host: EncodeTiled: buffer element is 4 bytes, DataType is 2"


def test_encode_tiled_rejects_unaligned_pointer(cudair):
    with pytest.raises(cudair.CudairError) as e:
        _encode(cudair, ptr=PTR + 4)
    assert "is not 16-byte aligned" in str(e.value)


def test_encode_tiled_rejects_nil_buffer(cudair):
    with pytest.raises(cudair.CudairError) as e:
        _encode(cudair, ptr=0)
    assert str(e.value) == "host: EncodeTiled: nil buffer"


def test_launch_ex_rejects_nil_function_and_empty_config(cudair):
    grid = (ctypes.c_uint32 * 3)(1, 1, 1)
    block = (ctypes.c_uint32 * 3)(32, 1, 1)
    rc = cudair.lib().cudair_launch_ex(None, grid, block, 0, None, None, 0, 0, None)
    assert rc == 1 and cudair.last_error() == "host: LaunchEx: nil function"


def test_module_load_rejects_empty_image(cudair):
    m = ctypes.c_void_p()
    rc = cudair.lib().cudair_module_load(None, 0, ctypes.byref(m))
    assert rc == 1 and cudair.last_error() == "host: LoadModule: empty PTX"


def test_matmul16_rejects_n_not_multiple_of_16(cudair):
    rc = cudair.lib().cudair_matmul16(16, 16, 16, 24, None)
    assert rc == 1 and "multiple of 16" in cudair.last_error()


def test_matmul16_zero_is_noop(cudair):
    assert cudair.lib().cudair_matmul16(None, None, None, 0, None) == 0


@pytest.mark.parametrize("args,needle", [
    ((16, 16, 16, -1, 8, 8, 8, 8, 8), "negative size"),
    ((16, 16, 16, 8, 8, 8, 4, 8, 8), "leading dimensions"),
    ((16, 16, 16, 8, 8, 12, 12, 8, 8), "multiples of 8"),
    ((24, 16, 16, 8, 8, 8, 8, 8, 8), "16-byte aligned"),
    ((None, 16, 16, 8, 8, 8, 8, 8, 8), "nil pointer"),
])
def test_gemm_validation(cudair, args, needle):
    rc = cudair.lib().cudair_gemm_f16f32(*args, None)
    assert rc == 1 and needle in cudair.last_error(), cudair.last_error()


def test_gemm_empty_sizes_are_noops(cudair):
    for M, N, K in ((0, 8, 8), (8, 0, 8), (8, 8, 0)):
        assert cudair.lib().cudair_gemm_f16f32(None, None, None, M, N, K, 8, 8, 8, None) == 0


@pytest.mark.parametrize("size,lds,ptrs,rpb,needle", [
    ((16, 16, -1), (16, 16, 16), 16, 0, "negative size"),
    ((16, 16, 16), (8, 16, 16), 16, 0, "host leading dimensions"),
    ((16, 12, 16), (16, 12, 12), 16, 0, "multiples of 8"),
    ((16, 16, 16), (16, 16, 16), None, 0, "nil pointer"),
    ((16, 16, 16), (16, 16, 16), 16, -256, "rows_per_block"),
])
def test_gemm_host_validation(cudair, size, lds, ptrs, rpb, needle):
    # Argument checks come before any CUDA call, so they run without a GPU.
    M, N, K = size
    rc = cudair.lib().cudair_gemm_f16f32_host(16, 16, 16, M, N, K, *lds, 16, 16, ptrs, rpb, None)
    assert rc == 1 and needle in cudair.last_error(), cudair.last_error()


def test_gemm_host_empty_c_is_noop(cudair):
    for M, N in ((0, 8), (8, 0)):
        assert cudair.lib().cudair_gemm_f16f32_host(None, None, None, M, N, 8, 8, 8, 8,
                                                    None, None, None, 0, None) == 0


def test_gemm_pdl_mode_validation(cudair):
    L = cudair.lib()
    assert L.cudair_set_gemm_pdl(3) == 1 and "PDL mode 3" in cudair.last_error()
    assert L.cudair_set_gemm_pdl(-1) == 1
    for mode in (2, 1, 0):
        assert L.cudair_set_gemm_pdl(mode) == 0


@pytest.mark.parametrize("flags,bias,c,ldc,needle", [
    (0x8, None, 16, 16, "needs CUDAIR_GEMM_OVERWRITE"),
    (0x10, None, 16, 16, "unknown flags"),
    (0x0, 16, 16, 16, "a bias needs"),
    (0xC, 16, 16, 16, "a bias needs"),
    (0x4, None, 20, 16, "16-byte aligned"),
    (0x4, None, 16, 18, "16-byte aligned"),
    (0x2, None, 16, 16, "leading dimensions"),
])
def test_gemm_family_validation(cudair, flags, bias, c, ldc, needle):
    # M = N = 16, K = 32: with B^T (flag 0x2) ldb = 16 < K is too small.
    rc = cudair.lib().cudair_gemm(16, 16, c, bias, 16, 16, 32, 32, 16, ldc, 16, flags, None)
    assert rc == 1 and needle in cudair.last_error(), cudair.last_error()


def test_vecadd_and_reduce_validation(cudair):
    L = cudair.lib()
    assert L.cudair_vecadd(None, None, None, -1, None) == 1
    assert L.cudair_vecadd(None, None, None, 0, None) == 0
    assert L.cudair_reduce_f32(16, 16, 33, None) == 1
    assert "multiple of 32" in cudair.last_error()


def test_saxpy_and_square_validation(cudair):
    L = cudair.lib()
    assert L.cudair_saxpy(2.0, None, None, -1, None) == 1
    assert "Saxpy: n = -1" in cudair.last_error()
    assert L.cudair_saxpy(2.0, None, None, 0, None) == 0
    assert L.cudair_saxpy(2.0, None, None, 16, None) == 1
    assert "Saxpy: nil pointer" in cudair.last_error()
    assert L.cudair_square(None, -1, None) == 1
    assert "Square: n = -1" in cudair.last_error()
    assert L.cudair_square(None, 0, None) == 0
    assert L.cudair_square(None, 16, None) == 1
    assert "Square: nil pointer" in cudair.last_error()


def test_host_entries_validation(cudair):
    L = cudair.lib()
    assert L.cudair_vecadd_host(None, None, None, -1, None, None, None, 0, None) == 1
    assert L.cudair_vecadd_host(None, None, None, 16, None, None, None, -1, None) == 1
    assert L.cudair_vecadd_host(None, None, None, 0, None, None, None, 0, None) == 0
    assert L.cudair_vecadd_host(None, None, None, 16, None, None, None, 0, None) == 1
    assert "vecadd_host: nil pointer" in cudair.last_error()
    assert L.cudair_matmul16_host(None, None, None, 24, None, None, None, None) == 1
    assert "multiple of 16" in cudair.last_error()
    assert L.cudair_matmul16_host(None, None, None, 0, None, None, None, None) == 0
    assert L.cudair_matmul16_host(None, None, None, 32, None, None, None, None) == 1
    assert "matmul16_host: nil pointer" in cudair.last_error()


def test_fill_validation(cudair):
    # Checked before the device is touched.
    L = cudair.lib()
    assert L.cudair_fill(None, 2, 0, 4, 1, 0, 0.0, 1.0, None) == 1
    assert "output type 2" in cudair.last_error()
    assert L.cudair_fill(None, 0, 5, 4, 1, 0, 0.0, 1.0, None) == 1
    assert "distribution 5" in cudair.last_error()
    assert L.cudair_fill(None, 0, 0, -1, 1, 0, 0.0, 1.0, None) == 1
    assert L.cudair_fill(None, 1, 1, 4, 1, -3, 0.0, 1.0, None) == 1
    assert L.cudair_fill(None, 0, 0, 0, 1, 0, 0.0, 1.0, None) == 0
    assert L.cudair_fill(None, 0, 0, 4, 1, 0, 0.0, 1.0, None) == 1
    assert "nil pointer" in cudair.last_error()
    assert L.cudair_fill(18, 0, 0, 4, 1, 0, 0.0, 1.0, None) == 1
    assert "aligned" in cudair.last_error()


# The no-alloc few-row entry checks its arguments before it touches the
# device: sizes beyond its fixed scratch array, pitches and alignment.
@pytest.mark.parametrize("M,N,K,lda,ldb,ldc,ptr,needle", [
    (-1, 16, 16, 16, 16, 16, 256, "negative size"),
    (65, 16, 16, 16, 16, 16, 256, "exceeds the maximum of 64 rows"),
    (16, 4096 * 128 + 8, 16, 16, 4096 * 128 + 8, 4096 * 128 + 8, 256, "columns"),
    (16, 16, 16, 8, 16, 16, 256, "too small"),
    (16, 16, 12, 12, 16, 16, 256, "multiples of 8"),
    (16, 16, 16, 16, 16, 16, 264, "16-byte aligned"),
    (16, 16, 16, 16, 16, 16, 0, "nil pointer"),
])
def test_noalloc_validation(cudair, M, N, K, lda, ldb, ldc, ptr, needle):
    rc = cudair.lib().cudair_gemm_f16f32_noalloc(ptr, ptr, ptr, M, N, K, lda, ldb, ldc, None)
    assert rc == 1 and needle in cudair.last_error(), cudair.last_error()


def test_noalloc_empty_sizes_are_noops(cudair):
    L = cudair.lib()
    for M, N, K in ((0, 16, 16), (16, 0, 16), (16, 16, 0)):
        assert L.cudair_gemm_f16f32_noalloc(None, None, None, M, N, K, 16, 16, 16, None) == 0


def test_errors_are_thread_local(cudair):
    import threading
    L = cudair.lib()
    L.cudair_vecadd(None, None, None, -1, None)
    seen = []

    def other():
        seen.append(cudair.last_error())

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen == [""]
    assert "VecAdd" in cudair.last_error()
