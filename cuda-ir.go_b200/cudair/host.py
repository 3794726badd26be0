"""Python mirror of the reference's host/ package (tensor maps, modules,
attribute launches) over the C ABI of libcudair_b200.so.

Names, argument meaning and errors follow the Go API so a test reads like the
reference's own:

    Go (host/)                              here
    host.TiledTensor{...}                   TiledTensor(...)
    host.EncodeTiled(ctx, buf, d)           EncodeTiled(buf, d)      buf: torch tensor
    host.EncodeTiledPtr(ctx, ptr, d)        EncodeTiledPtr(ptr, d)
    TensorMap.Bytes() / Arg() / ArgEx()     TensorMap.Bytes() / Arg() / ArgEx()
    host.LoadModule(ctx, ptx)               LoadModule(image)
    Module.Function(name) / Close()         Module.Function(name) / Close()
    Function.LaunchEx(cfg, attrs, args...)  Function.LaunchEx(cfg, attrs, *args)
    Function.LaunchExOn(stream, ...)        Function.LaunchExOn(stream, ...)
    host.LaunchAttrs{ClusterDim, ...}       LaunchAttrs(ClusterDim=..., ...)
    host.ArgValue / ArgBuffer / ArgBytes    ArgValue / ArgBuffer / ArgBytes
    cuda.LaunchConfig / LaunchConfig1D      LaunchConfig / LaunchConfig1D

The Go context argument has no counterpart: calls use the CUDA context
current on the calling thread (torch's, i.e. the device's primary context).
Every failure raises CudairError carrying the library's message.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional, Sequence

from ._lib import CUBIN_PATH, CudairError, check, lib

# ---- tensor maps (host/tensormap.go:37-108) -----------------------------------

TensorMapUint8, TensorMapUint16, TensorMapUint32, TensorMapInt32 = 0, 1, 2, 3
TensorMapUint64, TensorMapInt64, TensorMapFloat16, TensorMapFloat32 = 4, 5, 6, 7
TensorMapFloat64, TensorMapBFloat16, TensorMapFloat32FTZ = 8, 9, 10
TensorMapTFloat32, TensorMapTF32FTZ = 11, 12

InterleaveNone, Interleave16B, Interleave32B = 0, 1, 2
SwizzleNone, Swizzle32B, Swizzle64B, Swizzle128B = 0, 1, 2, 3
L2PromotionNone, L2Promotion64B, L2Promotion128B, L2Promotion256B = 0, 1, 2, 3
OOBFillNone, OOBFillNaN = 0, 1

TENSOR_MAP_BYTES = 128


@dataclass
class TiledTensor:
    """host.TiledTensor (host/tensormap.go:113-132); dimensions innermost first."""
    DataType: int
    GlobalDim: Sequence[int]
    GlobalStrides: Sequence[int]
    BoxDim: Sequence[int]
    ElementStrides: Optional[Sequence[int]] = None
    Interleave: int = InterleaveNone
    Swizzle: int = SwizzleNone
    L2Promotion: int = L2PromotionNone
    OOBFill: int = OOBFillNone


class TensorMap:
    """An encoded CUtensorMap kept 64-byte aligned (host/tensormap.go:134-163)."""

    def __init__(self):
        self._backing = (ctypes.c_uint8 * (TENSOR_MAP_BYTES + 63))()
        base = ctypes.addressof(self._backing)
        self.addr = base + (-base) % 64

    def Bytes(self) -> bytes:
        return ctypes.string_at(self.addr, TENSOR_MAP_BYTES)

    def Arg(self) -> "Arg":
        return ArgBytes(self.Bytes())

    ArgEx = Arg


def _arr(ctype, values):
    values = list(values)
    return (ctype * max(1, len(values)))(*values), len(values)


def EncodeTiledPtr(ptr: int, d: TiledTensor, _elem_size: int = 0) -> TensorMap:
    """Encodes a tensor map over a raw device pointer (host/tensormap.go:180)."""
    m = TensorMap()
    gd, nrank = _arr(ctypes.c_uint64, d.GlobalDim)
    gs, ngs = _arr(ctypes.c_uint64, d.GlobalStrides)
    bd, nbd = _arr(ctypes.c_uint32, d.BoxDim)
    if d.ElementStrides is None:
        es, nes = None, 0
    else:
        es, nes = _arr(ctypes.c_uint32, d.ElementStrides)
    check(lib().cudair_encode_tiled(
        ctypes.c_void_p(m.addr), d.DataType, nrank, int(ptr), gd, gs, ngs, bd, nbd, es, nes,
        d.Interleave, d.Swizzle, d.L2Promotion, d.OOBFill, _elem_size))
    return m


def EncodeTiled(buf, d: TiledTensor) -> TensorMap:
    """Encodes a tensor map over a device buffer (a torch tensor), checking that
    its element size matches d.DataType (host/tensormap.go:167-176)."""
    if buf is None:
        raise CudairError(1, "host: EncodeTiled: nil buffer")
    return EncodeTiledPtr(buf.data_ptr(), d, _elem_size=buf.element_size())


# ---- kernel arguments (host/launchex.go:235-276) -----------------------------


class Arg:
    """One kernel parameter: the bytes the driver copies into parameter space,
    held in 8-byte aligned storage."""

    def __init__(self, data: bytes):
        n = len(data)
        self._store = (ctypes.c_uint64 * max(1, (n + 7) // 8))()
        ctypes.memmove(self._store, data, n)
        self.size = n

    @property
    def ptr(self) -> int:
        return ctypes.addressof(self._store)


def ArgValue(v) -> Arg:
    """Passes a ctypes scalar or structure by value (ArgValue[T])."""
    return Arg(bytes(v))


def ArgBuffer(t) -> Arg:
    """Passes a device buffer's pointer (ArgBuffer[T]); t is a torch tensor or an int.
    The argument keeps the tensor alive, so a temporary buffer is not freed (and its
    memory handed to another allocation) before the launch that reads it."""
    ptr = t if isinstance(t, int) else t.data_ptr()
    a = Arg(bytes(ctypes.c_uint64(ptr)))
    a.buffer = None if isinstance(t, int) else t
    return a


def ArgBytes(p: bytes) -> Arg:
    return Arg(bytes(p))


# ---- launch configuration (gocudrv cuda.LaunchConfig) ------------------------


@dataclass
class LaunchConfig:
    GridX: int = 1
    GridY: int = 1
    GridZ: int = 1
    BlockX: int = 1
    BlockY: int = 1
    BlockZ: int = 1
    SharedMemBytes: int = 0


def LaunchConfig1D(n: int, block: int) -> LaunchConfig:
    """ceil(n/block) blocks of `block` threads (gocudrv cuda.LaunchConfig1D)."""
    return LaunchConfig(GridX=(n + block - 1) // block, BlockX=block)


@dataclass
class LaunchAttrs:
    """host.LaunchAttrs (host/launchex.go:105-120)."""
    ClusterDim: Sequence[int] = field(default_factory=lambda: (0, 0, 0))
    Cooperative: bool = False
    ProgrammaticStreamSerialization: bool = False


# ---- modules and functions (host/launchex.go:31-101) -------------------------


class Function:
    def __init__(self, mod: "Module", raw: int, name: str):
        self.mod, self.raw, self.name = mod, raw, name

    def LaunchEx(self, cfg: LaunchConfig, attrs: LaunchAttrs, *args: Arg) -> None:
        """Launches on the default stream, then waits for the context."""
        self.LaunchExOn(None, cfg, attrs, *args)

    def LaunchExOn(self, stream, cfg: LaunchConfig, attrs: LaunchAttrs, *args: Arg) -> None:
        """Launches on `stream` (a torch.cuda.Stream, a raw handle, or None for
        the legacy default stream, which also synchronises)."""
        if self.raw is None:
            raise CudairError(1, "host: LaunchEx: nil function")
        grid = (ctypes.c_uint32 * 3)(cfg.GridX, cfg.GridY, cfg.GridZ)
        block = (ctypes.c_uint32 * 3)(cfg.BlockX, cfg.BlockY, cfg.BlockZ)
        cluster = (ctypes.c_uint32 * 3)(*attrs.ClusterDim)
        params = (ctypes.c_void_p * max(1, len(args)))(*[a.ptr for a in args])
        check(lib().cudair_launch_ex(
            ctypes.c_void_p(self.raw), grid, block, cfg.SharedMemBytes, _stream_handle(stream),
            cluster, int(attrs.Cooperative), int(attrs.ProgrammaticStreamSerialization),
            params if args else None))


class Module:
    def __init__(self, raw: int):
        self.raw = raw

    def Function(self, name: str) -> Function:
        if not self.raw:
            raise CudairError(1, "host: Function: module is closed")
        f = ctypes.c_void_p()
        check(lib().cudair_module_function(ctypes.c_void_p(self.raw), name.encode(),
                                           ctypes.byref(f)))
        return Function(self, f.value, name)

    def Close(self) -> None:
        if self.raw:
            raw, self.raw = self.raw, None
            check(lib().cudair_module_unload(ctypes.c_void_p(raw)))


def LoadModule(image: bytes) -> Module:
    """Loads a module image (cubin, or PTX text) into the current context."""
    buf = ctypes.create_string_buffer(bytes(image), len(image))
    m = ctypes.c_void_p()
    check(lib().cudair_module_load(buf, len(image), ctypes.byref(m)))
    return Module(m.value)


def KernelsImage() -> bytes:
    """The sm_100a module with the reference's kernel names (MatMul16, VecAdd,
    ReduceF32): the drop-in for the PTX cudair.Build produces."""
    with open(CUBIN_PATH, "rb") as f:
        return f.read()


def Synchronize() -> None:
    check(lib().cudair_ctx_synchronize())


def _stream_handle(stream) -> Optional[int]:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream  # torch.cuda.Stream
