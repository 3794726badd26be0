"""Host logic of the row-sharded GEMM over several GPUs (one process per GPU).

Rank g of G owns a contiguous block of rows of A and C; B is replicated into
every GPU's own memory by a peer copy from rank 0 (CUDA IPC: rank 0 exports
its allocation, the others map it, copy it over NVLink into local HBM and
unmap it).  No kernel ever reads another GPU's memory, and no collective runs
on the data path; an all-gather of C, if wanted, is a separate NCCL call.

The process-group plumbing here works on any torch.distributed backend, so
the same functions run on gloo ranks on CPU in the tests (with the GPU copy
replaced) and on NCCL ranks on B200s in bench.py.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional, Tuple

IPC_HANDLE_BYTES = 64


def row_block(m_total: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, end) of the rows rank owns: contiguous blocks whose sizes
    differ by at most one row, in rank order."""
    if world < 1 or not (0 <= rank < world) or m_total < 0:
        raise ValueError(f"row_block: m_total={m_total} world={world} rank={rank}")
    base, extra = divmod(m_total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def exchange_from_rank0(payload: Optional[bytes], rank: int, world: int) -> bytes:
    """Returns rank 0's payload on every rank (all_gather_object: the same
    collective step on every rank)."""
    if world == 1:
        assert payload is not None
        return payload
    import torch.distributed as dist
    objs = [None] * world
    dist.all_gather_object(objs, payload if rank == 0 else None)
    if not isinstance(objs[0], (bytes, bytearray)):
        raise RuntimeError("exchange_from_rank0: rank 0 sent no payload")
    return bytes(objs[0])


def max_over_ranks(x: float, world: int, device=None) -> float:
    """The largest x over all ranks (device: where the reduction tensor lives;
    a CUDA device for NCCL, None for gloo)."""
    if world == 1:
        return float(x)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def any_rank(flag: bool, world: int, device=None) -> bool:
    """True on every rank when flag is true on any rank (one all-reduce: the
    same collective step everywhere, so a local failure cannot leave the
    other ranks waiting in a later collective)."""
    return max_over_ranks(1.0 if flag else 0.0, world, device) > 0.0


def replicate_from_rank0(buf, rank: int, world: int,
                         copy_fn: Optional[Callable[[int, int, int], float]] = None) -> float:
    """Makes every rank's `buf` (a CUDA tensor of the same size on each GPU)
    equal to rank 0's by one peer copy over NVLink; returns the copy time in
    ms on this rank (0 on rank 0).

    copy_fn(kind, buf, arg) may replace the GPU copy (tests); by default the C
    ABI does it: cudair_ipc_export on rank 0, cudair_ipc_open /
    cudair_peer_copy / cudair_ipc_close on the others.

    Failures are collective: if rank 0 cannot export, it sends the error in
    place of the handle, and if any rank cannot copy, an all-reduce tells
    every rank; all ranks then raise RuntimeError after the same collective
    steps, so none is left waiting for a peer that gave up."""
    if world == 1:
        return 0.0
    from . import _lib
    nbytes = buf.numel() * buf.element_size()
    payload = None
    if rank == 0:
        try:
            if copy_fn is None:
                h = (ctypes.c_uint8 * IPC_HANDLE_BYTES)()
                off = ctypes.c_uint64()
                _lib.check(_lib.lib().cudair_ipc_export(ctypes.c_void_p(buf.data_ptr()), h,
                                                        ctypes.byref(off)))
                # The handle maps the whole allocation; the offset locates buf in it.
                handle = bytes(h) + off.value.to_bytes(8, "little")
            else:
                handle = copy_fn("export", buf, nbytes)
            payload = b"OK" + handle
        except Exception as e:  # reported to every rank below
            payload = b"ER" + f"{type(e).__name__}: {e}".encode()
    payload = exchange_from_rank0(payload, rank, world)
    if payload[:2] != b"OK":
        raise RuntimeError("replicate_from_rank0: rank 0 could not export B: " + payload[2:].decode())
    handle = payload[2:]
    ms, err = 0.0, None
    if rank != 0:
        try:
            ms = _peer_copy_cuda(buf, handle, nbytes) if copy_fn is None else copy_fn("import", buf, handle)
        except Exception as e:
            err = f"{type(e).__name__}: {e}"
    # Also the barrier that keeps rank 0's B alive until every copy has landed.
    if any_rank(err is not None, world, buf.device if buf.is_cuda else None):
        raise RuntimeError("replicate_from_rank0: a peer copy failed"
                           + (f" on this rank ({err})" if err else " on another rank"))
    return ms


def _peer_copy_cuda(buf, handle: bytes, nbytes: int) -> float:
    import torch
    from . import _lib
    L = _lib.lib()
    h = (ctypes.c_uint8 * IPC_HANDLE_BYTES).from_buffer_copy(handle[:IPC_HANDLE_BYTES])
    offset = int.from_bytes(handle[IPC_HANDLE_BYTES:IPC_HANDLE_BYTES + 8], "little")
    peer = ctypes.c_void_p()
    _lib.check(L.cudair_ipc_open(h, ctypes.byref(peer)))
    try:
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        _lib.check(L.cudair_peer_copy(ctypes.c_void_p(buf.data_ptr()),
                                      ctypes.c_void_p(peer.value + offset), nbytes,
                                      ctypes.c_void_p(s.cuda_stream)))
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)
    finally:
        _lib.check(L.cudair_ipc_close(peer))
