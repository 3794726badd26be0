"""The row-sharded GEMM on two GPUs (skipped with fewer): one process per
GPU, each owns a block of rows of A and C, B reaches rank 1 by a peer copy
from rank 0's memory (CUDA IPC over NVLink), and each rank's C shard is
checked against an fp32 product of its own rows within the GEMM tolerance."""
import os
import socket
import sys

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    sys.path.insert(0, os.path.join(REPO, "cuda-ir.go_b200"))
    import datetime
    import math

    import torch
    import torch.distributed as dist
    from cudair import kernels, multigpu

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        M, N, K = 2048, 1024, 1024
        r0, r1 = multigpu.row_block(M, world, rank)
        g = torch.Generator(device=dev)
        g.manual_seed(11)  # the same full A and C on every rank
        a_full = (torch.randn(M, K, generator=g, device=dev) / math.sqrt(K)).half()
        c_full = torch.randn(M, N, generator=g, device=dev)
        b = torch.empty(K, N, dtype=torch.float16, device=dev)
        if rank == 0:
            gb = torch.Generator(device=dev)
            gb.manual_seed(12)
            b.copy_((torch.randn(K, N, generator=gb, device=dev) / math.sqrt(K)).half())
        torch.cuda.synchronize()
        ms = multigpu.replicate_from_rank0(b, rank, world)
        gb = torch.Generator(device=dev)
        gb.manual_seed(12)
        b_ref = (torch.randn(K, N, generator=gb, device=dev) / math.sqrt(K)).half()
        b_ok = bool(torch.equal(b, b_ref))
        a = a_full[r0:r1].contiguous()
        c = c_full[r0:r1].contiguous()
        want = (a.float() @ b_ref.float()) + c
        kernels.gemm(a, b, c)
        torch.cuda.synchronize()
        rel = ((c - want).norm() / want.norm()).item()
        mx = (c - want).abs().max().item()
        bound = 5e-3 * math.sqrt(K) * a.abs().max().item() * b_ref.abs().max().item()
        q.put((rank, {"b_ok": b_ok, "rel": rel, "max": mx, "bound": bound, "ms": ms,
                      "rows": (r0, r1)}))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_row_sharded_gemm_two_gpus(dev):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, out = q.get(timeout=300)
        res[rank] = out
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0]["rows"] == (0, 1024) and res[1]["rows"] == (1024, 2048)
    for r in range(world):
        assert res[r]["b_ok"], f"rank {r}: B differs from rank 0's after the peer copy"
        assert res[r]["rel"] <= 1e-3 and res[r]["max"] <= res[r]["bound"], res[r]


def test_tensor_on_another_gpu_is_refused(dev):
    # The launchers run on the current device; a tensor of another GPU is
    # refused before anything is launched (its kernels would otherwise read it
    # across NVLink).
    import torch
    from cudair import kernels
    from cudair._lib import CudairError
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with torch.cuda.device(0):
        a = torch.ones(1024, device="cuda:1")
        b = torch.ones(1024, device="cuda:0")
        out = torch.empty(1024, device="cuda:0")
        with pytest.raises(CudairError, match="current device is cuda:0"):
            kernels.vecadd(a, b, out)
