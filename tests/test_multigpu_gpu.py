"""The row-sharded GEMM on two GPUs (skipped with fewer): one process per
GPU, each owns a block of rows of A and C, B reaches rank 1 by a peer copy
from rank 0's memory (CUDA IPC over NVLink), and each rank's C shard is
checked against the oracle's fp32 product of the same operands within the
GEMM tolerance.  The operands come from the seeded streams (cudair_fill on
the device: A seed 11 at the rank's row offset, B seed 12 on rank 0 only,
C seed 13), and every rank's B is checked bit for bit against the oracle's."""
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
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import numpy as np
        import oracle
        M, N, K = 2048, 1024, 1024
        std = 1.0 / math.sqrt(K)
        r0, r1 = multigpu.row_block(M, world, rank)
        a = torch.empty(r1 - r0, K, dtype=torch.float16, device=dev)
        kernels.fill_normal(a, 11, 0.0, std, offset=r0 * K)
        c = torch.empty(r1 - r0, N, device=dev)
        kernels.fill_normal(c, 13, 0.0, 1.0, offset=r0 * N)
        b = torch.empty(K, N, dtype=torch.float16, device=dev)
        if rank == 0:
            kernels.fill_normal(b, 12, 0.0, std)
        torch.cuda.synchronize()
        ms = multigpu.replicate_from_rank0(b, rank, world)
        kernels.gemm(a, b, c)
        torch.cuda.synchronize()
        b16 = oracle.f32_to_f16(oracle.normal(K * N, 12, 0.0, std)).reshape(K, N)
        b_ok = bool(np.array_equal(b.cpu().view(torch.int16).numpy().view(np.uint16), b16))
        a16 = oracle.f32_to_f16(oracle.normal((r1 - r0) * K, 11, 0.0, std, offset=r0 * K))
        af, bf = oracle.f16_to_f32(a16).reshape(r1 - r0, K), oracle.f16_to_f32(b16)
        c0 = oracle.normal((r1 - r0) * N, 13, 0.0, 1.0, offset=r0 * N).reshape(r1 - r0, N)
        want = oracle.gemm_ikj(af, bf, c0)
        rel, mx, bad = oracle.error_norms(c.cpu().numpy(), want)
        tol_rel, tol_max = oracle.gemm_tolerance(K, float(np.abs(af).max()), float(np.abs(bf).max()))
        q.put((rank, {"b_ok": b_ok, "rel": rel, "max": mx, "bad": bad, "tol_rel": tol_rel,
                      "bound": tol_max, "ms": ms, "rows": (r0, r1)}))
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
        assert res[r]["bad"] == 0 and res[r]["rel"] <= res[r]["tol_rel"], res[r]
        assert res[r]["max"] <= res[r]["bound"], res[r]


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
