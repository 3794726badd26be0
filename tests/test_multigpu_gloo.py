"""The multi-GPU host logic on CPU: two gloo ranks run the same functions the
NCCL ranks of bench.py run (row blocks, the rank-0 handle exchange, the B
replication protocol with the GPU copy replaced, the max-over-ranks timing)."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    sys.path.insert(0, os.path.join(REPO, "cuda-ir.go_b200"))
    import datetime

    import torch
    import torch.distributed as dist
    from cudair import multigpu

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        out = {}
        out["block"] = multigpu.row_block(65536, world, rank)
        out["max"] = multigpu.max_over_ranks(1.5 + rank, world)
        # Rank 0's B reaches every rank through the export/import protocol.
        b = torch.full((1000,), float(rank))
        if rank == 0:
            b = torch.arange(1000, dtype=torch.float32)
        exported = {}

        def fake_copy(kind, buf, arg):
            if kind == "export":
                exported["bytes"] = buf.numpy().tobytes()[:64]
                return buf.numpy().tobytes()  # stands in for the IPC handle
            src = torch.frombuffer(bytearray(arg), dtype=torch.float32)
            buf.copy_(src)
            return 0.25

        ms = multigpu.replicate_from_rank0(b, rank, world, copy_fn=fake_copy)
        out["b_ok"] = bool(torch.equal(b, torch.arange(1000, dtype=torch.float32)))
        out["ms"] = ms
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_row_block_partition():
    sys.path.insert(0, os.path.join(REPO, "cuda-ir.go_b200"))
    from cudair import multigpu
    for M in (0, 1, 7, 8192, 65536, 65537):
        for G in (1, 2, 3, 4, 8):
            blocks = [multigpu.row_block(M, G, g) for g in range(G)]
            assert blocks[0][0] == 0 and blocks[-1][1] == M
            assert all(blocks[i][1] == blocks[i + 1][0] for i in range(G - 1))
            sizes = [e - s for s, e in blocks]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        multigpu.row_block(10, 2, 2)


def test_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, out = q.get(timeout=120)
        results[rank] = out
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0]["block"] == (0, 32768) and results[1]["block"] == (32768, 65536)
    assert results[0]["max"] == results[1]["max"] == 2.5
    assert results[0]["b_ok"] and results[1]["b_ok"]
    assert results[0]["ms"] == 0.0 and results[1]["ms"] == 0.25
