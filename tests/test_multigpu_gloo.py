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


# ---- failures, made on the host (no GPU involved) ------------------------------


def _fail_worker(rank, world, port, q, where):
    sys.path.insert(0, os.path.join(REPO, "cuda-ir.go_b200"))
    import datetime

    import torch
    import torch.distributed as dist
    from cudair import multigpu

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        def failing_copy(kind, buf, arg):
            if kind == where:
                raise OSError(f"injected {kind} failure")
            return buf.numpy().tobytes() if kind == "export" else 0.5

        b = torch.zeros(16)
        try:
            multigpu.replicate_from_rank0(b, rank, world, copy_fn=failing_copy)
            msg = None
        except RuntimeError as e:
            msg = str(e)
        # The group is still in step: one more collective completes.
        after = multigpu.max_over_ranks(float(rank), world)
        q.put((rank, {"msg": msg, "after": after}))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("where", ["export", "import"])
def test_replication_failure_reaches_every_rank(where):
    # An IPC export that fails on rank 0, or a peer copy that fails on rank 1
    # (the "peer access unavailable" case): every rank raises, none waits for
    # a peer that gave up, and the process group stays usable.
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fail_worker, args=(r, world, port, q, where)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r]["msg"] is not None, res
        assert res[r]["after"] == 1.0
    if where == "export":
        assert all("could not export" in res[r]["msg"] and "injected export failure" in res[r]["msg"]
                   for r in range(world))
    else:
        assert "on this rank" in res[1]["msg"] and "injected import failure" in res[1]["msg"]
        assert "on another rank" in res[0]["msg"]


def _vanishing_worker(rank, world, port, q):
    sys.path.insert(0, os.path.join(REPO, "cuda-ir.go_b200"))
    import datetime
    import time

    import torch.distributed as dist
    from cudair import multigpu

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    multigpu.max_over_ranks(float(rank), world)  # one step together
    if rank == 1:
        os._exit(0)  # leaves between steps, without a goodbye
    time.sleep(1.0)
    t0 = time.monotonic()
    try:
        multigpu.max_over_ranks(1.0, world)
        outcome = "completed"
    except Exception as e:  # the peer is gone: the collective fails
        outcome = type(e).__name__
    q.put((rank, {"outcome": outcome, "seconds": time.monotonic() - t0}))
    q.close()
    q.join_thread()  # the result is sent before the process ends
    os._exit(0)  # no teardown with a peer that is gone


def test_rank_that_leaves_ends_the_next_collective_with_an_error():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_vanishing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        rank, out = q.get(timeout=90)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert rank == 0
    assert out["outcome"] != "completed"
    assert out["seconds"] < 60
