"""Benchmark of the MatMul16 / VecAdd path on B200s (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload (weak scaling, fixed work per GPU): the row-sharded GEMM
C = A.B + C with fp16 A, B and fp32 C.  Rank g owns rows [8192 g, 8192 (g+1))
of A and C, B (K x N) is replicated; M = 8192 N, N = K = 8192.  At N = 1 this
is the 8192^3 GEMM, at N = 8 the M = 65536 row-sharded GEMM.  A, B ~
fp16(N(0,1)/sqrt(8192)), C ~ N(0,1), seeded, generated on the device.  B is
replicated once before timing by a peer copy over NVLink from rank 0's memory
(CUDA IPC), timed separately; no collective runs on the data path.  Inputs
(A 128 MiB, B 128 MiB, C 256 MiB per GPU) exceed the 126 MB L2, so no flush
is needed between steps.

One step = one launch of the tcgen05 GEMM over the GPU's shard.  `value` is
the aggregate TFLOP/s over all ranks (2 M N K per step / the max over ranks of
the device-timed step).  `e2e` times the same step through the C ABI's host
entry (cudair_gemm_f16f32_host): pinned host -> device copies of A, B, C, the
GEMM, and the device -> host copy of C, all inside the timed region, the
copies of one block of rows overlapping the GEMM of another.  The line also
carries VecAdd, Saxpy and Square (n = 2^28 fp32 per GPU, HBM-bound) and the
decode-shaped GEMM (M=16, N=14336, K=4096, three copies of B cycled so each
launch reads B from HBM, timed from a CUDA graph) as secondary results, each
against its roofline.

`--impl reference` times the reference's CPU implementation of the path (the
i-j-k float32 loop of its tests, restated in C under oracle/) on all host
threads, on a bounded sample of rows of the same workload; under torchrun
only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "cuda-ir.go_b200"))

METRIC = "fp16 GEMM TFLOP/s & % tensor peak; VecAdd GB/s & % HBM; at 1/2/4/8 GPUs"
ROWS_PER_GPU = 8192
N_DIM = 8192
K_DIM = 8192
VEC_N = 1 << 28
SKINNY = (16, 14336, 4096)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic():
    """DRAM bytes per launch from the committed ncu summaries
    (profiles/dram_traffic.txt: `<workload> <bytes>` lines)."""
    out = {}
    p = os.path.join(REPO, "profiles", "dram_traffic.txt")
    if os.path.exists(p):
        for line in open(p):
            parts = line.split()
            if len(parts) >= 2 and not line.startswith("#"):
                try:
                    out[parts[0]] = float(parts[1])
                except ValueError:
                    pass
    return out


# ---- clocks during the timed region ------------------------------------------


class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU through NVML in a
    background thread (read-only queries)."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period_s: float = 0.002):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            uuid_env = os.environ.get("CUDA_VISIBLE_DEVICES")
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self._physical_index(index, uuid_env))
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report no clocks rather than guess
            log(f"clock sampler unavailable: {e}")

    @staticmethod
    def _physical_index(index, env):
        if env:
            ids = [x for x in env.split(",") if x.strip()]
            if index < len(ids) and ids[index].strip().isdigit():
                return int(ids[index])
        return index

    def _sample(self):
        nv = self._nv
        mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
        try:
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except Exception:
            r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
        self.samples.append(mhz)
        for name, bit in self.REASONS.items():
            if r & bit:
                self.reasons.add(name)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._t:
            self._stop.set()
            self._t.join()
            try:
                self._sample()
            except Exception:
                pass

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


# ---- distributed plumbing -------------------------------------------------------


def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return world, rank, local  # CPU only: no process group, no GPU
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(x: float, world: int, dev) -> float:
    from cudair import multigpu
    return multigpu.max_over_ranks(x, world, dev)


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---- timing helpers ----------------------------------------------------------------


def time_steps(fn, steps, warmup, world, dev, sampler=None):
    """W untimed warm-up steps, then K steps bracketed by barrier + synchronize,
    timed with CUDA events on the current stream; returns ms per step (max
    over ranks)."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx = sampler if sampler is not None else _Null()
    with ctx:
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = start.elapsed_time(end) / steps
    return max_over_ranks(ms, world, dev)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


# ---- B replication by peer copy ------------------------------------------------


def replicate_b(b, world, rank, dev):
    """Copies rank 0's B into every other rank's local B over NVLink (CUDA IPC
    export on rank 0, map + one device-to-device copy + unmap elsewhere);
    returns the max copy time over ranks in ms."""
    from cudair import multigpu
    ms = multigpu.replicate_from_rank0(b, rank, world)
    if world > 1:
        log(f"rank {rank}: B replicated in {ms:.3f} ms")
    return max_over_ranks(ms, world, dev)


# ---- CPU baseline (the reference's CPU loop, restated in C) ---------------------


class CpuGemm:
    """The reference's CPU loop for this path: the i-j-k float32 GEMM of its
    tests (advanced_test.go:466-475, restated in oracle/oracle.c), over whole
    rows of the 8192 x 8192 x 8192 problem; rows are independent, so a sample
    of rows measures the loop's rate exactly."""

    def __init__(self, max_rows: int):
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import oracle
        self.o = oracle
        s = 1.0 / math.sqrt(K_DIM)
        self.af = oracle.f16_to_f32(oracle.f32_to_f16(
            oracle.normal(max_rows * K_DIM, 106, 0.0, s))).reshape(max_rows, K_DIM)
        self.bf = oracle.f16_to_f32(oracle.f32_to_f16(
            oracle.normal(K_DIM * N_DIM, 107, 0.0, s))).reshape(K_DIM, N_DIM)
        self.c = oracle.normal(max_rows * N_DIM, 108).reshape(max_rows, N_DIM)

    def run(self, rows: int, threads: int) -> float:
        """Seconds to compute `rows` rows on `threads` threads."""
        t0 = time.perf_counter()
        self.o.gemm_ijk(self.af[:rows], self.bf, self.c[:rows], threads=threads)
        return time.perf_counter() - t0

    def sample(self, threads: int, budget_s: float):
        """Rows sized to about budget_s seconds; returns (TFLOP/s, rows, s)."""
        rows = threads
        dt = self.run(rows, threads)
        more = int(max(0.0, budget_s - dt) / max(dt / rows, 1e-9))
        more = min(more, self.af.shape[0] - rows)
        more -= more % max(1, threads)
        if more > 0:
            dt2 = self.run(more, threads)
            rows, dt = rows + more, dt + dt2
        return 2.0 * rows * N_DIM * K_DIM / dt / 1e12, rows, dt


def run_matmul16_n256(dev, kernels):
    """The MatMul16 parity configuration (n = 256, the reference test's size):
    per-launch latency of the module entry under the reference's launch
    (grid (n/16, n/16) x 32 threads) and of the library's cudair_matmul16
    (which picks that same one-warp-per-tile kernel for n <= 512), each from a
    CUDA graph of 20 launches (a single launch timed from Python measures the
    host's launch cost), beside the CPU i-j-k loop on the same operands.
    Inputs: fp16(U(-1,1)) A and B, U(-1,1) C, seeded."""
    import ctypes

    import torch
    from cudair import host
    n = 256
    g = torch.Generator(device=dev)
    g.manual_seed(256)
    a = (torch.rand(n, n, generator=g, device=dev) * 2 - 1).half()
    b = (torch.rand(n, n, generator=g, device=dev) * 2 - 1).half()
    c = torch.rand(n, n, generator=g, device=dev) * 2 - 1
    af, bf, c0 = a.float().cpu().numpy(), b.float().cpu().numpy(), c.cpu().numpy()
    mod = host.LoadModule(host.KernelsImage())
    fn = mod.Function("MatMul16")
    cfg = host.LaunchConfig(GridX=n // 16, GridY=n // 16, BlockX=32)
    args = (host.ArgBuffer(a), host.ArgBuffer(b), host.ArgBuffer(c), host.ArgValue(ctypes.c_int32(n)))
    out = {}
    for name, launch in (("reference_launch_us", lambda s: fn.LaunchExOn(s, cfg, host.LaunchAttrs(), *args)),
                         ("library_us", lambda s: kernels.matmul16(a, b, c, stream=s))):
        st = torch.cuda.Stream(device=dev)
        for _ in range(3):
            launch(st)
        st.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            for _ in range(20):
                launch(st)
        graph.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) / 20 * 1e3)
        out[name] = statistics.median(ts)
        del graph
    mod.Close()
    # The CPU baseline of this configuration: the oracle's i-j-k loop.
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    t0 = time.perf_counter()
    oracle.gemm_ijk(af, bf, c0, threads=1)
    out["cpu_us_1thread"] = (time.perf_counter() - t0) * 1e6
    out["timing"] = "CUDA graph of 20 launches, per launch; CPU: the i-j-k loop, 1 thread"
    return out


def cpu_secondary():
    """The reference's CPU loops for the VecAdd (2^26-element sample of the
    2^28 workload) and decode-shaped GEMM configurations, 1 thread and all
    host threads."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    T = oracle.num_threads()
    out = {}
    n = 1 << 26
    a, b = oracle.uniform(n, 4), oracle.uniform(n, 5)
    for t in (1, T):
        best = float("inf")
        for _ in range(2):  # the second call reuses the output pages the first one touched
            t0 = time.perf_counter()
            oracle.vecadd(a, b, threads=t)
            best = min(best, time.perf_counter() - t0)
        out[f"vecadd_GB/s_{'1thread' if t == 1 else 'all'}"] = 12 * n / best / 1e9
    sm, sn, sk = SKINNY
    af = oracle.normal(sm * sk, 9).reshape(sm, sk)
    bf = (oracle.normal(sk * sn, 10) * 0.02).astype("float32").reshape(sk, sn)
    c = oracle.uniform(sm * sn, 11).reshape(sm, sn) * 0
    for t in (1, T):
        t0 = time.perf_counter()
        oracle.gemm_ikj(af, bf, c, threads=t)
        out[f"skinny_ms_{'1thread' if t == 1 else 'all'}"] = (time.perf_counter() - t0) * 1e3
    out["threads"] = T
    out["sample"] = "VecAdd: 2^26 elements; decode GEMM: the whole 16x14336x4096 (i-k-j float32 loop)"
    return out


def run_reference(args, world, rank):
    """The reference arm: the CPU i-j-k loop on all host threads, rank 0 only;
    each step computes one row per thread of the workload."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    threads = oracle.num_threads()
    cpu = CpuGemm(max_rows=threads)
    rows_total, secs_total = 0, 0.0
    for i in range(args.warmup + args.steps):
        dt = cpu.run(threads, threads)
        if i >= args.warmup:
            rows_total += threads
            secs_total += dt
    value = 2.0 * rows_total * N_DIM * K_DIM / secs_total / 1e12
    sample = (f"{rows_total} rows of C = A.B + C with N=K={N_DIM} over {args.steps} steps "
              f"({threads} rows per step, one per thread), i-j-k float32 loop")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * secs_total / max(1, args.steps), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (fp16-rounded inputs)",
        "data": "synthetic (seeded N(0,1)/sqrt(K) operands)",
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(n_gpus):
    return {"workload": "row-sharded MatMul16 GEMM C=A.B+C (fp16 A,B; fp32 C, fp32 accumulate)",
            "M": ROWS_PER_GPU * n_gpus, "N": N_DIM, "K": K_DIM, "rows_per_gpu": ROWS_PER_GPU,
            "partition": "row blocks of A and C; B replicated by peer copy",
            "l2": "inputs exceed L2 (512 MiB per GPU vs 126 MB)",
            "secondary": {"vecadd_n_per_gpu": VEC_N, "skinny_MNK": list(SKINNY)}}


# ---- our arm -------------------------------------------------------------------------


def run_e2e(args, world, rank, dev, a, b, c, flops, kernels):
    """The GEMM step from pinned host buffers through the C ABI's host entry
    (cudair_gemm_f16f32_host): every step copies A, B and C in, multiplies
    and copies C back to the host, all inside the timed region, with the
    copies of one block of rows overlapping the GEMM of another.  With
    several GPUs, B (the same on every rank) is not sent over every host link
    in full: each rank copies 1/world of its rows in, and an all-gather over
    NVLink assembles B on every GPU before the host entry takes over."""
    import torch
    a_h = a.cpu().pin_memory()
    b_h = b.cpu().pin_memory()
    c_h = c.cpu().pin_memory()
    a_d, b_d, c_d = torch.empty_like(a), torch.empty_like(b), torch.empty_like(c)
    K = b.shape[0]
    if world > 1 and K % world == 0:
        import torch.distributed as dist
        rows = K // world
        b_h_part = b_h[rank * rows:(rank + 1) * rows]
        b_part = torch.empty(rows, b.shape[1], dtype=b.dtype, device=dev)

        def e2e_step():
            b_part.copy_(b_h_part, non_blocking=True)
            dist.all_gather_into_tensor(b_d.view(-1), b_part.view(-1))
            kernels.gemm_host(a_h, None, c_h, a_d, b_d, c_d)

        b_bytes = b_part.numel() * 2
        api = ("B: 1/world of its rows per rank over the host link, all-gathered over NVLink; "
               "then cudair_gemm_f16f32_host (row blocks of 512: H2D, GEMM and D2H overlapped; "
               "B is already on the device)")
    else:
        def e2e_step():
            kernels.gemm_host(a_h, b_h, c_h, a_d, b_d, c_d)

        b_bytes = b_h.numel() * 2
        api = ("cudair_gemm_f16f32_host (4 x 4 tiles of 2048 x 2048: B by column blocks, A by row "
               "blocks, C by tiles; H2D, GEMM and D2H overlapped)")

    steps = max(3, min(args.steps, 20))
    ms = time_steps(e2e_step, steps, 3, world, dev)
    return {"value": flops * world / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": a_h.numel() * 2 + b_bytes + c_h.numel() * 4,
            "d2h_bytes_per_step": c_h.numel() * 4, "ms_per_step": ms, "steps": steps, "api": api}


def run_gather(world, dev, M, N):
    """Optional reassembly of C on every GPU with NCCL all-gather (not part of
    the step; timed on its own)."""
    import torch
    import torch.distributed as dist
    c = torch.zeros(M, N, dtype=torch.float32, device=dev)
    full = torch.empty(world * M, N, dtype=torch.float32, device=dev)
    t = time_steps(lambda: dist.all_gather_into_tensor(full, c), 3, 3, world, dev)
    out = {"ms": t, "bytes_received_per_gpu": (world - 1) * M * N * 4,
           "GB/s_per_gpu": (world - 1) * M * N * 4 / (t * 1e-3) / 1e9}
    del full, c
    return out


def run_vecadd(args, world, rank, dev, g, kernels):
    """VecAdd over n = 2^28 fp32 per GPU (3 GiB of traffic per step, > L2)."""
    import torch
    g.manual_seed(4000 + rank)
    va = torch.rand(VEC_N, generator=g, device=dev) * 2 - 1
    vb = torch.rand(VEC_N, generator=g, device=dev) * 2 - 1
    vo = torch.empty_like(va)
    ms = time_steps(lambda: kernels.vecadd(va, vb, vo), args.steps, args.warmup, world, dev)
    del va, vb, vo
    return ms, 3 * 4 * VEC_N / (ms * 1e-3) / 1e9


def run_saxpy_square(args, world, rank, dev, g, kernels):
    """Saxpy (12 bytes per element: read x and y, write y) and Square (8: read
    and write x) over n = 2^28 fp32 per GPU, each step one launch."""
    import torch
    g.manual_seed(4100 + rank)
    x = torch.rand(VEC_N, generator=g, device=dev) * 2 - 1
    y = torch.rand(VEC_N, generator=g, device=dev) * 2 - 1
    ms_saxpy = time_steps(lambda: kernels.saxpy(0.5, x, y), args.steps, args.warmup, world, dev)
    ms_square = time_steps(lambda: kernels.square(x), args.steps, args.warmup, world, dev)
    del x, y
    return {"saxpy": (ms_saxpy, 12 * VEC_N / (ms_saxpy * 1e-3) / 1e9),
            "square": (ms_square, 8 * VEC_N / (ms_square * 1e-3) / 1e9)}


def run_skinny(args, world, rank, dev, g, kernels):
    """M=16, N=14336, K=4096 (decode-shaped): B is 117 MB, so three copies of
    it are cycled (351 MB > L2) and every launch streams its B from HBM.  A
    decode step issues such GEMMs back to back from a captured CUDA graph, so
    30 launches are captured once and the graph replays are timed with events
    (per launch: replay time / 30); a launch timed alone from Python would
    measure the host's launch cost, which exceeds the kernel's time.  The
    launches use programmatic dependent launch with B requested before the
    dependency wait (cudair_set_gemm_pdl(2)): B is never written in the chain."""
    import torch
    sm, sn, sk = SKINNY
    g.manual_seed(9000 + rank)
    sa = torch.randn(sm, sk, generator=g, device=dev).half()
    sbs = [(torch.randn(sk, sn, generator=g, device=dev) * 0.02).half() for _ in range(3)]
    sc = torch.zeros(sm, sn, device=dev)
    kernels.set_gemm_pdl(2)
    for i in range(max(3, args.warmup)):
        kernels.gemm(sa, sbs[i % 3], sc)
    torch.cuda.synchronize()
    per_graph = 30
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=dev)):
        for i in range(per_graph):
            kernels.gemm(sa, sbs[i % 3], sc)
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(max(3, min(args.steps, 10))):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / per_graph)
    kernels.set_gemm_pdl(0)
    ms = max_over_ranks(statistics.median(times), world, dev)
    gbs = (sk * sn * 2 + sm * sk * 2 + 2 * sm * sn * 4) / (ms * 1e-3) / 1e9
    del graph, sa, sbs, sc
    return ms, gbs


def run_ours(args, world, rank, local):
    import torch
    from cudair import kernels

    dev = torch.device("cuda", local)
    kernels.set_gemm_variant(args.gemm_variant)
    peaks, peak_kind = load_peaks()
    traffic = load_traffic()
    g = torch.Generator(device=dev)
    only = args.workload

    if only == "vecadd":
        v_ms, v_gbs = run_vecadd(args, world, rank, dev, g, kernels)
        log(f"rank {rank}: vecadd {v_ms:.4f} ms/step {v_gbs:.1f} GB/s")
        return
    if only == "skinny":
        s_ms, s_gbs = run_skinny(args, world, rank, dev, g, kernels)
        log(f"rank {rank}: skinny {s_ms:.4f} ms {s_gbs:.1f} GB/s")
        return

    # -- the row-sharded GEMM: inputs resident in HBM
    M, N, K = ROWS_PER_GPU, N_DIM, K_DIM
    g.manual_seed(6000 + rank)
    a = (torch.randn(M, K, generator=g, device=dev) / math.sqrt(K)).half()
    b = torch.empty(K, N, dtype=torch.float16, device=dev)
    if rank == 0:
        g.manual_seed(7000)
        b.copy_((torch.randn(K, N, generator=g, device=dev) / math.sqrt(K)).half())
    g.manual_seed(8000 + rank)
    c = torch.randn(M, N, generator=g, device=dev)
    torch.cuda.synchronize()
    b_ms = replicate_b(b, world, rank, dev)

    flops = 2.0 * M * N * K
    sampler = ClockSampler(local)
    ms = time_steps(lambda: kernels.gemm(a, b, c), args.steps, args.warmup, world, dev, sampler)
    clocks = sampler.summary()
    kernels.wait_status(clear=True)
    achieved = flops / (ms * 1e-3) / 1e12
    log(f"rank {rank}: gemm {ms:.4f} ms/step, {achieved:.1f} TFLOP/s per GPU")
    if only == "gemm":
        return

    e2e = run_e2e(args, world, rank, dev, a, b, c, flops, kernels)
    del a, b, c
    torch.cuda.empty_cache()
    gather = run_gather(world, dev, M, N) if (args.gather and world > 1) else None
    v_ms, v_gbs = run_vecadd(args, world, rank, dev, g, kernels)
    streams = run_saxpy_square(args, world, rank, dev, g, kernels)
    sm, sn, sk = SKINNY
    s_ms, s_gbs = run_skinny(args, world, rank, dev, g, kernels)
    kernels.wait_status(clear=True)

    # -- the n = 256 parity configuration and the CPU baselines (rank 0, N = 1 only)
    mm256 = run_matmul16_n256(dev, kernels) if (rank == 0 and world == 1) else None
    cpu = None
    cpu_more = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu_more = cpu_secondary()
        r, rows, dt = CpuGemm(max_rows=256).sample(1, budget_s=args.cpu_budget)
        cpu = {"value": r, "unit": "TFLOP/s", "cores": 1, "kind": "port",
               "sample": f"{rows} rows of the 8192^3 C = A.B + C by the i-j-k float32 loop "
                         f"(oracle/oracle.c restating advanced_test.go:466-475), 1 thread, "
                         f"{dt:.1f} s"}

    if rank != 0:
        return
    tensor_peak = peaks["bf16_tflops"]
    line = {
        "metric": METRIC, "value": achieved * world, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,1)/sqrt(8192) fp16 operands, N(0,1) fp32 C)",
        "config": workload_config(world),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": tensor_peak,
                     "unit": "TFLOP/s", "frac": achieved / tensor_peak,
                     "traffic": traffic.get("gemm_8192"),
                     "peak_kind": f"{peak_kind} bf16 burst (fp16 dense rate is equal)",
                     "frac_of_nominal": achieved / 2250.0},
        "e2e": e2e,
        "cpu_baseline": cpu,
        "gpu_launches": args.steps * world,
        "clocks": clocks,
        "b_replication_ms": b_ms,
        "gather": gather,
        "matmul16_n256": mm256,
        "cpu_secondary": cpu_more,
        "vecadd": {"value": v_gbs * world, "unit": "GB/s", "ms_per_step": v_ms, "n_per_gpu": VEC_N,
                   "roofline": {"bound": "hbm", "achieved": v_gbs, "peak": peaks["hbm_gbs"],
                                "unit": "GB/s", "frac": v_gbs / peaks["hbm_gbs"],
                                "traffic": traffic.get("vecadd_2p28"),
                                "frac_of_nominal": v_gbs / 8000.0}},
        **{name: {"value": gbs * world, "unit": "GB/s", "ms_per_step": ms, "n_per_gpu": VEC_N,
                  "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                               "frac": gbs / peaks["hbm_gbs"]}}
           for name, (ms, gbs) in streams.items()},
        "skinny": {"M": sm, "N": sn, "K": sk, "ms": s_ms, "GB/s": s_gbs,
                   "timing": "CUDA graph of 30 launches cycling 3 copies of B, per launch; "
                             "programmatic dependent launch, B requested before the wait",
                   "TFLOP/s": 2.0 * sm * sn * sk / (s_ms * 1e-3) / 1e12,
                   "roofline": {"bound": "hbm", "achieved": s_gbs, "peak": peaks["hbm_gbs"],
                                "unit": "GB/s", "frac": s_gbs / peaks["hbm_gbs"],
                                "traffic": traffic.get("skinny_16x14336x4096")}},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--gather", action="store_true", help="also all-gather C over NCCL (timed apart)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds for the CPU baseline")
    ap.add_argument("--gemm-variant", type=int, default=0,
                    help="GEMM kernel choice (cudair_set_gemm_variant; 0 = automatic)")
    ap.add_argument("--workload", choices=["all", "gemm", "vecadd", "skinny"], default="all",
                    help="run one part only (for profiling); the JSON line needs 'all'")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
