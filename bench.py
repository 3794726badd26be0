"""Benchmark of the MatMul16 / VecAdd path on B200s (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload (weak scaling, fixed work per GPU): the row-sharded GEMM
C = A.B + C with fp16 A, B and fp32 C, fp32 accumulation.  Rank g owns rows
[8192 g, 8192 (g+1)) of A and C, B (K x N) is replicated; M = 8192 N,
N = K = 8192.  At N = 1 this is the 8192^3 GEMM (A, B seeds 6, 7: fp16 of
N(0, 1/sqrt(8192)); C seed 8: N(0, 1)); at N > 1 it is the row-sharded GEMM
(A seed 11 at the rank's row offset, B seed 12, C = 0), which at N = 8 is the
M = 65536 configuration.  Every operand comes from the seeded counter-based
streams, generated in HBM by the library (cudair_fill) bit for bit as the CPU
oracle generates them.  B is generated on rank 0 and replicated once, before
timing, by a peer copy over NVLink (CUDA IPC), timed separately; no
collective runs on the data path.  Inputs (A 128 MiB, B 128 MiB, C 256 MiB
per GPU) exceed the 126 MB L2, so no flush is needed between steps.

One step = one launch of the tcgen05 GEMM over the GPU's shard.  `value` is
the aggregate TFLOP/s over all ranks (2 M N K per step / the max over ranks of
the device-timed step).  After timing, every rank restores C, runs one more
step and checks rows on both sides of the tile boundaries against the oracle
(`parity`); the inputs it read are checked bit for bit against the oracle's
streams, and B against rank 0's on every rank.

`e2e` times the same step through the C ABI's host entry
(cudair_gemm_f16f32_host): pinned host -> device copies of A, B, C, the GEMM
and the device -> host copy of C, all inside the timed region.  With N GPUs
each rank copies 1/N of B's rows in and an NCCL all-gather assembles B over
NVLink; `e2e.breakdown` times each part alone and the step's copies alone
(the host-link bound).  Each rank is bound to its GPU's NUMA node, so its
pinned host buffers are local to the GPU's PCIe root.

Also on the line: `strong_scaling` (the M = 65536 GEMM on one GPU against its
1/N row blocks on N), `gather` (NCCL all-gather of C, N > 1), VecAdd / Saxpy /
Square (n = 2^28 fp32 per GPU, HBM-bound; VecAdd with parity and e2e), the
decode-shaped GEMM (M=16, N=14336, K=4096, from a CUDA graph; parity and
e2e), and the MatMul16 n = 256 parity configuration (latency; e2e through
cudair_matmul16_host), each against its roofline.

`--impl reference` times the reference's CPU implementation of the path (the
i-j-k float32 loop of its tests, restated in C under oracle/) on all host
threads, on a bounded sample of rows of the same workload; under torchrun
only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import hashlib
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
STRONG_M = 65536
VEC_N = 1 << 28
SKINNY = (16, 14336, 4096)
OPERAND_STD = 1.0 / math.sqrt(8192.0)
NVLINK_GBS = 900.0           # NVLink 5, per direction per GPU (nominal)
PEER_COPY_GBS = 770.0        # measured peer copy on this part, per direction
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


def oracle_mod():
    """The CPU oracle: the checker of the parity legs and the timed CPU
    baseline; nothing timed on the GPU goes through it."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    return oracle


class GemmData:
    """Seeds of one GEMM configuration's operands: A and B fp16 of
    N(0, 1/sqrt(8192)), C N(0, 1) (seed_c) or zero (seed_c None)."""

    def __init__(self, name, seed_a, seed_b, seed_c):
        self.name, self.seed_a, self.seed_b, self.seed_c = name, seed_a, seed_b, seed_c

    def describe(self):
        c = f"N(0,1) seed {self.seed_c}" if self.seed_c is not None else "0"
        return (f"{self.name}: A fp16(N(0,1/sqrt(8192))) seed {self.seed_a} at the rank's row offset, "
                f"B fp16(N(0,1/sqrt(8192))) seed {self.seed_b}, C {c}")


CUBE = GemmData("8192^3 GEMM", 6, 7, 8)
SHARDED = GemmData("row-sharded GEMM", 11, 12, None)


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
            self._h = pynvml.nvmlDeviceGetHandleByIndex(physical_index(index))
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report no clocks rather than guess
            log(f"clock sampler unavailable: {e}")

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


def physical_index(index):
    env = os.environ.get("CUDA_VISIBLE_DEVICES")
    if env:
        ids = [x for x in env.split(",") if x.strip()]
        if index < len(ids) and ids[index].strip().isdigit():
            return int(ids[index])
    return index


def bind_host_to_gpu(index):
    """Restricts this process to the CPUs NVML lists as local to the GPU (its
    NUMA node), so the pinned host buffers it allocates afterwards sit on the
    memory next to the GPU's PCIe root.  Returns the CPU count, or None when
    nothing was changed."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(physical_index(index))
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (w >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
            return len(cpus)
    except Exception as e:
        log(f"no NUMA binding: {e}")
    return None


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


def gather_objects(obj, world):
    if world == 1:
        return [obj]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


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


# ---- operands ----------------------------------------------------------------------


def fill_c(kernels, c, data, row0):
    if data.seed_c is None:
        c.zero_()
    else:
        kernels.fill_normal(c, data.seed_c, 0.0, 1.0, offset=row0 * c.shape[1])


def gemm_operands(kernels, dev, M, row0, data, b="fill"):
    """A (rows row0.. of the configuration's A), B and C of one rank, from
    the seeded streams, in HBM.  b: "fill" generates B, "empty" only
    allocates it (a replica to be copied into), None leaves it out."""
    import torch
    a = torch.empty(M, K_DIM, dtype=torch.float16, device=dev)
    kernels.fill_normal(a, data.seed_a, 0.0, OPERAND_STD, offset=row0 * K_DIM)
    bt = None
    if b is not None:
        bt = torch.empty(K_DIM, N_DIM, dtype=torch.float16, device=dev)
        if b == "fill":
            kernels.fill_normal(bt, data.seed_b, 0.0, OPERAND_STD)
    c = torch.empty(M, N_DIM, dtype=torch.float32, device=dev)
    fill_c(kernels, c, data, row0)
    return a, bt, c


def check_rows(M):
    """Rows of a shard on both sides of the CTA (128) and pair-tile (256)
    boundaries at its start, middle and end."""
    rows = {0, 1, 127, 128, 255, 256, M // 2 - 1, M // 2, M - 257, M - 256, M - 2, M - 1}
    return sorted(r for r in rows if 0 <= r < M)


def gemm_parity(world, rank, dev, kernels, a, b, c, row0, data):
    """Restores C, runs one step and checks the sampled rows of this rank's C
    against the oracle's fp32 product of the oracle's own operands
    (mirroring the reference test's launch, download, compare with the CPU
    loop: advanced_test.go:476-483).  The device's operands are checked bit
    for bit against the oracle's streams: sampled rows of A and B on every
    rank, the whole of B on rank 0, and every rank's B against rank 0's."""
    import numpy as np
    import torch
    o = oracle_mod()
    M, K = a.shape
    N = b.shape[1]
    fill_c(kernels, c, data, row0)
    kernels.gemm(a, b, c)
    torch.cuda.synchronize()
    rows = check_rows(M)
    idx = torch.tensor(rows, device=dev)
    got = c.index_select(0, idx).cpu().numpy()
    a_dev = a.index_select(0, idx).cpu().view(torch.int16).numpy().view(np.uint16)
    b_h = b.cpu().view(torch.int16).numpy().view(np.uint16)
    a16 = np.stack([o.f32_to_f16(o.normal(K, data.seed_a, 0.0, OPERAND_STD, offset=(row0 + r) * K))
                    for r in rows])
    inputs_ok = bool(np.array_equal(a_dev, a16))
    for k in (0, 1, K // 2, K - 1):
        want_row = o.f32_to_f16(o.normal(N, data.seed_b, 0.0, OPERAND_STD, offset=k * N))
        inputs_ok &= bool(np.array_equal(b_h[k], want_row))
    if rank == 0:
        inputs_ok &= bool(np.array_equal(
            b_h.ravel(), o.f32_to_f16(o.normal(K * N, data.seed_b, 0.0, OPERAND_STD))))
    digest = hashlib.sha256(b_h.tobytes()).hexdigest()
    af = o.f16_to_f32(a16)
    bf = o.f16_to_f32(b_h)
    if data.seed_c is None:
        c0 = np.zeros((len(rows), N), dtype=np.float32)
    else:
        c0 = np.stack([o.normal(N, data.seed_c, 0.0, 1.0, offset=(row0 + r) * N) for r in rows])
    threads = max(1, len(os.sched_getaffinity(0)) // world)
    want = o.gemm_ikj(af, bf, c0, threads=threads)
    rel, mx, bad = o.error_norms(got, want)
    tol_rel, tol_max = o.gemm_tolerance(K, float(np.abs(af).max()), float(np.abs(bf).max()))
    mine = {"rel": rel, "max": mx, "bad": bad, "tol_rel": tol_rel, "tol_max": tol_max,
            "inputs_ok": inputs_ok, "digest": digest, "rows": len(rows)}
    allr = gather_objects(mine, world)
    b_same = all(r["digest"] == allr[0]["digest"] for r in allr)
    out = {
        "rows_checked": sum(r["rows"] for r in allr),
        "rows_per_rank": rows,
        "rel_fro": max(r["rel"] for r in allr),
        "max_abs": max(r["max"] for r in allr),
        "bound_rel_fro": min(r["tol_rel"] for r in allr),
        "bound_max_abs": min(r["tol_max"] for r in allr),
        "non_finite": sum(r["bad"] for r in allr),
        "inputs_match_oracle": all(r["inputs_ok"] for r in allr),
        "b_same_on_all_ranks": b_same,
        "against": "oracle/oracle.c fp32 product (i-k-j) of the oracle's fp16-rounded operands",
    }
    out["ok"] = bool(out["non_finite"] == 0 and out["inputs_match_oracle"] and b_same and all(
        r["rel"] <= r["tol_rel"] and r["max"] <= r["tol_max"] for r in allr))
    return out


# ---- CPU baseline (the reference's CPU loop, restated in C) ---------------------


class CpuGemm:
    """The reference's CPU loop for this path: the i-j-k float32 GEMM of its
    tests (advanced_test.go:466-475, restated in oracle/oracle.c), over whole
    rows of the 8192 x 8192 x 8192 problem with the bench's own operands
    (seeds 6, 7, 8); rows are independent, so a sample of rows measures the
    loop's rate exactly."""

    def __init__(self, max_rows: int):
        o = oracle_mod()
        self.o = o
        self.af = o.f16_to_f32(o.f32_to_f16(
            o.normal(max_rows * K_DIM, CUBE.seed_a, 0.0, OPERAND_STD))).reshape(max_rows, K_DIM)
        self.bf = o.f16_to_f32(o.f32_to_f16(
            o.normal(K_DIM * N_DIM, CUBE.seed_b, 0.0, OPERAND_STD))).reshape(K_DIM, N_DIM)
        self.c = o.normal(max_rows * N_DIM, CUBE.seed_c).reshape(max_rows, N_DIM)

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


def cpu_secondary():
    """The reference's CPU loops for the VecAdd (2^26-element sample of the
    2^28 workload) and decode-shaped GEMM configurations, 1 thread and all
    host threads."""
    o = oracle_mod()
    T = o.num_threads()
    out = {}
    n = 1 << 26
    a, b = o.uniform(n, 4), o.uniform(n, 5)
    for t in (1, T):
        best = float("inf")
        for _ in range(2):  # the second call reuses the output pages the first one touched
            t0 = time.perf_counter()
            o.vecadd(a, b, threads=t)
            best = min(best, time.perf_counter() - t0)
        out[f"vecadd_GB/s_{'1thread' if t == 1 else 'all'}"] = 12 * n / best / 1e9
    sm, sn, sk = SKINNY
    af, bf, c = skinny_host_operands(o)
    for t in (1, T):
        t0 = time.perf_counter()
        o.gemm_ikj(af, bf, c, threads=t)
        out[f"skinny_ms_{'1thread' if t == 1 else 'all'}"] = (time.perf_counter() - t0) * 1e3
    out["threads"] = T
    out["sample"] = "VecAdd: 2^26 elements; decode GEMM: the whole 16x14336x4096 (i-k-j float32 loop)"
    return out


def skinny_host_operands(o):
    """The decode-shaped GEMM's operands as the oracle generates them: A
    fp16(N(0,1)) seed 9, B fp16(N(0,0.02)) seed 10, C = 0 (fp32 copies of
    the fp16 values)."""
    sm, sn, sk = SKINNY
    af = o.f16_to_f32(o.f32_to_f16(o.normal(sm * sk, 9, 0.0, 1.0))).reshape(sm, sk)
    bf = o.f16_to_f32(o.f32_to_f16(o.normal(sk * sn, 10, 0.0, 0.02))).reshape(sk, sn)
    import numpy as np
    return af, bf, np.zeros((sm, sn), dtype=np.float32)


def run_reference(args, world, rank):
    """The reference arm: the CPU i-j-k loop on all host threads, rank 0 only;
    each step computes one row per thread of the workload."""
    if rank != 0:
        return
    o = oracle_mod()
    threads = o.num_threads()
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
    data = CUBE if n_gpus == 1 else SHARDED
    return {"workload": "row-sharded MatMul16 GEMM C=A.B+C (fp16 A,B; fp32 C, fp32 accumulate)",
            "M": ROWS_PER_GPU * n_gpus, "N": N_DIM, "K": K_DIM, "rows_per_gpu": ROWS_PER_GPU,
            "partition": "row blocks of A and C; B replicated by peer copy",
            "operands": data.describe(),
            "l2": "inputs exceed L2 (512 MiB per GPU vs 126 MB)",
            "secondary": {"vecadd_n_per_gpu": VEC_N, "skinny_MNK": list(SKINNY),
                          "strong_scaling_M": STRONG_M}}


# ---- our arm -------------------------------------------------------------------------


def pinned_copy(t):
    """A page-locked host copy of a device tensor."""
    import torch
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    h.copy_(t)
    return h


def copies_only_ms(h2d, d2h, steps, world, dev):
    """The step's host copies alone: every H2D (dst, src) pair on one stream
    and every D2H on another, concurrently, as the host entries issue them;
    the time the host link needs for the step's bytes."""
    import torch
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    cur = torch.cuda.current_stream()

    def step():
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_in):
            for dst, src in h2d:
                dst.copy_(src, non_blocking=True)
        with torch.cuda.stream(s_out):
            for dst, src in d2h:
                dst.copy_(src, non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)

    return time_steps(step, steps, 2, world, dev)


def run_e2e(args, world, rank, dev, a, b, c, flops, kernels):
    """The GEMM step from pinned host buffers through the C ABI's host entry
    (cudair_gemm_f16f32_host): every step copies A, B and C in, multiplies
    and copies C back to the host, all inside the timed region, with the
    copies of one tile overlapping the GEMM of another.  With several GPUs,
    B (the same on every rank) is not sent over every host link in full: each
    rank copies 1/world of its rows in, and an all-gather over NVLink
    assembles B on every GPU before the host entry takes over.  The parts are
    also timed alone, and so are the step's copies without the GEMM."""
    import torch
    a_h, b_h, c_h = pinned_copy(a), pinned_copy(b), pinned_copy(c)
    a_d, b_d, c_d = torch.empty_like(a), torch.empty_like(b), torch.empty_like(c)
    K = b.shape[0]
    steps = max(3, min(args.steps, 20))
    breakdown = {}
    if world > 1 and K % world == 0:
        import torch.distributed as dist
        rows = K // world
        b_h_part = b_h[rank * rows:(rank + 1) * rows]
        b_part = torch.empty(rows, b.shape[1], dtype=b.dtype, device=dev)

        def b_in():
            b_part.copy_(b_h_part, non_blocking=True)

        def b_gather():
            dist.all_gather_into_tensor(b_d.view(-1), b_part.view(-1))

        def gemm_from_host():
            kernels.gemm_host(a_h, None, c_h, a_d, b_d, c_d)

        def e2e_step():
            b_in()
            b_gather()
            gemm_from_host()

        b_bytes = b_part.numel() * 2
        api = ("B: 1/world of its rows per rank over the host link, all-gathered over NVLink; "
               "then cudair_gemm_f16f32_host (row blocks: H2D, GEMM and D2H overlapped; "
               "B is already on the device)")
        breakdown["b_h2d_ms"] = time_steps(b_in, 3, 2, world, dev)
        breakdown["b_allgather_ms"] = time_steps(b_gather, 3, 2, world, dev)
        breakdown["a_c_in_gemm_c_out_ms"] = time_steps(gemm_from_host, 3, 2, world, dev)
        h2d = [(a_d, a_h), (b_part, b_h_part), (c_d, c_h)]
    else:
        def e2e_step():
            kernels.gemm_host(a_h, b_h, c_h, a_d, b_d, c_d)

        b_bytes = b_h.numel() * 2
        api = ("cudair_gemm_f16f32_host (4 x 4 tiles of 2048 x 2048: B by column blocks, A by row "
               "blocks, C by tiles; H2D, GEMM and D2H overlapped)")
        h2d = [(a_d, a_h), (b_d, b_h), (c_d, c_h)]
    c_back = torch.empty(c.shape, dtype=c.dtype, pin_memory=True)
    breakdown["copies_only_ms"] = copies_only_ms(h2d, [(c_back, c_d)], 3, world, dev)
    ms = time_steps(e2e_step, steps, 3, world, dev)
    breakdown["link_bound_frac"] = breakdown["copies_only_ms"] / ms
    h2d_bytes = a_h.numel() * 2 + b_bytes + c_h.numel() * 4
    d2h_bytes = c_h.numel() * 4
    breakdown["host_link_GB/s_per_gpu"] = (h2d_bytes + d2h_bytes) / (breakdown["copies_only_ms"] * 1e-3) / 1e9
    del a_h, b_h, c_h, a_d, b_d, c_d, c_back
    return {"value": flops * world / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes, "ms_per_step": ms,
            "steps": steps, "api": api, "breakdown": breakdown}


def run_gather(world, dev, c):
    """Reassembly of C on every GPU with an NCCL all-gather over NVLink (not
    part of the step; timed on its own)."""
    import torch
    import torch.distributed as dist
    M, N = c.shape
    full = torch.empty(world * M, N, dtype=torch.float32, device=dev)
    t = time_steps(lambda: dist.all_gather_into_tensor(full, c), 5, 3, world, dev)
    got = (world - 1) * M * N * 4
    gbs = got / (t * 1e-3) / 1e9
    del full
    return {"ms": t, "bytes_received_per_gpu": got, "GB/s_per_gpu": gbs,
            "frac_of_nvlink_900": gbs / NVLINK_GBS, "frac_of_peer_copy_770": gbs / PEER_COPY_GBS}


def run_strong(world, rank, dev, kernels, b_sharded):
    """The M = 65536, N = K = 8192 row-sharded GEMM (A seed 11, B seed 12,
    C = 0) as strong scaling: each rank times its 1/N row block, and rank 0
    alone also times the whole problem on its GPU (t1), so
    eff = t1 / (N tN) comes from one job."""
    import torch
    from cudair import multigpu
    r0, r1 = multigpu.row_block(STRONG_M, world, rank)
    if b_sharded is None:
        b_sharded = torch.empty(K_DIM, N_DIM, dtype=torch.float16, device=dev)
        kernels.fill_normal(b_sharded, SHARDED.seed_b, 0.0, OPERAND_STD)
    a, _, c = gemm_operands(kernels, dev, r1 - r0, r0, SHARDED, b=None)
    if world > 1 and rank == 0:
        a1, _, c1 = gemm_operands(kernels, dev, STRONG_M, 0, SHARDED, b=None)
    # The two are timed in turn, three times, and each median is kept: a
    # GPU's clock under its power limit drifts between runs of this length.
    tns, t1s = [], []
    for _ in range(3):
        tns.append(time_steps(lambda: kernels.gemm(a, b_sharded, c), 5, 3, world, dev))
        if world > 1:
            t1 = 0.0
            if rank == 0:
                t1 = time_steps(lambda: kernels.gemm(a1, b_sharded, c1), 5, 3, 1, dev)
            barrier(world)
            t1s.append(max_over_ranks(t1, world, dev))
    del a, c
    if world > 1 and rank == 0:
        del a1, c1
    torch.cuda.empty_cache()
    tn = statistics.median(tns)
    t1 = statistics.median(t1s) if world > 1 else tn
    flops = 2.0 * STRONG_M * N_DIM * K_DIM
    return {"M": STRONG_M, "t1_ms": t1, "tN_ms": tn, "eff": t1 / (world * tn),
            "TFLOP/s_aggregate": flops / (tn * 1e-3) / 1e12, "rows_per_gpu": r1 - r0,
            "timing": "medians of 3 alternating runs of 5 launches (t1 on rank 0's GPU alone)"}


def run_vecadd(args, world, rank, dev, kernels, peaks, traffic):
    """VecAdd over n = 2^28 fp32 per GPU (3 GiB of traffic per step, > L2): a
    and b are U(-1,1) seeds 4 and 5 at the rank's offset (ranks hold
    contiguous ranges of one 2^28 N vector).  Checked bit for bit against the
    oracle's add on three slices; e2e through cudair_vecadd_host."""
    import numpy as np
    import torch
    o = oracle_mod()
    off = rank * VEC_N
    va = torch.empty(VEC_N, device=dev)
    vb = torch.empty(VEC_N, device=dev)
    kernels.fill_uniform(va, 4, -1.0, 1.0, offset=off)
    kernels.fill_uniform(vb, 5, -1.0, 1.0, offset=off)
    vo = torch.empty_like(va)
    ms = time_steps(lambda: kernels.vecadd(va, vb, vo), args.steps, args.warmup, world, dev)
    gbs = 3 * 4 * VEC_N / (ms * 1e-3) / 1e9
    ok = True
    for s0 in (0, VEC_N // 2 - 77, VEC_N - (1 << 16)):
        n = 1 << 16
        want = o.vecadd(o.uniform(n, 4, offset=off + s0), o.uniform(n, 5, offset=off + s0))
        ok &= bool(np.array_equal(vo[s0:s0 + n].cpu().numpy(), want))
    # e2e: host buffers in, the sum back in host memory.
    a_h, b_h = pinned_copy(va), pinned_copy(vb)
    o_h = torch.empty(VEC_N, pin_memory=True)
    d_a, d_b, d_o = torch.empty_like(va), torch.empty_like(va), torch.empty_like(va)
    e2e_steps = max(3, min(args.steps, 5))
    e2e_ms = time_steps(lambda: kernels.vecadd_host(a_h, b_h, o_h, d_a, d_b, d_o), e2e_steps, 3, world, dev)
    e2e_ok = bool(torch.equal(o_h[: 1 << 20], vo[: 1 << 20].cpu()) and torch.equal(o_h[-(1 << 20):],
                                                                                  vo[-(1 << 20):].cpu()))
    copies = copies_only_ms([(d_a, a_h), (d_b, b_h)], [(o_h, d_o)], 3, world, dev)
    del va, vb, vo, a_h, b_h, o_h, d_a, d_b, d_o
    torch.cuda.empty_cache()
    parity_all = all(gather_objects(ok and e2e_ok, world))
    hbm = peaks["hbm_gbs"]
    return {"value": gbs * world, "unit": "GB/s", "ms_per_step": ms, "n_per_gpu": VEC_N,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "traffic": traffic.get("vecadd_2p28"), "frac_of_nominal": gbs / 8000.0},
            "parity": {"ok": parity_all, "checked": "3 slices of 2^16 per rank bit for bit against the "
                                                    "oracle's add, and the e2e result against the device's"},
            "e2e": {"value": 12 * VEC_N * world / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": 8 * VEC_N, "d2h_bytes_per_step": 4 * VEC_N, "ms_per_step": e2e_ms,
                    "steps": e2e_steps, "api": "cudair_vecadd_host (about 16 chunks: H2D, VecAdd, D2H overlapped)",
                    "copies_only_ms": copies, "link_bound_frac": copies / e2e_ms}}


def run_saxpy_square(args, world, rank, dev, kernels, peaks):
    """Saxpy (12 bytes per element: read x and y, write y) and Square (8: read
    and write x) over n = 2^28 fp32 per GPU, each step one launch; x, y are
    U(-1,1) from seeds 4 and 5."""
    import torch
    x = torch.empty(VEC_N, device=dev)
    y = torch.empty(VEC_N, device=dev)
    kernels.fill_uniform(x, 4, -1.0, 1.0, offset=rank * VEC_N)
    kernels.fill_uniform(y, 5, -1.0, 1.0, offset=rank * VEC_N)
    ms_saxpy = time_steps(lambda: kernels.saxpy(0.5, x, y), args.steps, args.warmup, world, dev)
    ms_square = time_steps(lambda: kernels.square(x), args.steps, args.warmup, world, dev)
    del x, y
    out = {}
    for name, ms, per in (("saxpy", ms_saxpy, 12), ("square", ms_square, 8)):
        gbs = per * VEC_N / (ms * 1e-3) / 1e9
        out[name] = {"value": gbs * world, "unit": "GB/s", "ms_per_step": ms, "n_per_gpu": VEC_N,
                     "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                  "frac": gbs / peaks["hbm_gbs"]}}
    return out


def run_skinny(args, world, rank, dev, kernels, peaks, traffic):
    """M=16, N=14336, K=4096 (decode-shaped; A fp16(N(0,1)) seed 9, B
    fp16(N(0,0.02)) seed 10, C = 0): B is 117 MB, so three copies of it are
    cycled (351 MB > L2) and every launch streams its B from HBM.  A decode
    step issues such GEMMs back to back from a captured CUDA graph, so 30
    launches are captured once and the graph replays are timed with events
    (per launch: replay time / 30); a launch timed alone from Python would
    measure the host's launch cost, which exceeds the kernel's time.  The
    launches use programmatic dependent launch with B requested before the
    dependency wait (cudair_set_gemm_pdl(2)): B is never written in the chain.
    Parity: one launch on C = 0 against the oracle's product; e2e through
    cudair_gemm_f16f32_host."""
    import torch
    o = oracle_mod()
    sm, sn, sk = SKINNY
    sa = torch.empty(sm, sk, dtype=torch.float16, device=dev)
    kernels.fill_normal(sa, 9, 0.0, 1.0)
    sbs = []
    for _ in range(3):
        t = torch.empty(sk, sn, dtype=torch.float16, device=dev)
        kernels.fill_normal(t, 10, 0.0, 0.02)
        sbs.append(t)
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
    del graph
    ms = max_over_ranks(statistics.median(times), world, dev)
    alg_bytes = sk * sn * 2 + sm * sk * 2 + 2 * sm * sn * 4
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    # parity
    sc.zero_()
    kernels.gemm(sa, sbs[0], sc)
    af, bf, c0 = skinny_host_operands(o)
    want = o.gemm_ikj(af, bf, c0)
    rel, mx, bad = o.error_norms(sc.cpu().numpy(), want)
    tol_rel, tol_max = o.gemm_tolerance(sk, float(abs(af).max()), float(abs(bf).max()))
    inputs_ok = bool((sa.cpu().view(torch.int16).numpy().view("uint16") ==
                      o.f32_to_f16(o.normal(sm * sk, 9, 0.0, 1.0)).reshape(sm, sk)).all())
    parity = {"rel_fro": rel, "max_abs": mx, "bound_rel_fro": tol_rel, "bound_max_abs": tol_max,
              "inputs_match_oracle": inputs_ok, "ok": bool(bad == 0 and inputs_ok and rel <= tol_rel
                                                           and mx <= tol_max)}
    # e2e: A, B, C from pinned host memory, C back.
    a_h, b_h, c_h = pinned_copy(sa), pinned_copy(sbs[0]), pinned_copy(torch.zeros_like(sc))
    a_d, b_d, c_d = torch.empty_like(sa), torch.empty_like(sbs[0]), torch.empty_like(sc)
    e2e_steps = max(3, min(args.steps, 10))
    e2e_ms = time_steps(lambda: kernels.gemm_host(a_h, b_h, c_h, a_d, b_d, c_d), e2e_steps, 3, world, dev)
    h2d = sm * sk * 2 + sk * sn * 2 + sm * sn * 4
    del sa, sbs, sc, a_h, b_h, c_h, a_d, b_d, c_d
    torch.cuda.empty_cache()
    return {"M": sm, "N": sn, "K": sk, "ms": ms, "GB/s": gbs,
            "timing": "CUDA graph of 30 launches cycling 3 copies of B, per launch; "
                      "programmatic dependent launch, B requested before the wait",
            "TFLOP/s": 2.0 * sm * sn * sk / (ms * 1e-3) / 1e12,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"],
                         "traffic": traffic.get("skinny_16x14336x4096")},
            "parity": parity,
            "e2e": {"value": 2.0 * sm * sn * sk / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": sm * sn * 4, "ms_per_step": e2e_ms,
                    "steps": e2e_steps, "api": "cudair_gemm_f16f32_host"}}


def run_matmul16_n256(dev, kernels):
    """The MatMul16 parity configuration (n = 256, the reference test's size;
    A, B fp16(U(-1,1)) seeds 1, 2 and C U(-1,1) seed 3): per-launch latency
    of the module entry under the reference's launch (grid (n/16, n/16) x
    32 threads) and of the library's cudair_matmul16, each from a CUDA graph
    of 20 launches (a single launch timed from Python measures the host's
    launch cost); the result against the oracle's i-j-k loop (which is also
    timed, as this configuration's CPU baseline); and e2e, the test's whole
    flow (copies in, launch, copy out) through cudair_matmul16_host."""
    import ctypes

    import numpy as np
    import torch
    from cudair import host
    o = oracle_mod()
    n = 256
    a = torch.empty(n, n, dtype=torch.float16, device=dev)
    b = torch.empty(n, n, dtype=torch.float16, device=dev)
    c = torch.empty(n, n, device=dev)
    kernels.fill_uniform(a, 1)
    kernels.fill_uniform(b, 2)
    kernels.fill_uniform(c, 3)
    c_init = c.clone()
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
    # parity: one launch of each path on the initial C against the oracle's
    # i-j-k loop (the loop is also this configuration's CPU baseline)
    af = o.f16_to_f32(o.f32_to_f16(o.uniform(n * n, 1))).reshape(n, n)
    bf = o.f16_to_f32(o.f32_to_f16(o.uniform(n * n, 2))).reshape(n, n)
    c0 = o.uniform(n * n, 3).reshape(n, n)
    t0 = time.perf_counter()
    want = o.gemm_ijk(af, bf, c0, threads=1)
    out["cpu_us_1thread"] = (time.perf_counter() - t0) * 1e6
    tol_rel, tol_max = o.gemm_tolerance(n, 1.0, 1.0)
    ok = bool(np.array_equal(c_init.cpu().numpy(), c0))
    worst = 0.0
    cur = torch.cuda.current_stream()
    for launch in (lambda: fn.LaunchExOn(cur, cfg, host.LaunchAttrs(), *args),
                   lambda: kernels.matmul16(a, b, c)):
        c.copy_(c_init)
        launch()
        torch.cuda.synchronize()
        rel, mx, bad = o.error_norms(c.cpu().numpy(), want)
        ok &= bad == 0 and rel <= tol_rel and mx <= tol_max
        worst = max(worst, rel)
    mod.Close()
    out["parity"] = {"ok": bool(ok), "rel_fro_worst": worst, "bound_rel_fro": tol_rel,
                     "against": "oracle i-j-k loop (advanced_test.go:466-475 restated)"}
    # e2e: host buffers in, C back in host memory, per call.
    a_h, b_h, c_h = pinned_copy(a), pinned_copy(b), pinned_copy(c_init)
    calls = 50
    st = torch.cuda.current_stream()
    for _ in range(5):
        kernels.matmul16_host(a_h, b_h, c_h, a, b, c)
    st.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(calls):
        kernels.matmul16_host(a_h, b_h, c_h, a, b, c)
    e1.record()
    st.synchronize()
    us = e0.elapsed_time(e1) / calls * 1e3
    out["e2e"] = {"value": us, "unit": "us per call", "h2d_bytes_per_step": 2 * n * n * 2 + n * n * 4,
                  "d2h_bytes_per_step": n * n * 4, "api": "cudair_matmul16_host (copies in, launch, copy out)"}
    out["timing"] = "CUDA graph of 20 launches, per launch; CPU: the i-j-k loop, 1 thread"
    return out


def run_ours(args, world, rank, local):
    import torch
    from cudair import kernels

    dev = torch.device("cuda", local)
    cpus = bind_host_to_gpu(local)
    kernels.set_gemm_variant(args.gemm_variant)
    peaks, peak_kind = load_peaks()
    traffic = load_traffic()
    only = args.workload

    if only == "vecadd":
        v = run_vecadd(args, world, rank, dev, kernels, peaks, traffic)
        log(f"rank {rank}: vecadd {v['ms_per_step']:.4f} ms/step {v['roofline']['achieved']:.1f} GB/s")
        return
    if only == "skinny":
        s = run_skinny(args, world, rank, dev, kernels, peaks, traffic)
        log(f"rank {rank}: skinny {s['ms']:.4f} ms {s['GB/s']:.1f} GB/s")
        return

    # -- the row-sharded GEMM: inputs resident in HBM, from the seeded streams
    data = CUBE if world == 1 else SHARDED
    M, N, K = ROWS_PER_GPU, N_DIM, K_DIM
    row0 = rank * ROWS_PER_GPU
    a, b, c = gemm_operands(kernels, dev, M, row0, data, b="fill" if rank == 0 else "empty")
    torch.cuda.synchronize()
    b_ms = replicate_b(b, world, rank, dev)

    flops = 2.0 * M * N * K
    sampler = ClockSampler(local)
    ms = time_steps(lambda: kernels.gemm(a, b, c), args.steps, args.warmup, world, dev, sampler)
    clocks = sampler.summary()
    kernels.wait_status(clear=True)
    achieved = flops / (ms * 1e-3) / 1e12
    log(f"rank {rank}: gemm {ms:.4f} ms/step, {achieved:.1f} TFLOP/s per GPU")
    parity = gemm_parity(world, rank, dev, kernels, a, b, c, row0, data)
    log(f"rank {rank}: parity {parity['ok']} rel {parity['rel_fro']:.3g} max {parity['max_abs']:.3g}")
    if only == "gemm":
        return

    # The strong-scaling GEMMs run at the power limit; the host-link-bound
    # e2e leg after them lets the clocks recover before the HBM-bound legs.
    strong = run_strong(world, rank, dev, kernels, b if data is SHARDED else None)
    e2e = run_e2e(args, world, rank, dev, a, b, c, flops, kernels)
    gather = run_gather(world, dev, c) if world > 1 else None
    del a, b, c
    torch.cuda.empty_cache()
    vecadd = run_vecadd(args, world, rank, dev, kernels, peaks, traffic)
    streams = run_saxpy_square(args, world, rank, dev, kernels, peaks)
    skinny = run_skinny(args, world, rank, dev, kernels, peaks, traffic)
    kernels.wait_status(clear=True)

    # -- the n = 256 parity configuration and the CPU baselines (rank 0)
    mm256 = run_matmul16_n256(dev, kernels) if (rank == 0 and world == 1) else None
    cpu = None
    cpu_more = None
    if rank == 0 and not args.no_cpu:
        if world == 1:
            cpu_more = cpu_secondary()
        budget = args.cpu_budget if world == 1 else min(args.cpu_budget, 4.0)
        r, rows, dt = CpuGemm(max_rows=256).sample(1, budget_s=budget)
        cpu = {"value": r, "unit": "TFLOP/s", "cores": 1, "kind": "port",
               "sample": f"{rows} rows of the 8192^3 C = A.B + C by the i-j-k float32 loop "
                         f"(oracle/oracle.c restating advanced_test.go:466-475), 1 thread, "
                         f"{dt:.1f} s"}
    barrier(world)

    if rank != 0:
        return
    tensor_peak = peaks["bf16_tflops"]
    line = {
        "metric": METRIC, "value": achieved * world, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: " + data.describe(),
        "config": workload_config(world),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": tensor_peak,
                     "unit": "TFLOP/s", "frac": achieved / tensor_peak,
                     "traffic": traffic.get("gemm_8192"),
                     "peak_kind": f"{peak_kind} bf16 burst (fp16 dense rate is equal)",
                     "frac_of_nominal": achieved / 2250.0},
        "parity": parity,
        "e2e": e2e,
        "cpu_baseline": cpu,
        "gpu_launches": args.steps * world,
        "clocks": clocks,
        "host_cpus_bound": cpus,
        "b_replication_ms": b_ms,
        "strong_scaling": strong,
        "gather": gather,
        "matmul16_n256": mm256,
        "cpu_secondary": cpu_more,
        "vecadd": vecadd,
        **streams,
        "skinny": skinny,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
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
