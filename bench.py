"""MatMulNBits INT4 benchmark on B200 (one JSON line on rank 0).

Headline: the 7B-shaped decode GEMV sweep at M=1, block_size 128, fp32
A ~ N(0,1), packed uint4 zero points, fp32 scales U[0.001, 0.01], shapes (K, N) = (4096, 4096),
(4096, 1024), (4096, 14336), (14336, 4096), (4096, 32000). One step = one MatMulNBits op per
shape (5 ops, 144 216 064 algorithmic bytes: weights + scales + zero points as the reference
stores them). value = algorithmic GB/s of the whole job.

* value     inputs resident in HBM; each step is one CUDA-graph replay of the 5 launches; 4
            weight replicas rotate so the 577 MB working set exceeds the 126 MB L2. Timed as
            --windows windows of exactly --steps steps (each bracketed by a barrier and a
            synchronize); value from the median window, the spread in config.timing.
* per_M     the same sweep at M = 4 and M = 16 (configs[1]'s batched rows; same weight bytes).
* e2e       the same ops through the C-ABI host-buffer entry (msq_matmul_host_async per op, the ops
            alternating over two streams, both synchronized per step; beside it one stream, and
            msq_matmul_host, synchronous per op): pinned host
            A copied in and Y copied out inside the timed region, every step.
* roofline  the decode GEMV kernel: algorithmic bytes / its CUDA-event launch duration vs
            the measured HBM copy bandwidth (MEASURED_PEAKS.json).
* cpu_baseline  the reference's own ms_qgemm_nbits (oracle/_ref, built from the reference
            sources) on this host's cores over whole sweeps for ~10 s.
* sub       at N = 1 the other two headline metrics, each a full record of its own (timing,
            clocks, parity, roofline, CPU baseline, e2e): "prefill" (configs[2], TFLOP/s of the
            tcgen05 GEMM at M = 512 / 2048 / 8192) and "decode7b" (configs[4], tok/s of the
            synthetic 7B decoder, 128 greedy tokens after a 512-token prompt, every token checked
            against the CPU checker); and "layers70b_m32" (configs[3] at M = 32 on one GPU: the
            up and down projections of the 70B MLP, GB/s). --no-sub skips them.

Multi-GPU (torchrun, N > 1): the sweep column-split over the ranks: every shape's rows are
sharded, each shard's GEMV stores its outputs into every rank's full Y over NVLink, and each op
waits on the device for all ranks' shards of the previous op's Y (strong scaling, max over
ranks). --impl reference times the reference CPU kernel as the arm itself (rank 0 only, all host
threads). --workload prefill / nsplit70b / decode7b run one of the other configs alone.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SWEEP = [(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096), (4096, 32000)]  # (K, N)
BS = 128
SCALE_LO, SCALE_HI = 0.001, 0.01
REPLICAS = 4
METRIC = "MatMulNBits INT4 M=1 HBM GB/s"
WORKLOAD = ("7B decode GEMV sweep (BASELINE configs[1]) at M=1: (K,N) = (4096,4096), (4096,1024), "
            "(4096,14336), (14336,4096), (4096,32000); bits=4, block_size=128, packed zero points, fp32 A and "
            "scales")
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) per algorithmic byte of the decode GEMV, measured by an ncu
# capture of one K=4096, N=14336 launch of this bench's sweep.
NCU_DRAM_PER_ALG_BYTE = 31480064 / 31424512


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def make_cases(seed0: int = 0):
    from modelsharp_b200 import synth
    return [synth.make_case(seed0 + i, 1, N, K, 4, BS, "packed", a_dist="normal",
                            scale_lo=SCALE_LO, scale_hi=SCALE_HI) for i, (K, N) in enumerate(SWEEP)]


def step_bytes() -> int:
    from modelsharp_b200 import synth
    return sum(synth.algorithmic_bytes(N, K, 4, BS, "packed") for K, N in SWEEP)


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def tensor_peak() -> tuple[float, str]:
    """Dense bf16 tensor peak for kernels timed inside a long step: the measured sustained cuBLAS
    rate, else the fallback sustained figure."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops_sustained"]), "measured sustained cuBLAS bf16"
        except Exception:
            pass
    return 1400.0, "fallback sustained bf16"


def burst_tensor_peak() -> tuple[float, str]:
    """Dense bf16 tensor peak for a kernel timed in isolation: the measured burst cuBLAS rate."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured burst cuBLAS bf16"
        except Exception:
            pass
    return 1590.0, "fallback burst bf16"


def timed_windows(args, world: int, dev, stream, replay) -> list[float]:
    """args.windows timed windows of exactly args.steps calls of replay(i) on `stream`, each
    bracketed by a barrier and a synchronize; CUDA-event ms per window, max over ranks."""
    import torch
    import torch.distributed as dist
    out = []
    i = 0
    for _ in range(args.windows):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                replay(i)
                i += 1
        e1.record(stream)
        torch.cuda.synchronize(dev)
        out.append(e0.elapsed_time(e1))
    if world > 1:
        t = torch.tensor(out, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out = [float(v) for v in t.tolist()]
    return out


def window_stats(wins: list[float]) -> tuple[float, dict]:
    """Median window (ms) and the spread of all windows in ms per window."""
    srt = sorted(wins)
    q = lambda f: srt[min(len(srt) - 1, int(f * (len(srt) - 1) + 0.5))]
    return statistics.median(srt), {"windows": len(srt), "ms_per_window": {
        "median": statistics.median(srt), "min": srt[0], "p10": q(0.1), "p90": q(0.9), "max": srt[-1]}}


# ---------------------------------------------------------------- clocks (NVML, in-process)
class ClockSampler:
    """Samples SM clock and throttle reasons every ~2 ms on a background thread."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: report nothing rather than guess
            log(f"clock sampling unavailable: {e}")

    def _sample(self):
        nv = self._nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
        r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        for bit, name in self.REASONS.items():
            if r & bit and name != "gpu_idle":
                self.reasons.add(name)

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(0.002)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._h is not None:
            self._stop.set()
            self._t.join()
            self._sample()

    def summary(self):
        if not self.samples:
            return None
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------- CPU reference timing
def time_reference_sweep(cases, budget_s: float, min_reps: int = 2):
    """Whole sweeps of the reference's ms_qgemm_nbits on all host cores; returns (median s, reps, kind)."""
    from oracle import oracle
    if oracle.reference_available():
        fn, kind = oracle.reference_native, "reference"
    else:
        fn, kind = oracle.managed, "port"
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < min_reps or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        for c in cases:
            fn(c)
        times.append(time.perf_counter() - t0)
        if len(times) >= 1000:
            break
    return statistics.median(times), len(times), kind


def use_all_host_threads() -> int:
    """OpenMP over every host thread for the CPU reference, also under torchrun (which sets
    OMP_NUM_THREADS=1 for its workers): the env var for libraries not yet loaded, and
    omp_set_num_threads for the process's libgomp."""
    n = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        gomp = C.CDLL("libgomp.so.1")
        gomp.omp_set_num_threads(n)
        return int(gomp.omp_get_max_threads())
    except OSError:
        return n


def run_reference_arm(args, rank: int, world: int):
    if rank != 0:
        return
    threads = use_all_host_threads()
    cases = make_cases()
    nbytes = step_bytes()
    from oracle import oracle
    kind = "reference" if oracle.reference_available() else "port"
    fn = oracle.reference_native if kind == "reference" else oracle.managed
    for _ in range(max(args.warmup, 1)):
        for c in cases:
            fn(c)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for c in cases:
            fn(c)
    dt = time.perf_counter() - t0
    value = nbytes * args.steps / dt / 1e9
    cores = threads
    out = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "bytes_per_step": nbytes},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": f"{args.steps} whole sweeps of ms_qgemm_nbits, OpenMP over all {cores} host "
                                   "threads (native/src/qgemm.cpp built from the reference sources)"
                         if kind == "reference" else f"{args.steps} whole sweeps of the C restatement"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------- GPU arm
def run_ours(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    from modelsharp_b200 import QuantizedWeights
    from modelsharp_b200 import _native as N

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib = N.lib()
    nbytes = step_bytes()
    cases = make_cases()

    # Device-resident weights: REPLICAS independent packs of each shape.
    stream = torch.cuda.Stream(dev)
    reps = []
    for r in range(REPLICAS):
        reps.append([QuantizedWeights(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, BS, device=dev)
                     for c in cases])
    a_dev = [torch.from_numpy(c["a"]).to(dev) for c in cases]
    y_dev = [torch.empty(1, c["N"], device=dev) for c in cases]
    torch.cuda.synchronize(dev)
    sptr = stream.cuda_stream

    def launch_step(r: int):
        for w, a, y, c in zip(reps[r], a_dev, y_dev, cases):
            rc = lib.msq_matmul(None, sptr, w.handle, a.data_ptr(), N.DT_F32, 1, y.data_ptr(), c["N"])
            if rc:
                N.check(rc)

    # Warm-up (also sets kernel attributes before capture), then one graph per replica.
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            launch_step(i % REPLICAS)
    stream.synchronize()
    path = N.last_path()
    graphs = []
    launches_before = N.launch_count()
    for r in range(REPLICAS):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            launch_step(r)
        graphs.append(g)
    launches_per_step = (N.launch_count() - launches_before) // REPLICAS
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            graphs[i % REPLICAS].replay()
    stream.synchronize()

    # Parity spot check of this exact data (not timed).
    y_chk = [y.cpu().numpy() for y in y_dev]

    # ---- timed region: args.windows windows of exactly K graph replays, each bracketed by a
    # barrier and a synchronize; value from the median window (max over ranks per window)
    with ClockSampler(local_rank) as clk:
        wins = timed_windows(args, world, dev, stream, lambda i: graphs[i % REPLICAS].replay())
    ms, spread = window_stats(wins)
    value = world * nbytes * args.steps / (ms * 1e-3) / 1e9

    # ---- roofline. Every launch of the timed region is the decode GEMV, so its average
    # launch duration there is ms_per_step / launches_per_step and the algorithmic bytes per
    # launch are bytes_per_step / launches_per_step. Per-shape figures come from one CUDA
    # graph per shape of 2 * REPLICAS back-to-back launches (the same launch chaining as the
    # step), timed with CUDA events on the launching stream.
    from modelsharp_b200 import synth
    per_shape = []
    for si, c in enumerate(cases):
        b = synth.algorithmic_bytes(c["N"], c["K"], 4, BS, "packed")
        g = torch.cuda.CUDAGraph()
        n_in = 2 * REPLICAS
        with torch.cuda.graph(g, stream=stream):
            for it in range(n_in):
                w = reps[it % REPLICAS][si]
                rc = lib.msq_matmul(None, sptr, w.handle, a_dev[si].data_ptr(), N.DT_F32, 1, y_dev[si].data_ptr(),
                                    c["N"])
                if rc:
                    N.check(rc)
        with torch.cuda.stream(stream):
            for _ in range(3):
                g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            n_rep = 50
            for _ in range(n_rep):
                g.replay()
            e1.record(stream)
        stream.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (n_rep * n_in)
        per_shape.append({"K": c["K"], "N": c["N"], "bytes": b, "us": us, "GB/s": b / (us * 1e-6) / 1e9})
        del g
    peak, peak_kind = peaks()
    launch_us = ms * 1e3 / args.steps / launches_per_step
    bytes_per_launch = nbytes / launches_per_step
    achieved = bytes_per_launch / (launch_us * 1e-6) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": (NCU_DRAM_PER_ALG_BYTE * bytes_per_launch) if NCU_DRAM_PER_ALG_BYTE else None,
                "peak_source": f"{peak_kind} HBM copy bandwidth", "kernel": path,
                "bytes_per_launch": bytes_per_launch, "launch_us": launch_us, "per_shape": per_shape}

    # ---- configs[1] at M = 4 and 16: the same sweep, weights and bytes, more A rows; one CUDA
    # graph per replica, timed like the step (median of windows)
    per_m = []
    y_chk_m = {}
    for M in (4, 16):
        a_m = [torch.from_numpy(synth.make_case(50 + i, M, c["N"], c["K"], 4, BS, "packed")["a"]).to(dev)
               for i, c in enumerate(cases)]
        y_m = [torch.empty(M, c["N"], device=dev) for c in cases]

        def step_m(r: int):
            for w, a, y, c in zip(reps[r], a_m, y_m, cases):
                rc = lib.msq_matmul(None, sptr, w.handle, a.data_ptr(), N.DT_F32, M, y.data_ptr(), c["N"])
                if rc:
                    N.check(rc)

        with torch.cuda.stream(stream):
            step_m(0)
        stream.synchronize()
        path_m = N.last_path()
        c0 = N.launch_count()
        gm = []
        for r in range(REPLICAS):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                step_m(r)
            gm.append(g)
        launches_m = (N.launch_count() - c0) // REPLICAS
        with torch.cuda.stream(stream):
            for i in range(3):
                gm[i % REPLICAS].replay()
        wins_m = timed_windows(argparse.Namespace(windows=5, steps=args.steps), world, dev, stream,
                               lambda i: gm[i % REPLICAS].replay())
        ms_m = statistics.median(wins_m)
        y_chk_m[M] = (a_m, [y.cpu().numpy() for y in y_m])
        per_m.append({"M": M, "ms_per_step": ms_m / args.steps, "GB/s": world * nbytes * args.steps / (ms_m * 1e-3) / 1e9,
                      "launches_per_step": launches_m, "path": path_m})
        del gm

    # ---- e2e: host buffers through the C ABI, copies inside the timed region
    a_host = [torch.from_numpy(c["a"]).pin_memory() for c in cases]
    y_host = [torch.empty(1, c["N"]).pin_memory() for c in cases]
    h2d = sum(a.numel() * 4 for a in a_host)
    d2h = sum(y.numel() * 4 for y in y_host)
    e2e_steps = max(1, min(args.steps, 2000))

    stream2 = torch.cuda.Stream(dev)

    def e2e_step(r: int, mode: str):
        # "sync": msq_matmul_host, which synchronizes after every op; "one": every op's upload,
        # GEMV and download enqueued through msq_matmul_host_async on one stream, then one
        # synchronize before the host has the step's Y; "two": the same with the ops alternating
        # over two streams (one op's copies overlap the other stream's GEMV), both synchronized
        fn = lib.msq_matmul_host if mode == "sync" else lib.msq_matmul_host_async
        streams = (stream, stream2) if mode == "two" else (stream,)
        for i, (w, a, y) in enumerate(zip(reps[r], a_host, y_host)):
            rc = fn(None, streams[i % len(streams)].cuda_stream, w.handle, a.data_ptr(), N.DT_F32, 1, y.data_ptr())
            if rc:
                N.check(rc)
        if mode != "sync":
            for s_ in streams:
                s_.synchronize()

    def time_e2e(mode: str) -> tuple[float, bool]:
        for y in y_host:
            y.fill_(float("nan"))
        for i in range(max(args.warmup, 3)):
            e2e_step(i % REPLICAS, mode)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(e2e_steps):
            e2e_step(i % REPLICAS, mode)
        e1.record(stream)  # every step ended with the host waiting for both streams
        torch.cuda.synchronize(dev)
        t_ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([t_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_ms = float(t.item())
        ok = all(np.array_equal(y.numpy(), yc) for y, yc in zip(y_host, y_chk))
        return world * nbytes * e2e_steps / (t_ms * 1e-3) / 1e9, ok

    e2e_value, e2e_ok = time_e2e("two")
    e2e_one_value, e2e_one_ok = time_e2e("one")
    e2e_sync_value, e2e_sync_ok = time_e2e("sync")

    # ---- parity spot check + CPU baseline (rank 0, N = 1)
    cpu = None
    parity = None
    if rank == 0:
        from oracle import oracle
        parity = max(oracle.rel_l2(y, oracle.managed(c)) for y, c in zip(y_chk, cases))
        for pm in per_m:
            a_m, ys = y_chk_m[pm["M"]]
            pm["parity_rel_l2"] = max(oracle.rel_l2(y, oracle.managed(dict(c, a=a.cpu().numpy(), M=pm["M"])))
                                      for y, a, c in zip(ys, a_m, cases))
        if world == 1:
            med, reps_done, kind = time_reference_sweep(cases, budget_s=args.cpu_seconds)
            cores = os.cpu_count()
            cpu = {"value": nbytes / med / 1e9, "unit": "GB/s", "cores": cores, "kind": kind,
                   "sample": f"{reps_done} whole sweeps (5 ops, {nbytes} B each), median, OpenMP over all "
                             f"{cores} host threads"}

    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "bytes_per_step": nbytes, "weights": "u4 (int4 codes)",
                       "l2": f"inputs larger than L2: {REPLICAS} weight replicas rotate, "
                             f"{REPLICAS * nbytes / 1e6:.0f} MB working set vs 126 MB L2",
                       "launch": "one CUDA graph replay per step", "parity_rel_l2": parity,
                       "parallelism": f"replicas{world}", "timing": spread,
                       "per_M": per_m},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps,
                    "entry": "msq_matmul_host_async per op, ops alternating over two streams, both synchronized "
                             "per step",
                    "matches_device_run": e2e_ok,
                    "one_stream": {"value": e2e_one_value, "entry": "msq_matmul_host_async per op, one stream "
                                   "synchronize per step", "matches_device_run": e2e_one_ok},
                    "synchronous_entry": {"value": e2e_sync_value, "entry": "msq_matmul_host (synchronize per op)",
                                          "matches_device_run": e2e_sync_ok}},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
        }
    else:
        out = None
    for g in graphs:
        del g
    for rr in reps:
        for w in rr:
            w.free()
    return out


# ---------------------------------------------------------------- the sweep column-split (N > 1)
def run_split_sweep(args, rank: int, world: int, local_rank: int):
    """The configs[1] sweep split over the ranks (the default under torchrun): every shape's
    rows are sharded over the ranks (ShardedMatMulNBits), each shard's decode GEMV stores its
    outputs into every rank's full Y over NVLink (msq_matmul_gather, plain peer stores), and
    each op waits on the device for all ranks' shards of the previous op's Y before it starts,
    as a layer that reads that Y would; the step's last Y is waited for by the next step's first
    op. value = the sweep's algorithmic bytes per step over the max-over-ranks step time
    (strong scaling: the total work is fixed)."""
    import torch
    import torch.distributed as dist

    from modelsharp_b200 import QuantizedWeights, synth
    from modelsharp_b200 import _native as N
    from modelsharp_b200.nsplit import ShardedMatMulNBits

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    nbytes = step_bytes()
    cases = make_cases()
    ops = [ShardedMatMulNBits(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, BS, device=dev, gather="p2p")
           for c in cases]
    shard_bytes = nbytes / world
    reps_n = max(REPLICAS, -(-int(480e6) // int(shard_bytes)))  # the rotation exceeds L2 on every rank
    reps_n += reps_n % 2  # even: each op's two exchange buffers alternate across the graphs' wrap-around
    # weight replicas of this rank's shards; replica 0 is the op's own
    reps = [[op.weights] + [QuantizedWeights(c["b"], c["scales"], c["zp"], c["N"], c["K"], 4, BS,
                                             rows=(op.n0, op.n1), device=dev) for _ in range(reps_n - 1)]
            for op, c in zip(ops, cases)]
    a_dev = [torch.from_numpy(c["a"]).to(dev) for c in cases]
    stream = torch.cuda.Stream(dev)
    outs = [None] * len(ops)

    def step(r: int):
        for si, op in enumerate(ops):
            op.weights = reps[si][r]
            prev = ops[si - 1].out_wait  # the previous op's gathered Y (the last op's, for op 0)
            outs[si] = op(a_dev[si], wait=prev)

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(i % reps_n)
    stream.synchronize()
    c0 = N.launch_count()
    graphs = []
    for r in range(reps_n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(r)
        graphs.append(g)
    launches_per_step = (N.launch_count() - c0) // reps_n
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            graphs[i % reps_n].replay()
        ops[-1].wait_gathered()
    stream.synchronize()
    with ClockSampler(local_rank) as clk:
        wins = timed_windows(args, world, dev, stream, lambda i: graphs[i % reps_n].replay())
    ms, spread = window_stats(wins)
    value = nbytes * args.steps / (ms * 1e-3) / 1e9
    with torch.cuda.stream(stream):
        for op in ops:
            op.wait_gathered()
    stream.synchronize()
    y_chk = [o.cpu().numpy().copy() for o in outs]

    # e2e: pinned host A in and every op's gathered Y out, each step, timed with events
    a_host = [torch.from_numpy(c["a"]).pin_memory() for c in cases]
    y_host = [torch.empty(1, c["N"]).pin_memory() for c in cases]
    e2e_steps = max(1, min(args.steps, 500))

    def e2e_step(i: int):
        r = i % reps_n
        with torch.cuda.stream(stream):
            for si, op in enumerate(ops):
                op.weights = reps[si][r]
                y = op(a_host[si].to(dev, non_blocking=True), wait=ops[si - 1].out_wait)
                op.wait_gathered()
                y_host[si].copy_(y, non_blocking=True)

    for i in range(3):
        e2e_step(i)
    stream.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record(stream)
    stream.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = nbytes * e2e_steps / (e2e_ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    per_rank = shard_bytes / (ms / args.steps * 1e-3) / 1e9
    out = None
    if rank == 0:
        from oracle import oracle
        parity = max(oracle.rel_l2(y, oracle.managed(c)) for y, c in zip(y_chk, cases))
        out = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD + f"; every shape column-split over {world} ranks, Y assembled on every "
                                              "rank by peer stores", "bytes_per_step": nbytes,
                       "weights": "u4 (int4 codes)", "parallelism": f"nsplit{world}",
                       "l2": f"inputs larger than L2: {reps_n} replicas of each rank's shards rotate "
                             f"({reps_n * shard_bytes / 1e6:.0f} MB per rank vs 126 MB L2)",
                       "launch": f"one CUDA graph replay per step: {launches_per_step} decode-GEMV launches, each "
                                 "storing its shard into every rank's Y over NVLink and waiting on the device for "
                                 "all ranks' shards of the previous op's Y",
                       "gather": "p2p peer stores (msq_matmul_gather), no multicast", "timing": spread,
                       "parity_rel_l2": parity, "parity_of": "rank 0's assembled full Y of every op vs the checker"},
            "roofline": {"bound": "hbm", "achieved": per_rank, "peak": peak, "unit": "GB/s", "frac": per_rank / peak,
                         "traffic": None, "peak_source": f"{peak_kind} HBM copy bandwidth",
                         "note": "per-rank shard bytes over the whole step time (peer stores and waits included)"},
            "cpu_baseline": None,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": sum(a.numel() * 4 for a in a_host),
                    "d2h_bytes_per_step": sum(y.numel() * 4 for y in y_host), "steps": e2e_steps,
                    "entry": "ShardedMatMulNBits (pinned host A in, gathered Y out)"},
            "gpu_launches": launches_per_step * args.steps * args.windows,
            "clocks": clk.summary(),
        }
    for g in graphs:
        del g
    graphs.clear()
    for si, op in enumerate(ops):
        op.weights = reps[si][0]
        for w in reps[si][1:]:
            w.free()
        op.free()
    return out


# ---------------------------------------------------------------- N-split workload
NSPLIT_LAYERS = [(8192, 28672), (28672, 8192)]  # (K, N): 70B MLP up-proj, then down-proj
NSPLIT_WORKLOAD = ("70B-shaped MLP (BASELINE configs[3]) column-split over the ranks with a gather of Y: "
                   "up-proj K=8192 N=28672 then down-proj K=28672 N=8192 fed with the gathered up-proj output; "
                   "bits=4, block_size=128, packed zero points, fp16 scales, fp16 A")


def run_nsplit(args, rank: int, world: int, local_rank: int):
    """Each rank packs its row shard of both layers; one step = up-proj shard, all-gather, down-proj
    shard, all-gather, captured in one CUDA graph; value = the layers' algorithmic bytes per step
    over the max-over-ranks step time (total work fixed: strong scaling)."""
    import torch
    import torch.distributed as dist

    from modelsharp_b200 import _native as N
    from modelsharp_b200 import synth
    from modelsharp_b200.nsplit import ShardedMatMulNBits

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    M = args.m
    cases = [synth.make_case(100 + i, M, n, k, 4, BS, "packed", a_dtype="f16", scale_dtype="f16",
                             scale_lo=SCALE_LO, scale_hi=SCALE_HI) for i, (k, n) in enumerate(NSPLIT_LAYERS)]
    nbytes = sum(synth.algorithmic_bytes(n, k, 4, BS, "packed", scale_bytes=2) for k, n in NSPLIT_LAYERS)
    shard_bytes = nbytes / world
    # enough replicas of this rank's shards that the rotation exceeds L2 (>= 320 MB per rank)
    reps_n = max(2, -(-int(320e6) // int(shard_bytes)))
    reps_n += reps_n % 2  # even: each layer's two exchange buffers alternate across the graphs' wrap-around
    full = [[torch.from_numpy(np.ascontiguousarray(x)).to(dev) if x is not None else None
             for x in (c["b"], c["scales"], c["zp"])] for c in cases]
    gather = args.gather if M <= 4 else "nccl"
    reps = [[ShardedMatMulNBits(b, s, z, c["N"], c["K"], 4, BS, device=dev, gather=gather)
             for (b, s, z), c in zip(full, cases)] for _ in range(reps_n)]
    del full
    a0 = torch.from_numpy(cases[0]["a"]).to(dev)
    stream = torch.cuda.Stream(dev)

    def step(r: int, a: torch.Tensor) -> torch.Tensor:
        y_up = reps[r][0](a)
        return reps[r][1](y_up, wait=reps[r][0].out_wait)

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            y = step(i % reps_n, a0)
    stream.synchronize()
    graphs, outs = [], []
    for r in range(reps_n):
        g = torch.cuda.CUDAGraph()
        c0 = N.launch_count()
        with torch.cuda.graph(g, stream=stream):
            outs.append(step(r, a0))
        per_step_launches = N.launch_count() - c0  # library kernels in one step (GEMV / GEMM, split-K reduce)
        graphs.append(g)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            graphs[i % reps_n].replay()
    with torch.cuda.stream(stream):
        graphs[0].replay()
        reps[0][1].wait_gathered()  # every rank's shard of the output has landed here
    stream.synchronize()
    y_chk = outs[0].float().cpu().numpy()

    with ClockSampler(local_rank) as clk:
        wins = timed_windows(args, world, dev, stream, lambda i: graphs[i % reps_n].replay())
    ms, spread = window_stats(wins)
    value = nbytes * args.steps / (ms * 1e-3) / 1e9

    # e2e through the sharded op with host buffers: A in, the down-proj Y out, every step
    a_host = torch.from_numpy(cases[0]["a"]).pin_memory()
    y_host = torch.empty(M, NSPLIT_LAYERS[1][1]).pin_memory()
    e2e_steps = max(1, min(args.steps, 500))
    def e2e_step(i: int):
        y = step(i % reps_n, a_host.to(dev, non_blocking=True))
        reps[i % reps_n][1].wait_gathered()
        y_host.copy_(y, non_blocking=True)

    for i in range(max(args.warmup, 3)):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    dist.barrier() if world > 1 else None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record()
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = nbytes * e2e_steps / (e2e_ms * 1e-3) / 1e9

    peak, peak_kind = peaks()
    per_rank_achieved = shard_bytes / (ms / args.steps * 1e-3) / 1e9
    flops = 2.0 * M * sum(n * k for k, n in NSPLIT_LAYERS)  # whole step, all ranks
    tc_peak = tensor_peak()
    # the bound by arithmetic intensity: FLOPs per weight byte against the ridge of the measured
    # peaks (about 210 FLOP/B; M = 32 does about 120, so it is HBM-bound even on the tensor cores)
    if flops / nbytes > tc_peak[0] * 1e12 / (peak * 1e9):
        tflops_rank = flops / world / (ms / args.steps * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": tflops_rank, "peak": tc_peak[0], "unit": "TFLOP/s",
                "frac": tflops_rank / tc_peak[0], "traffic": None, "peak_source": tc_peak[1],
                "note": "per-rank FLOPs over the whole step time (all-gathers included)"}
    else:
        roof = {"bound": "hbm", "achieved": per_rank_achieved, "peak": peak, "unit": "GB/s",
                "frac": per_rank_achieved / peak, "traffic": None, "peak_source": f"{peak_kind} HBM copy bandwidth",
                "note": "per-rank shard bytes over the whole step time (all-gathers included)",
                "tflops_per_rank": flops / world / (ms / args.steps * 1e-3) / 1e12}
    if rank == 0:
        from oracle import oracle
        # parity of the assembled output against the checker chain (up-proj output fed to the down-proj)
        y_up_ref = oracle.managed(cases[0])
        c1 = dict(cases[1], a=y_up_ref, M=M)
        parity = oracle.rel_l2(y_chk, oracle.managed(c1))
        cpu = None
        if world == 1:
            t0 = time.perf_counter()
            reps_cpu = 0
            while time.perf_counter() - t0 < max(args.cpu_seconds, 0.1) or reps_cpu < 1:
                ref_fn = oracle.reference_native if oracle.reference_available() else oracle.managed
                ref_fn(dict(cases[0], a=cases[0]["a"].astype(np.float32), scales=cases[0]["scales"].astype(np.float32)))
                ref_fn(dict(c1, scales=c1["scales"].astype(np.float32)))
                reps_cpu += 1
            dt = (time.perf_counter() - t0) / reps_cpu
            cpu = {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": os.cpu_count(),
                   "kind": "reference" if oracle.reference_available() else "port",
                   "sample": f"{reps_cpu} steps (both layers, fp16 inputs widened to fp32), mean, all host threads"}
        out = {
            "metric": "MatMulNBits INT4 N-split HBM GB/s", "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 in, f32 accumulate", "data": "synthetic",
            "config": {"workload": NSPLIT_WORKLOAD, "M": M, "bytes_per_step": nbytes, "parallelism": f"nsplit{world}",
                       "l2": f"{reps_n} replicas of each rank's shards rotate ({reps_n * shard_bytes / 1e6:.0f} MB per rank)",
                       "launch": ("one CUDA graph replay per step: 2 GEMV launches that store into every rank's "
                                  "Y over NVLink and signal completion" if gather == "p2p" else
                                  f"one CUDA graph replay per step: {per_step_launches} library launches "
                                  f"({'tensor-core GEMM' if M >= 17 else 'decode GEMV'})"
                                  + (" + 2 NCCL all-gathers" if world > 1 else " (one GPU: nothing to gather)")),
                       "gather": gather, "flops_per_step": flops, "timing": spread,
                       "tflops": flops / (ms / args.steps * 1e-3) / 1e12,
                       "parity_rel_l2": parity},
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": a_host.numel() * 2,
                    "d2h_bytes_per_step": y_host.numel() * 4, "steps": e2e_steps, "entry": "ShardedMatMulNBits"},
            "gpu_launches": per_step_launches * args.steps,
            "clocks": clk.summary(),
        }
    else:
        out = None
    for g in graphs:
        del g
    graphs.clear()
    for rr in reps:
        for sh in rr:
            sh.free()
    return out


# ---------------------------------------------------------------- prefill GEMM workload
PREFILL_MS = (512, 2048, 8192)
PREFILL_K, PREFILL_N, PREFILL_BS = 4096, 14336, 32
PREFILL_WORKLOAD = ("prefill tensor-core GEMM (BASELINE configs[2]): M in {512, 2048, 8192}, K=4096, N=14336, "
                    "bits=4, block_size=32, packed zero points, fp16 A ~N(0,1), fp16 scales U[0.001, 0.01]")


def run_prefill(args, rank: int, world: int, local_rank: int):
    """One step = the three GEMMs (one CUDA graph); value = 2*M*N*K summed over the three / step
    time. Weight replicas rotate so weights + activations exceed L2 every step."""
    import torch
    import torch.distributed as dist

    from modelsharp_b200 import QuantizedWeights, synth
    from modelsharp_b200 import _native as N

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib = N.lib()
    cases = [synth.make_case(200 + i, m, PREFILL_N, PREFILL_K, 4, PREFILL_BS, "packed", a_dtype="f16",
                             scale_dtype="f16", scale_lo=SCALE_LO, scale_hi=SCALE_HI) for i, m in enumerate(PREFILL_MS)]
    flops = sum(2.0 * m * PREFILL_N * PREFILL_K for m in PREFILL_MS)
    reps_n = 4
    wb = cases[0]
    reps = [QuantizedWeights(wb["b"], wb["scales"], wb["zp"], PREFILL_N, PREFILL_K, 4, PREFILL_BS, device=dev)
            for _ in range(reps_n)]
    a_dev = [torch.from_numpy(c["a"]).to(dev) for c in cases]
    y_dev = [torch.empty(c["M"], PREFILL_N, device=dev) for c in cases]
    stream = torch.cuda.Stream(dev)
    sptr = stream.cuda_stream

    gpath = N.PATH_GEMM_SPLIT if getattr(args, "split", False) else N.PATH_GEMM

    def launch_step(r: int):
        for a, y in zip(a_dev, y_dev):
            rc = lib.msq_matmul_ex(None, sptr, reps[r].handle, a.data_ptr(), N.DT_F16, a.shape[0], y.data_ptr(),
                                   PREFILL_N, gpath)
            if rc:
                N.check(rc)

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            launch_step(i % reps_n)
    stream.synchronize()
    path = N.last_path()
    before = N.launch_count()
    graphs = []
    for r in range(reps_n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            launch_step(r)
        graphs.append(g)
    launches_per_step = (N.launch_count() - before) // reps_n
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            graphs[i % reps_n].replay()
    stream.synchronize()
    # per-M duration: one graph per M of reps_n launches
    per_m = []
    for mi, (a, y) in enumerate(zip(a_dev, y_dev)):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for r in range(reps_n):
                lib.msq_matmul_ex(None, sptr, reps[r].handle, a.data_ptr(), N.DT_F16, a.shape[0], y.data_ptr(),
                                  PREFILL_N, gpath)
        with torch.cuda.stream(stream):
            g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            nrep = 5
            for _ in range(nrep):
                g.replay()
            e1.record(stream)
        stream.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (nrep * reps_n)
        per_m.append({"M": PREFILL_MS[mi], "us": us, "TFLOP/s": 2.0 * PREFILL_MS[mi] * PREFILL_N * PREFILL_K / us / 1e6})
        del g

    # timed like the sweep: windows of exactly --steps graph replays, the median window
    with ClockSampler(local_rank) as clk:
        wins = timed_windows(argparse.Namespace(windows=getattr(args, "windows", 30), steps=args.steps), world, dev,
                             stream, lambda i: graphs[i % reps_n].replay())
    ms, spread = window_stats(wins)
    value = world * flops * args.steps / (ms * 1e-3) / 1e12

    # e2e: host A in (fp16), Y out (fp32) through msq_matmul_host, every step
    a_host = [torch.from_numpy(c["a"]).pin_memory() for c in cases]
    y_host = [torch.empty(c["M"], PREFILL_N).pin_memory() for c in cases]
    e2e_steps = max(1, min(args.steps, 5))

    def e2e_step(r: int):
        for a, y in zip(a_host, y_host):
            rc = lib.msq_matmul_host(None, sptr, reps[r].handle, a.data_ptr(), N.DT_F16, a.shape[0], y.data_ptr())
            if rc:
                N.check(rc)

    e2e_step(0)
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(e2e_steps):
        e2e_step(i % reps_n)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * flops * e2e_steps / (e2e_ms * 1e-3) / 1e12

    if rank == 0:
        from oracle import oracle
        par = []
        for c, y in zip(cases, y_dev):
            m = c["M"]
            rows = [slice(0, 16), slice(m // 2, m // 2 + 16), slice(m - 16, m)]
            yy = y.cpu().numpy()
            cw = dict(wb, a=c["a"], M=m)  # every GEMM runs on the first case's weights
            par.append(oracle.rel_l2(np.concatenate([yy[r] for r in rows]),
                                     np.concatenate([oracle.managed(cw, rows=r) for r in rows])))
        # The step is timed as 30 windows back to back, about a second of GEMMs, so the 1 kW power
        # cap engages (sw_power_cap in the clock record): the sustained cuBLAS rate, measured
        # back to back under the same cap, is the matching denominator; the burst figure (one
        # GEMM alone at full clock) is reported beside it.
        peak, peak_src = tensor_peak()
        burst, burst_src = burst_tensor_peak()
        cpu = None
        if world == 1:
            c = cases[0]
            sample = dict(c, a=c["a"][:64].astype(np.float32), M=64)
            fn = oracle.reference_native if oracle.reference_available() else oracle.managed
            fn(sample)
            t_0 = time.perf_counter()
            n = 0
            while time.perf_counter() - t_0 < max(args.cpu_seconds, 0.1) or n < 1:
                fn(sample)
                n += 1
            dt = (time.perf_counter() - t_0) / n
            cpu = {"value": 2.0 * 64 * PREFILL_N * PREFILL_K / dt / 1e12, "unit": "TFLOP/s", "cores": os.cpu_count(),
                   "kind": "reference" if oracle.reference_available() else "port",
                   "sample": f"{n} calls of M=64 rows of the M=512 case (fp16 widened to fp32), mean, all host threads"}
        out = {
            "metric": "MatMulNBits INT4 prefill TFLOPS" + (" (split operands)" if gpath == N.PATH_GEMM_SPLIT else ""),
            "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 operands, f32 accumulate", "data": "synthetic",
            "config": {"workload": PREFILL_WORKLOAD, "flops_per_step": flops, "parallelism": f"replicas{world}",
                       "l2": f"{reps_n} weight replicas rotate; A up to {8192 * PREFILL_K * 2 / 1e6:.0f} MB",
                       "launch": "one CUDA graph replay per step", "kernel_path": path,
                       "parity_rel_l2_sampled_rows": max(par), "timing": spread},
            "roofline": {"bound": "tensor", "achieved": value / world, "peak": peak, "unit": "TFLOP/s",
                         "frac": value / world / peak, "traffic": None,
                         "peak_source": peak_src, "peak_burst": burst, "frac_burst": value / world / burst,
                         "per_M": per_m},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": sum(a.numel() * 2 for a in a_host),
                    "d2h_bytes_per_step": sum(y.numel() * 4 for y in y_host), "steps": e2e_steps,
                    "entry": "msq_matmul_host"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
        }
    else:
        out = None
    graphs.clear()
    for w in reps:
        w.free()
    return out


# ---------------------------------------------------------------- end-to-end decoder
DECODE_WORKLOAD = ("synthetic 7B-shaped INT4 decoder (BASELINE configs[4]): 32 layers, hidden 4096, 32 query / "
                   "8 key-value heads of 128, SwiGLU 14336, vocabulary 32000, every projection MatMulNBits bits=4 "
                   "block_size=32 with zero points; greedy decode of 128 tokens after a 512-token prompt of uniform "
                   "random ids; q/k/v and gate/up packed into one MatMulNBits each; fp32 glue: the library's "
                   "fused decode kernels (add+RMSNorm, rotary+KV append, split-K GQA, SwiGLU, argmax); the prompt's "
                   "projections on the split-operand tcgen05 GEMM (MSQ_PATH_GEMM_SPLIT), torch glue for the prompt pass")


def decode_checks(host_w, cfg, prompt_h, tokens, args):
    """Greedy parity of the timed generation's 128 tokens against the CPU checker (one
    teacher-forced pass over the prompt and the generated tokens, with the checker's top-2 logit
    margin per step), and the checker's own decode rate as the CPU baseline."""
    from oracle import decoder as od
    t0 = time.perf_counter()
    r = od.greedy_check(host_w, cfg, prompt_h.numpy(), np.asarray(tokens))
    fm = r["first_mismatch"]
    match = {"tokens_equal": r["matches"], "of": r["steps"], "first_mismatch": fm,
             "top2_margin_at_first_mismatch": r["margins"][fm] if fm is not None else None,
             "min_top2_margin": r["min_margin"], "min_margin_step": r["min_margin_step"],
             "check": f"teacher-forced CPU pass of oracle/decoder.py over the {len(prompt_h)}-token prompt and the "
                      f"generated tokens ({time.perf_counter() - t0:.0f} s)"}
    short = prompt_h[:16]
    cache = {"k": np.zeros((cfg.layers, cfg.kv_heads, cfg.max_seq, cfg.head_dim), np.float32),
             "v": np.zeros((cfg.layers, cfg.kv_heads, cfg.max_seq, cfg.head_dim), np.float32),
             "rope": od.rope_tables(cfg)}
    od.forward(host_w, cfg, short.numpy()[:8], 0, cache)
    t_0, n = time.perf_counter(), 0
    while n < 2 or time.perf_counter() - t_0 < max(args.cpu_seconds, 0.1):
        od.forward(host_w, cfg, short.numpy()[8 + n:9 + n], 8 + n, cache)
        n += 1
    dt = (time.perf_counter() - t_0) / n
    cpu = {"value": 1.0 / dt, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
           "sample": f"{n} decode steps of the CPU restatement (C MatMulNBits restatement on all host "
                     "threads, numpy glue) at context 8..16"}
    return cpu, match


def run_decode_engine(args, rank: int, world: int, local_rank: int):
    """configs[4] through the engine: the decoder as a graph (build_decoder_graph) run by
    CudaEngine's node loop on the CUDA registry: the prompt as one eager run, then one token per
    run, each a replay of one captured engine run. value = decode tokens/s over 127 steps per
    generation."""
    import torch
    import torch.distributed as dist

    from modelsharp_b200 import _native as N
    from modelsharp_b200.decoder import DecoderConfig, EngineDecoder, make_weights, weight_bytes_per_token

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = DecoderConfig(layers=args.layers)
    w = make_weights(cfg, 0, dev)
    eng = EngineDecoder(cfg, w, dev)
    host_w = None
    if rank == 0 and world == 1:
        from modelsharp_b200.decoder import weights_to_host
        host_w = weights_to_host(w)
    n_prompt, n_new = 512, 128
    prompt_h = torch.randint(0, cfg.vocab, (n_prompt,), generator=torch.Generator().manual_seed(1))
    prompt = prompt_h.to(dev)
    for _ in range(2):  # warm-up: GEMM tensor maps, library first calls, the prompt form's torch kernels
        eng.prefill(prompt)
    c0 = N.launch_count()
    eng.capture()
    per_run = (N.launch_count() - c0) // 2  # the warm-up run and the captured run
    stream = torch.cuda.current_stream(dev)
    reps = max(2, args.steps // n_new)
    pre_ms, dec_ms = 0.0, 0.0
    gen = torch.empty(reps, n_new, dtype=torch.long, device=dev)
    prompt_launches = 0
    if world > 1:
        dist.barrier()
    with ClockSampler(local_rank) as clk:
        for r in range(reps):
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record(stream)
            c1 = N.launch_count()
            tok = eng.prefill(prompt)["next_token"].clone()
            prompt_launches += N.launch_count() - c1  # the eager prompt run's library launches
            gen[r, 0] = tok[0, 0]
            e1.record(stream)
            for j in range(1, n_new):
                out = eng.step(tok, n_prompt + j - 1)
                tok = out["next_token"].clone()
                gen[r, j] = tok[0, 0]
            e2.record(stream)
            stream.synchronize()
            pre_ms += e0.elapsed_time(e1)
            dec_ms += e1.elapsed_time(e2)
    if world > 1:
        t = torch.tensor([pre_ms, dec_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pre_ms, dec_ms = (float(v) for v in t.tolist())
    steps = reps * (n_new - 1)
    ms_tok = dec_ms / steps
    # e2e: host prompt in, host tokens out, prompt runs included
    t0 = time.perf_counter()
    toks, _ = eng.generate(prompt_h.pin_memory().to(dev, non_blocking=True), n_new)
    toks_h = toks.cpu()
    e2e_value = world * n_new / (time.perf_counter() - t0)
    peak, peak_kind = peaks()
    wb = weight_bytes_per_token(cfg)
    achieved = wb / (ms_tok * 1e-3) / 1e9
    if rank == 0:
        cpu, match = None, None
        if host_w is not None:
            cpu, match = decode_checks(host_w, cfg, prompt_h, gen[0].cpu().numpy(), args)
        res = {
            "metric": "7B INT4 decode tok/s", "value": world * 1e3 / ms_tok, "unit": "tok/s", "n_gpus": world,
            "steps": steps, "warmup": 2, "ms_per_step": ms_tok, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 activations, int4 weights", "data": "synthetic",
            "config": {"workload": ("engine path of: " + DECODE_WORKLOAD) if cfg.layers == 32 else
                       f"{cfg.layers}-layer cut of the engine path (a profiling case, not the 7B shape)",
                       "entry": "EngineDecoder: build_decoder_graph, the graph_fusion pass (norms, SwiGLU and "
                                "residual adds into MatMulNBitsFused nodes), CudaEngine on the llm_ops registry, one "
                                "captured engine run replayed per token",
                       "prompt_tokens": n_prompt, "new_tokens": n_new, "generations": reps,
                       "prompt_ms": pre_ms / reps, "weight_bytes_per_token": wb, "parallelism": f"replicas{world}",
                       "l2": "4.5 GB of weights per token, far above L2", "greedy_parity": match,
                       "tokens_repeatable": bool((gen.cpu() == toks_h.reshape(1, -1)).all())},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "peak_source": f"{peak_kind} HBM copy bandwidth",
                         "note": "MatMulNBits weight bytes per token over the whole engine run"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": n_prompt * 8,
                    "d2h_bytes_per_step": n_new * 8, "entry": "EngineDecoder.generate (prompt run included)"},
            "gpu_launches": prompt_launches + per_run * reps * (n_new - 1),
            "clocks": clk.summary(),
        }
    else:
        res = None
    eng.release()
    return res


def run_decode(args, rank: int, world: int, local_rank: int):
    """Per rank: prompt (512 tokens, tensor-core GEMM) then 127 decode steps, each one CUDA-graph
    replay (the first token comes from the prompt pass). value = decode tokens/s; the prompt
    pass is timed separately. Repeated args.steps // 128 times (at least 2)."""
    import torch
    import torch.distributed as dist

    from modelsharp_b200 import _native as N
    from modelsharp_b200.decoder import CudaDecoder, DecoderConfig, make_weights, weight_bytes_per_token

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = DecoderConfig(layers=args.layers)
    w = make_weights(cfg, 0, dev)
    dec = CudaDecoder(cfg, w, dev)
    host_w = None
    if rank == 0 and world == 1:
        from modelsharp_b200.decoder import weights_to_host
        host_w = weights_to_host(w)
    del w
    torch.cuda.synchronize(dev)
    n_prompt, n_new = 512, 128
    prompt_h = torch.randint(0, cfg.vocab, (n_prompt,), generator=torch.Generator().manual_seed(1))
    prompt = prompt_h.to(dev)
    stream = torch.cuda.Stream(dev)
    tok = torch.zeros(1, dtype=torch.long, device=dev)
    pos = torch.zeros(1, dtype=torch.long, device=dev)
    with torch.cuda.stream(stream):
        for _ in range(2):
            dec.generate(prompt, 4)  # warm-up: settles the weights, sets kernel attributes
        tok.copy_(torch.argmax(dec.prefill(prompt)).view(1))
        pos.fill_(n_prompt)
        g = torch.cuda.CUDAGraph()
        c0 = N.launch_count()
        with torch.cuda.graph(g, stream=stream):
            dec.decode_step(tok, pos)
        per_replay = N.launch_count() - c0  # library kernels in one decode step
    stream.synchronize()
    reps = max(2, args.steps // n_new)
    out = torch.empty(reps, n_new, dtype=torch.long, device=dev)
    pre_ms, dec_ms = 0.0, 0.0
    launches0 = N.launch_count()
    if world > 1:
        dist.barrier()
    with ClockSampler(local_rank) as clk:
        for r in range(reps):
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            with torch.cuda.stream(stream):
                e0.record(stream)
                tok.copy_(torch.argmax(dec.prefill(prompt)).view(1))
                pos.fill_(n_prompt)
                out[r, 0] = tok[0]
                e1.record(stream)
                if r == 0:  # the first generation's decode steps are what `ncu --profile-from-start off` sees
                    torch.cuda.profiler.start()
                for i in range(1, n_new):
                    g.replay()
                    out[r, i] = tok[0]
                e2.record(stream)
            stream.synchronize()
            if r == 0:
                torch.cuda.profiler.stop()
            pre_ms += e0.elapsed_time(e1)
            dec_ms += e1.elapsed_time(e2)
    launches = N.launch_count() - launches0 + reps * (n_new - 1) * per_replay  # prompt passes + replays
    if world > 1:
        t = torch.tensor([pre_ms, dec_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pre_ms, dec_ms = (float(v) for v in t.tolist())
    steps = reps * (n_new - 1)
    ms_tok = dec_ms / steps
    value = world * 1e3 / ms_tok
    tokens = out.cpu().numpy()

    # e2e: host prompt in, host tokens out, prompt pass included, per generation
    e_reps = 2
    out_h = torch.empty(n_new, dtype=torch.long).pin_memory()
    prompt_pin = prompt_h.pin_memory()
    t0 = time.perf_counter()
    for _ in range(e_reps):
        with torch.cuda.stream(stream):
            p = prompt_pin.to(dev, non_blocking=True)
            tok.copy_(torch.argmax(dec.prefill(p)).view(1))
            pos.fill_(n_prompt)
            gen = torch.empty(n_new, dtype=torch.long, device=dev)
            gen[0] = tok[0]
            for i in range(1, n_new):
                g.replay()
                gen[i] = tok[0]
            out_h.copy_(gen, non_blocking=True)
        stream.synchronize()
    e2e_s = (time.perf_counter() - t0) / e_reps
    e2e_value = world * n_new / e2e_s
    consistent = bool((tokens == tokens[0]).all() and (out_h.numpy() == tokens[0]).all())

    peak, peak_kind = peaks()
    wb = weight_bytes_per_token(cfg)
    achieved = wb / (ms_tok * 1e-3) / 1e9
    if rank == 0:
        cpu, match = None, None
        if host_w is not None:
            cpu, match = decode_checks(host_w, cfg, prompt_h, tokens[0], args)
        res = {
            "metric": "7B INT4 decode tok/s", "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": 2, "ms_per_step": ms_tok, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 activations, int4 weights", "data": "synthetic",
            "config": {"workload": DECODE_WORKLOAD if cfg.layers == 32 else
                       f"{cfg.layers}-layer cut of: {DECODE_WORKLOAD} (a profiling case, not the 7B shape)",
                       "prompt_tokens": n_prompt, "new_tokens": n_new,
                       "generations": reps, "prompt_ms": pre_ms / reps, "prompt_tok_s": n_prompt / (pre_ms / reps) * 1e3,
                       "weight_bytes_per_token": wb, "parallelism": f"replicas{world}",
                       "l2": "4.5 GB of weights per token, far above L2",
                       "launch": "one CUDA graph replay per decode token", "greedy_parity": match,
                       "tokens_repeatable": consistent},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "peak_source": f"{peak_kind} HBM copy bandwidth",
                         "note": "MatMulNBits weight bytes per token over the whole decode step (glue included)"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": n_prompt * 8,
                    "d2h_bytes_per_step": n_new * 8, "entry": "CudaDecoder (prompt pass included)"},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
    else:
        res = None
    del g
    dec.free()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--workload", default="sweep7b", choices=["sweep7b", "nsplit70b", "prefill", "decode7b"])
    ap.add_argument("--rows", "--m", dest="m", type=int, default=1,
                    help="A rows for the nsplit70b workload (--rows under torchrun, whose parser takes --m as a "
                         "prefix of its own options)")
    ap.add_argument("--gather", default="p2p", choices=["p2p", "nccl"],
                    help="nsplit70b: fused peer-store gather (M <= 4) or NCCL all-gather")
    ap.add_argument("--engine", action="store_true",
                    help="decode7b: run the decoder graph through the engine (CudaEngine node loop) instead of "
                         "the fused decode step")
    ap.add_argument("--layers", type=int, default=32,
                    help="decode7b: decoder layers (32 = the 7B shape; fewer only for small profiling cases)")
    ap.add_argument("--windows", type=int, default=30,
                    help="timed windows of --steps steps each (sweep workloads); value from the median window")
    ap.add_argument("--split", action="store_true",
                    help="prefill: the split-operand GEMM (MSQ_PATH_GEMM_SPLIT) instead of the fp16 one")
    ap.add_argument("--no-sub", action="store_true",
                    help="N = 1 sweep only: skip the prefill, 7B decode and 70B M = 32 sub-records")
    ap.add_argument("--shapes", default="",
                    help="restrict the step to these KxN shapes (comma separated), for profiling one shape")
    args = ap.parse_args()
    if args.shapes:
        global WORKLOAD
        SWEEP[:] = [tuple(int(v) for v in sh.lower().split("x")) for sh in args.shapes.split(",")]
        WORKLOAD = ("subset of the 7B decode GEMV sweep at M=1: (K,N) = " +
                    ", ".join(f"({k},{n})" for k, n in SWEEP) + "; bits=4, block_size=128, packed zero points")
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "nsplit70b":
            out = run_nsplit(args, rank, world, local_rank)
        elif args.workload == "prefill":
            out = run_prefill(args, rank, world, local_rank)
        elif args.workload == "decode7b":
            out = (run_decode_engine if args.engine else run_decode)(args, rank, world, local_rank)
        elif world > 1:
            out = run_split_sweep(args, rank, world, local_rank)
        else:
            out = run_ours(args, rank, world, local_rank)
            if not args.no_sub:
                # the other two headline metrics (BASELINE metric: prefill TFLOPS, 7B decode tok/s),
                # each with its own timing, clocks, parity, roofline and CPU baseline
                log("sub-record: prefill (configs[2])")
                pre = run_prefill(args, rank, world, local_rank)
                log("sub-record: 7B decode (configs[4])")
                dec = run_decode(args, rank, world, local_rank)
                log("sub-record: 70B layers at M = 32 (configs[3], one GPU)")
                l70 = run_nsplit(argparse.Namespace(**{**vars(args), "m": 32, "gather": "nccl"}), rank, world,
                                 local_rank)
                if out is not None:
                    out["sub"] = {"prefill": pre, "decode7b": dec, "layers70b_m32": l70}
        if rank == 0 and out is not None:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
