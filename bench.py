#!/usr/bin/env python
"""Benchmark of the batched FP32 Cholesky hot path (custom_kernel) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (one rank per GPU, NCCL)

A *step* is one ``custom_kernel`` call over one (batch, n, n) input. Inputs are
the benchmark shapes' seeded synthetic families (linalg_kernels_b200.inputs), resident in HBM
before timing, taken round-robin from a pool of distinct inputs whose total size exceeds
twice the 126 MB L2 (no L2 reuse between steps). Timing: W warm-up steps, barrier +
synchronize, CUDA events around exactly K steps on the launching queue, barrier +
synchronize, maximum over ranks. Multi-GPU: every rank factors its own batch of the
configured size (independent matrices, no collective on the data path): weak scaling.

Printed (rank 0, one JSON line): value = matrices/s over all ranks; TFLOP/s at n^3/3 per
matrix; roofline of the dominant kernel (achieved / MEASURED_PEAKS.json peak; traffic from
the committed ncu capture); e2e = the same metric through the C ABI with pinned host
buffers and both copies inside the timed region; cpu_baseline = the reference's own CPU
path (torch.linalg.cholesky_ex on the host cores) on a bounded sample; clocks sampled by
nvidia-smi during the run; gpu_launches = our kernel launches in the timed region.
``--impl reference`` times that CPU path alone as the reference arm.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import re
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

DEFAULT_CONFIG = "b1024n64"
L2_BYTES = 126 * 1024 * 1024

# The reference's published single-B200 times per call for the benchmark grid: the seven
# configs as the reference's best snapshots (references/CURRENT_PERF.md, NEW_PERF3.md for
# b64n256, b640n512, b60n1024), the other eight from references/CURRENT_PERF.md.
REFERENCE_PUBLISHED_S = {
    "b4096n32": 15.7e-6, "b1024n64": 24.1e-6, "b64n256": 191e-6, "b640n512": 2.88e-3,
    "b60n1024": 2.20e-3, "b1n16384": 15.1e-3, "b1n32768": 42.9e-3,
    "b256n128": 70.9e-6, "b16n512": 537e-6, "b4n1024": 1199e-6, "b2n2048": 3.21e-3,
    "b8n2048": 4.88e-3, "b1n4096": 1527e-6, "b2n4096": 11.1e-3, "b1n8192": 6.37e-3,
}

# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu capture of the
# same workload (python bench.py --ncu-run --config <name>; the short summaries live in the
# profiles folder). None until captured.
NCU_TRAFFIC_BYTES: dict[str, float | None] = {
    "b1024n64": 12.74e6,   # small_potrf_kernel; its writes are still in L2 at kernel end
    "b4096n32": 16.80e6,   # small_potrf_kernel; likewise
}


def _peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# --------------------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------------------
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist
            # the first collectives set up NCCL's connections, partly in the background:
            # done here, before any timed region
            for _ in range(2):
                dist.barrier(device_ids=[self.local])
            torch.cuda.synchronize()

    def barrier(self):
        if self.pg:
            self.pg.barrier(device_ids=[self.local])

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# --------------------------------------------------------------------------------------
# clocks during the run
# --------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict | None:
        rows = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append({"sm": float(parts[1]), "max": float(parts[2]),
                             "power": float(parts[3]) if parts[3] not in ("[N/A]", "") else 0.0,
                             "hw_slowdown": parts[5], "hw_thermal": parts[6],
                             "sw_thermal": parts[7], "sw_power_cap": parts[8]})
            except ValueError:
                continue
        if not rows:
            return None
        peak_power = max(r["power"] for r in rows)
        loaded = [r for r in rows if r["power"] >= 0.5 * peak_power] or rows
        reasons = set()
        for r in rows:
            for key, name in (("hw_slowdown", "hw_slowdown"), ("hw_thermal", "hw_thermal_slowdown"),
                              ("sw_thermal", "sw_thermal_slowdown"),
                              ("sw_power_cap", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded),
                "sm_max_mhz": max(r["max"] for r in rows), "reasons": sorted(reasons),
                "samples": len(rows), "samples_under_load": len(loaded),
                "power_w_max": peak_power,
                "window": "nvidia-smi every 100 ms over warm-up + timed steps"}


# --------------------------------------------------------------------------------------
# helpers
# --------------------------------------------------------------------------------------
def _pool_count(cfg, max_inputs: int) -> int:
    in_bytes = cfg.batch * cfg.n * cfg.n * 4
    return 1 if in_bytes >= 2 * L2_BYTES else min(max_inputs, math.ceil(2 * L2_BYTES / in_bytes))


def _config(cfg, world: int) -> dict:
    """The workload description both arms print (identical for the same config and N)."""
    count = _pool_count(cfg, 32)
    in_bytes = cfg.batch * cfg.n * cfg.n * 4
    return {"workload": cfg.name, "batch": cfg.batch, "n": cfg.n,
            "global_batch": cfg.batch * world, "family": cfg.family, "param": cfg.param,
            "seed": cfg.seed,
            "parallelism": f"batch-sharded x{world} (independent matrices, no collective)",
            "l2": f"GPU arm: inputs rotate over {count} distinct (batch, n, n) tensors "
                  f"({count * in_bytes / 2**20:.0f} MiB > 2x L2)"}


def _pool(cfg, device, rank: int, max_inputs: int):
    from linalg_kernels_b200 import inputs

    in_bytes = cfg.batch * cfg.n * cfg.n * 4
    count = _pool_count(cfg, max_inputs)
    pool = []
    cond = None
    for i in range(count):
        c = inputs.Config(cfg.name, cfg.batch, cfg.n, cfg.family, cfg.param,
                          cfg.seed + 7919 * i + 104729 * rank)
        a, cnd = inputs.config_input(c, device=device)
        pool.append(a)
        if cond is None:
            cond = cnd
    return pool, in_bytes * count


def _time_steps(fn, pool, steps: int, warmup: int, dist: Dist):
    """W untimed steps, then exactly K timed steps between one pair of CUDA events (as the
    reference's evaluator does, references/popcorn-eval/eval.py:199-205); returns total ms."""
    for i in range(warmup):
        fn(pool[i % len(pool)])
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    q = torch.cuda.current_stream()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    npool = len(pool)
    start.record(q)
    for i in range(steps):
        fn(pool[i % npool])
    end.record(q)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    return start.elapsed_time(end), None


def _cpu_sample_size(cfg, a_host: torch.Tensor, budget_s: float) -> int:
    """Matrices per CPU step: the whole batch for n <= 1024 (every such config takes well under
    a second on the host cores), else as many as fit the budget (at least one), sized from a
    warm call."""
    from oracle import oracle

    torch.set_num_threads(os.cpu_count() or 1)
    sample_b = a_host.shape[0]
    if cfg.n <= 1024:
        return sample_b
    x = a_host[:1]
    oracle.reference_factor(x)  # warm: MKL's threads and buffers
    t0 = time.perf_counter()
    oracle.reference_factor(x)
    one = max(time.perf_counter() - t0, 1e-6)
    return sample_b if one * sample_b <= budget_s else max(1, int(budget_s / one))


def _cpu_reference_rate(cfg, a_host: torch.Tensor, budget_s: float) -> dict:
    """The reference's CPU path (submission.py:7 on CPU tensors: LAPACK via MKL) on a
    bounded sample of the workload; all host threads."""
    from oracle import oracle

    torch.set_num_threads(os.cpu_count() or 1)
    threads = torch.get_num_threads()
    per_mat = cfg.n ** 3 / 3.0
    sample_b = _cpu_sample_size(cfg, a_host, budget_s)
    x = a_host[:sample_b].contiguous()
    oracle.reference_factor(x)  # warm
    reps, times = 0, []
    t_end = time.perf_counter() + budget_s
    while reps < 3 or (time.perf_counter() < t_end and reps < 50):
        t0 = time.perf_counter()
        oracle.reference_factor(x)
        times.append(time.perf_counter() - t0)
        reps += 1
        if cfg.n >= 8192:
            break
    med = statistics.median(times)
    return {"value": sample_b / med, "unit": "matrices/s", "cores": threads, "kind": "reference",
            "sample": f"{sample_b} of {cfg.batch} matrices of n={cfg.n}, median of {reps} runs "
                      f"of torch.linalg.cholesky_ex on CPU (MKL LAPACK spotrf)",
            "tflops": sample_b * per_mat / med / 1e12,
            "cpu": _cpu_model()}


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# --------------------------------------------------------------------------------------
# arms
# --------------------------------------------------------------------------------------
def run_reference(args, dist: Dist):
    """Reference arm: the reference's own CPU implementation of the path on the host cores."""
    from linalg_kernels_b200 import inputs

    cfg = inputs.GRID[args.config]
    if dist.rank != 0:
        return
    if torch.cuda.is_available():
        a, _ = inputs.config_input(cfg, device="cuda")
        a_host = a.cpu()
        del a
    else:
        a_host, _ = inputs.config_input(cfg, device="cpu", batch=min(cfg.batch, 64))
    # each step: the whole batch for n <= 1024, else a bounded sample (about 1 s of CPU work)
    sample_b = _cpu_sample_size(cfg, a_host, budget_s=1.0)
    x = a_host[:sample_b].contiguous()
    from oracle import oracle

    threads = torch.get_num_threads()
    for _ in range(args.warmup):
        oracle.reference_factor(x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.reference_factor(x)
    dt = time.perf_counter() - t0
    value = sample_b * args.steps / dt
    sample = (f"{sample_b} of {cfg.batch} matrices of n={cfg.n} per step, "
              f"torch.linalg.cholesky_ex on CPU (MKL LAPACK spotrf)")
    line = {
        "impl": "reference", "metric": "matrices/s", "value": value, "unit": "matrices/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "tflops": value * cfg.n ** 3 / 3.0 / 1e12,
        "config": _config(cfg, args.gpus),
        "reference_step": sample,
        "cpu_baseline": {"value": value, "unit": "matrices/s", "cores": threads,
                         "kind": "reference", "sample": sample, "cpu": _cpu_model()},
        "e2e": {"value": value, "unit": "matrices/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, dist: Dist):
    from linalg_kernels_b200 import _lib, inputs
    from linalg_kernels_b200.cholesky import custom_kernel

    lib = _lib.load()
    dev = torch.device("cuda", dist.local if dist.world > 1 else 0)
    torch.cuda.set_device(dev)
    peaks, peak_kind = _peaks()
    cfg = inputs.GRID[args.config]
    n, b = cfg.n, cfg.batch
    pool, pool_bytes = _pool(cfg, dev, dist.rank, max_inputs=32)
    launches_per_call = int(lib.chol_launch_count(b, n))

    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(dev.index)).split(",")[dev.index]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else dev.index
    with ClockSampler(gpu_index) as clocks:
        total_ms, per = _time_steps(custom_kernel, pool, args.steps, args.warmup, dist)
    total_ms = dist.max(total_ms)
    ms_step = total_ms / args.steps
    value = dist.world * b * args.steps / (total_ms / 1e3)
    tflops = value * n ** 3 / 3.0 / 1e12

    # dominant kernel roofline
    roof = _roofline(args, cfg, per, peaks, peak_kind, lib, pool, dev, dist)

    # end to end through the C ABI: pinned host in -> device -> factor -> pinned host out
    e2e = _e2e(args, cfg, pool, lib, dev, dist)
    a_host = pool[0].cpu() if dist.world == 1 and not args.no_cpu_baseline else None
    del pool
    torch.cuda.empty_cache()

    cpu = None
    if dist.world == 1 and not args.no_cpu_baseline:
        cpu = _cpu_reference_rate(cfg, a_host, budget_s=args.cpu_budget)

    validator = None
    if dist.world == 1 and args.validate:
        validator = _validator_timing(dev, peaks, peak_kind, lib)

    # N > 1: the multi-GPU schedules of the larger configs, with a parity gate
    multi = _multi_gpu(args, dist, dev, peaks) if dist.world > 1 and args.multi else None

    shapes = None
    if dist.world == 1 and args.shapes:
        shapes = _other_shapes(args, cfg.name, dev, peaks, peak_kind, lib)

    line = {
        "metric": "matrices/s", "value": value, "unit": "matrices/s", "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (value / (b / REFERENCE_PUBLISHED_S[cfg.name])
                        if dist.world == 1 and cfg.name in REFERENCE_PUBLISHED_S else None),
        "dtype": "f32", "data": "synthetic",
        "tflops": tflops,
        "config": _config(cfg, dist.world),
        "roofline": roof,
        "e2e": e2e,
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "gpu_launches": launches_per_call * args.steps,
        "launches_per_step": launches_per_call,
    }
    if validator is not None:
        line["validator"] = validator
    if multi is not None:
        line["parity"] = multi.pop("parity")
        line["multi_gpu"] = multi
    if shapes is not None:
        line["grid"] = _grid_summary(cfg.name, ms_step, shapes)
        line["shapes"] = shapes
    if dist.rank == 0:
        print(json.dumps(line, separators=(",", ":")), flush=True)


def _kernel_ms_graph(lib, pool, dev, b, n, reps=20):
    """Average duration of one C-ABI call's kernels: `reps` calls captured into a CUDA graph
    (no host work between them), replayed after warm-up, timed with CUDA events on the
    replaying queue. Inputs rotate over the pool (> L2), outputs are preallocated."""
    from linalg_kernels_b200 import _lib

    need = int(lib.chol_workspace_bytes(b, n))
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    outs = [torch.empty_like(pool[0]) for _ in range(2)]
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))

    def calls():
        q = _lib.current_queue(dev)
        for i in range(reps):
            st = lib.chol_potrf_batched_ws_f32(pool[i % len(pool)].data_ptr(),
                                               outs[i % 2].data_ptr(), b, n, None,
                                               ws.data_ptr(), need, q)
            _lib.check(st, "chol_potrf_batched_ws_f32")

    with torch.cuda.stream(s):
        calls()  # warm: prepare, attributes, caches
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        calls()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream(dev)
    e0.record(cur)
    g.replay()
    e1.record(cur)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del g
    return ms


def _roofline(args, cfg, per_step_ms, peaks, peak_kind, lib, pool, dev, dist):
    n, b = cfg.n, cfg.batch
    if n <= 256 and int(lib.chol_launch_count(b, n)) == 1:
        # single launch per call: launches per second of back-to-back graph replay. Launches
        # of consecutive calls overlap (CHOL_OPT_OVERLAP_CALLS), so this is the steady-state
        # interval per launch; the isolated launch (overlap off) is reported beside it.
        from linalg_kernels_b200 import _lib

        t = dist.max(_kernel_ms_graph(lib, pool, dev, b, n)) / 1e3
        lib.chol_set_option(_lib.CHOL_OPT_OVERLAP_CALLS, 0)
        try:
            t_iso = dist.max(_kernel_ms_graph(lib, pool, dev, b, n)) / 1e3
        finally:
            lib.chol_set_option(_lib.CHOL_OPT_OVERLAP_CALLS, 1)
        bytes_ = 8.0 * n * n * b
        achieved = bytes_ / t / 1e9
        peak = peaks["hbm_gbs"]
        kernel = "small_potrf_kernel" if n <= 64 else "mid_potrf_kernel"
        return {"bound": "hbm", "kernel": kernel, "achieved": achieved,
                "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_kind": f"{peak_kind} hbm_gbs (burst copy)",
                "traffic": NCU_TRAFFIC_BYTES.get(cfg.name),
                "algorithmic_bytes_per_launch": bytes_, "launch_ms": t * 1e3,
                "isolated_launch_ms": t_iso * 1e3,
                "isolated_frac": bytes_ / t_iso / 1e9 / peak,
                "timing": "CUDA graph of 20 back-to-back calls, events around the replay; "
                          "launch_ms = replay time / 20 with consecutive launches overlapping, "
                          "isolated_launch_ms = the same with the overlap off"}
    # blocked path: time the largest trailing update launch alone (its own CUDA events)
    return _gemm_roofline(cfg, peaks, peak_kind, lib, pool, dev, dist)


def _gemm_roofline(cfg, peaks, peak_kind, lib, pool, dev, dist):
    from linalg_kernels_b200 import _lib

    n, b = cfg.n, cfg.batch
    kdim = 64 if n <= 1024 else 512
    m = n - kdim
    a = pool[0]
    c = torch.empty_like(a)
    q = ctypes.c_void_p(_lib.current_queue(dev))

    def launch():
        st = lib.chol_gemm_nt_f32(
            ctypes.c_void_p(c.data_ptr() + (kdim * n + kdim) * 4), b, n * n, n, m, m, kdim,
            ctypes.c_void_p(a.data_ptr() + kdim * n * 4), n * n, n,
            ctypes.c_void_p(a.data_ptr() + kdim * n * 4), n * n, n,
            -1.0, 1.0, 0, 1, q)
        _lib.check(st, "chol_gemm_nt_f32")

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    reps = 10
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    t = dist.max(e0.elapsed_time(e1) / reps) / 1e3
    flops = 2.0 * b * (m * (m + 1) / 2) * kdim  # lower triangle incl. diagonal
    achieved = flops / t / 1e12
    peak = peaks["bf16_tflops"] / 2.0  # TF32 dense rate is half the bf16 rate on tcgen05
    return {"bound": "tensor", "kernel": "trailing update C -= P P^T (lower tiles)",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_kind": f"{peak_kind} bf16_tflops / 2 (TF32 rate)",
            "traffic": NCU_TRAFFIC_BYTES.get(cfg.name + "/update"),
            "shape": {"m": m, "k": kdim, "batch": b}, "launch_ms": t * 1e3}


def _e2e(args, cfg, pool, lib, dev, dist):
    """End to end through the C ABI: every step copies its input from pinned host memory,
    factors it (chol_potrf_batched_f32) and copies the factor back to pinned host memory.
    Two queues and two buffer slots: step i's upload and factorisation run on one queue,
    its download on the other, so step i's download (device -> host copy engine) runs beside
    step i+1's upload (host -> device); a slot's next factorisation waits for its previous
    download. The events bracket everything (the download queue is joined before the end)."""
    from linalg_kernels_b200 import _lib

    n, b = cfg.n, cfg.batch
    nbytes = b * n * n * 4
    hosts = [p.cpu().pin_memory() for p in pool[: min(len(pool), 2)]]
    out_h = [torch.empty(b, n, n).pin_memory() for _ in range(2)]
    a_d = [torch.empty(b, n, n, device=dev) for _ in range(2)]
    l_d = [torch.empty(b, n, n, device=dev) for _ in range(2)]
    s_up = torch.cuda.Stream(device=dev)
    s_down = torch.cuda.Stream(device=dev)
    factored = [torch.cuda.Event() for _ in range(2)]
    downloaded = [torch.cuda.Event() for _ in range(2)]
    for ev in downloaded:
        ev.record(s_down)

    def step(i):
        k = i % 2
        with torch.cuda.stream(s_up):
            a_d[k].copy_(hosts[i % len(hosts)], non_blocking=True)
            s_up.wait_event(downloaded[k])
            st = lib.chol_potrf_batched_f32(ctypes.c_void_p(a_d[k].data_ptr()),
                                            ctypes.c_void_p(l_d[k].data_ptr()), b, n, None,
                                            ctypes.c_void_p(s_up.cuda_stream))
            _lib.check(st, "chol_potrf_batched_f32")
            factored[k].record(s_up)
        with torch.cuda.stream(s_down):
            s_down.wait_event(factored[k])
            out_h[k].copy_(l_d[k], non_blocking=True)
            downloaded[k].record(s_down)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_up)
    s_down.wait_event(e0)
    for i in range(args.steps):
        step(i)
    s_up.wait_stream(s_down)
    e1.record(s_up)
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(e0.elapsed_time(e1))
    return {"value": dist.world * b * args.steps / (ms / 1e3), "unit": "matrices/s",
            "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
            "ms_per_step": ms / args.steps,
            "path": "chol_potrf_batched_f32 (C ABI) with pinned host input/output; upload and "
                    "factorisation on one queue, download on another, two buffer slots"}


def _cyclic_shard(cfg, lay, dev) -> torch.Tensor:
    """This rank's columns of A = X X^T / n + shift I (the config's generator, X seeded
    N(0,1)), built block by block on the GPU with TF32 off."""
    n = cfg.n
    g = torch.Generator(device=dev).manual_seed(cfg.seed)
    x = torch.randn(n, n, generator=g, device=dev)
    shard = torch.zeros(n, lay.n_local, device=dev)
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for t in lay.owned():
            c0, w, lc = t * lay.bs, lay.width(t), lay.local_col(t)
            blk = (x[c0:] @ x[c0:c0 + w].T) / n
            blk[:w].diagonal().add_(cfg.param)
            shard[c0:, lc:lc + w] = torch.tril(blk)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    del x
    torch.cuda.empty_cache()
    return shard


def _cyclic_measure(args, dist: Dist, cfg, dev, steps: int, warmup: int, e2e: bool):
    """b1n32768 through the block-cyclic driver: resident shards, a step copies the pristine
    shard into the work buffer and factors it; CUDA events around `steps` steps, maximum over
    ranks. With e2e, also the same with each rank's shard uploaded from and downloaded to
    pinned host memory inside the timed region."""
    from linalg_kernels_b200.distributed import CyclicLayout, factor_block_cyclic

    n = cfg.n
    lay = CyclicLayout(n, dist.world, dist.rank, 256)
    shard = _cyclic_shard(cfg, lay, dev)
    work = torch.empty_like(shard)
    pg = dist.pg if dist.world > 1 else None

    def step(_):
        work.copy_(shard)
        factor_block_cyclic(work, lay, pg=pg)

    with ClockSampler(dev.index) as clocks:
        total_ms, _ = _time_steps(step, [None], steps, warmup, dist)
    out = {"ms_per_step": dist.max(total_ms) / steps, "clocks": clocks.summary(), "lay": lay,
           "shard_bytes": shard.numel() * 4}
    if e2e:
        host_in = shard.cpu().pin_memory()
        host_out = torch.empty_like(host_in).pin_memory()

        def hstep():
            work.copy_(host_in, non_blocking=True)
            factor_block_cyclic(work, lay, pg=pg)
            host_out.copy_(work, non_blocking=True)

        for _ in range(2):
            hstep()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            hstep()
        e1.record()
        torch.cuda.synchronize()
        dist.barrier()
        out["e2e_ms_per_step"] = dist.max(e0.elapsed_time(e1)) / steps
    del work, shard
    torch.cuda.empty_cache()
    return out


def run_cyclic(args, dist: Dist):
    """One matrix over all ranks, 1-D block-column-cyclic, NCCL panel broadcasts
    (linalg_kernels_b200.distributed). Inputs are resident shards: every rank builds its own
    columns of A = X X^T / n + shift I. A step copies the pristine shard into the work
    buffer and factors it. Strong scaling: one matrix per step whatever the rank count."""
    from linalg_kernels_b200 import _lib, inputs

    _lib.load()
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    cfg = inputs.GRID[args.config]
    n = cfg.n
    r = _cyclic_measure(args, dist, cfg, dev, args.steps, args.warmup, e2e=True)
    value = 1e3 / r["ms_per_step"]
    nbytes = r["shard_bytes"]
    line = {
        "metric": "matrices/s", "value": value, "unit": "matrices/s", "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": (value / (1 / REFERENCE_PUBLISHED_S[cfg.name]) if dist.world == 1
                        else None),
        "dtype": "f32", "data": "synthetic", "tflops": value * n ** 3 / 3.0 / 1e12,
        "config": {"workload": cfg.name, "batch": 1, "n": n, "family": cfg.family,
                   "param": cfg.param, "seed": cfg.seed, "block": r["lay"].bs,
                   "parallelism": f"1-D block-column-cyclic over {dist.world} GPUs, NCCL "
                                  f"broadcast of each factored 256-wide panel",
                   "l2": "input 4 GiB > L2"},
        "roofline": None,
        "e2e": {"value": 1e3 / r["e2e_ms_per_step"], "unit": "matrices/s",
                "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
                "note": "per rank: its resident shard in and out"},
        "cpu_baseline": None,
        "clocks": r["clocks"],
        "gpu_launches": None,
    }
    if dist.rank == 0:
        print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------
# N > 1: the multi-GPU schedules of the larger configs, each gated against one GPU
# --------------------------------------------------------------------------------------
def _agree(dist: Dist, ok: bool) -> bool:
    """Rank 0's verdict, on every rank (the same collective on all of them)."""
    t = torch.tensor([1.0 if ok else 0.0], dtype=torch.float64, device="cuda")
    dist.pg.broadcast(t, src=0)
    return bool(t.item() > 0.5)


def _gate(a: torch.Tensor, l: torch.Tensor, l_one: torch.Tensor, cond: torch.Tensor) -> dict:
    """The north star's gates for a factor l of a (both (b, n, n) on one GPU) against the
    one-GPU factor l_one: the device checker's gates (relative residual <= 1e-5, scaled
    inf-norm residual, structure) and max|L - L_one| <= cond(A) n eps_fp32 max|L_one| per
    matrix (cond: the generator's per-matrix bound)."""
    from linalg_kernels_b200 import validate

    good, msg = validate.check_implementation(a, l)
    v = validate.validate(a, l)
    cond = cond.to(a.device)
    n = a.shape[-1]
    diff = (l - l_one).abs().amax(dim=(1, 2)).double()
    scale = l_one.abs().amax(dim=(1, 2)).double()
    bound = cond * n * validate.EPS32 * scale
    within = bool((diff <= bound).all())
    return {"ok": bool(good and within), "check": msg or "ok",
            "rel_residual_max": _sig(float(v["rel_residual"].max())),
            "max_diff_over_bound": _sig(float((diff / bound).max()))}


def _cyclic_parity(dist: Dist, dev, n: int = 4096) -> dict:
    """One n x n covariance matrix factored by the block-cyclic driver over all ranks,
    gathered to rank 0 and gated against the one-GPU factor of the same matrix."""
    from linalg_kernels_b200 import inputs
    from linalg_kernels_b200.cholesky import custom_kernel
    from linalg_kernels_b200.distributed import (CyclicLayout, factor_block_cyclic,
                                                 gather_block_cyclic, scatter_block_cyclic)

    a, cond = inputs.covariance(1, n, 0.5, 48000 + n, device=dev)
    lay = CyclicLayout(n, dist.world, dist.rank, 256)
    if lay.nblocks % dist.world:
        raise ValueError("parity case needs whole rounds of blocks")
    local = scatter_block_cyclic(a[0], lay)
    factor_block_cyclic(local, lay, pg=dist.pg)
    parts = [torch.empty_like(local) for _ in range(dist.world)]
    dist.pg.all_gather(parts, local)
    res = {"ok": True}
    if dist.rank == 0:
        full = gather_block_cyclic(parts, n, dist.world, 256)
        res = _gate(a, full[None], custom_kernel(a), cond)
    res["ok"] = _agree(dist, res["ok"])
    return res


def _sharded(dist: Dist, cfg, dev, steps: int, warmup: int) -> dict:
    """One config's batch over all ranks (strong scaling: the config's batch, split).
    resident: every rank factors its own slice (no transfer); from_root: the whole batch on
    rank 0's GPU, slices out and factors back by NCCL point-to-point (factor_batch_sharded),
    the first run gated against rank 0's one-GPU factor of the same batch."""
    from linalg_kernels_b200 import inputs
    from linalg_kernels_b200.cholesky import custom_kernel
    from linalg_kernels_b200.distributed import batch_slices, factor_batch_sharded

    b, n = cfg.batch, cfg.n
    a, cond = inputs.config_input(cfg, device=dev) if dist.rank == 0 else (None, None)
    res: dict = {}
    l = factor_batch_sharded(a, b, n, dist.pg, root=0)
    ok = True
    if dist.rank == 0:
        g = _gate(a, l, custom_kernel(a), cond)
        ok = g["ok"]
        res["gate"] = {k: v for k, v in g.items() if k != "ok"}
    res["parity"] = _agree(dist, ok)
    del l

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        dist.barrier()
        return dist.max(e0.elapsed_time(e1)) / steps

    off, cnt = batch_slices(b, dist.world)[dist.rank]
    mine = inputs.config_input(cfg, device=dev)[0][off:off + cnt].contiguous() \
        if dist.rank != 0 else a[off:off + cnt]
    res["resident_ms"] = _sig(timed(lambda: custom_kernel(mine)))
    res["from_root_ms"] = _sig(timed(lambda: factor_batch_sharded(a, b, n, dist.pg, root=0)))
    res["one_gpu_published_ms"] = REFERENCE_PUBLISHED_S[cfg.name] * 1e3
    res["nvlink_bytes_per_step"] = 2.0 * (b - batch_slices(b, dist.world)[0][1]) * n * n * 4
    del a, mine
    torch.cuda.empty_cache()
    return res


def _bcast_ms(dist: Dist, dev, nbytes: int, reps: int = 10) -> float:
    """NCCL broadcast of nbytes from rank 0 (the largest panel of the block-cyclic driver at
    n = 32768 is 32 MiB): CUDA events around reps broadcasts, maximum over ranks."""
    buf = torch.empty(nbytes // 4, dtype=torch.float32, device=dev)
    for _ in range(3):
        dist.pg.broadcast(buf, src=0)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        dist.pg.broadcast(buf, src=0)
    e1.record()
    torch.cuda.synchronize()
    return dist.max(e0.elapsed_time(e1)) / reps


def _multi_gpu(args, dist: Dist, dev, peaks) -> dict:
    from linalg_kernels_b200 import inputs
    from linalg_kernels_b200.distributed import auto_queues

    out: dict = {}
    cp = _cyclic_parity(dist, dev)
    out["cyclic_parity_b1n4096"] = cp
    gates = [cp["ok"]]
    big = inputs.GRID["b1n32768"]
    r = _cyclic_measure(args, dist, big, dev, steps=max(1, min(args.steps, 5)), warmup=3,
                        e2e=False)
    ms = r["ms_per_step"]
    bc32 = _bcast_ms(dist, dev, 32 << 20)
    out["cyclic_b1n32768"] = {
        "ms_per_step": _sig(ms), "tflops": _sig(big.n ** 3 / 3.0 / (ms / 1e3) / 1e12),
        "reference_one_gpu_ms": REFERENCE_PUBLISHED_S["b1n32768"] * 1e3,
        "vs_reference_published": _sig(REFERENCE_PUBLISHED_S["b1n32768"] * 1e3 / ms),
        "panels": r["lay"].nblocks, "bcast_ms_32MiB": _sig(bc32),
        "bcast_gbs_32MiB": _sig((32 << 20) / (bc32 / 1e3) / 1e9),
        "bcast_ms_all_panels_serial": _sig(sum(
            bc32 * (big.n - j * 256) / big.n for j in range(r["lay"].nblocks))),
        "parallelism": f"1-D block-column-cyclic over {dist.world} GPUs (256-wide blocks), "
                       f"NCCL broadcast of each factored panel, depth-2 look-ahead on a chain "
                       f"queue beside the trailing update on a bulk queue, GEMM CTA caps "
                       f"{auto_queues(dist.world)}, strong scaling"}
    for name in ("b640n512", "b60n1024"):
        sh = _sharded(dist, inputs.GRID[name], dev, steps=10, warmup=3)
        gates.append(sh.pop("parity"))
        out[name] = sh
    out["parity"] = all(gates)
    return out


def _sig(x: float) -> float:
    return float(f"{x:.4g}")


def _other_shapes(args, skip, dev, peaks, peak_kind, lib):
    """Every other benchmark-grid entry through custom_kernel on resident inputs: one compact
    row each, [ms per call, the reference's published ms, its ratio to ours, roofline
    fraction] (the fraction of measured HBM bandwidth at 8 n^2 bytes per matrix for n <= 256,
    of the TF32 rate at n^3/3 flops per matrix above)."""
    from linalg_kernels_b200 import inputs
    from linalg_kernels_b200.cholesky import custom_kernel

    out = {"cols": ["ms", "ref_ms", "vs_ref", "frac"],
           "frac": "of measured hbm_gbs (n<=256) / of bf16_tflops/2 (n>256)"}
    names = [k for k in inputs.GRID if k != skip and (args.big or k != "b1n32768")]
    for name in names:
        cfg = inputs.GRID[name]
        pool, pool_bytes = _pool(cfg, dev, 0, max_inputs=16)
        # enough calls that the timed region is ~ms long (the event bracket's fixed cost
        # is then noise): 200 for the microsecond shapes, at most 20 for the others
        steps = 200 if cfg.n <= 128 else max(3, min(args.steps, 20 if cfg.n < 32768 else 5))
        total, per = _time_steps(custom_kernel, pool, steps, 3, _NoDist())
        ms = total / steps
        if cfg.n <= 256:
            frac = 8.0 * cfg.n ** 2 * cfg.batch / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]
        else:
            frac = cfg.batch * cfg.n ** 3 / 3.0 / (ms / 1e3) / 1e12 / (peaks["bf16_tflops"] / 2.0)
        ref_ms = REFERENCE_PUBLISHED_S[name] * 1e3
        out[name] = [_sig(ms), _sig(ref_ms), _sig(ref_ms / ms), _sig(frac)]
        del pool
        torch.cuda.empty_cache()
    return out


def _validator_timing(dev, peaks, peak_kind, lib, names=("b1024n64", "b640n512", "b1n16384")):
    """The device-side checker (chol_validate_f32: the residual tiles in FP64, then the scan
    of L) on factors of grid inputs: time per call and its rates. Work per matrix: the lower
    triangle of tril(L) tril(L)^T, sum_c (c + 1)(n - c) ~ n^3/6 FP64 multiply-adds (n^3/3
    flops); bytes: A's lower triangle and L read once each (4 n^2 + ...) at least."""
    from linalg_kernels_b200 import _lib, inputs
    from linalg_kernels_b200.cholesky import custom_kernel

    rows = []
    for name in names:
        cfg = inputs.GRID[name]
        a, _ = inputs.config_input(cfg, device=dev)
        l = custom_kernel(a)
        b, n = cfg.batch, cfg.n
        out = torch.empty(b, 8, dtype=torch.float64, device=dev)
        work = torch.empty(int(lib.chol_validate_work_bytes(b, n)), dtype=torch.uint8, device=dev)
        q = ctypes.c_void_p(_lib.current_queue(dev))

        def call():
            _lib.check(lib.chol_validate_f32(ctypes.c_void_p(a.data_ptr()),
                                             ctypes.c_void_p(l.data_ptr()), b, n,
                                             ctypes.c_void_p(out.data_ptr()),
                                             ctypes.c_void_p(work.data_ptr()), q),
                       "chol_validate_f32")

        for _ in range(3):
            call()
        torch.cuda.synchronize()
        reps = 5
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            call()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / reps / 1e3
        flops = 2.0 * b * sum((c + 1) * (n - c) for c in range(n))
        bytes_ = 8.0 * b * n * n
        st = out.cpu()
        rows.append({"workload": name, "ms": t * 1e3, "fp64_tflops": flops / t / 1e12,
                     "min_bytes_gbs": bytes_ / t / 1e9,
                     "hbm_frac_of_measured": bytes_ / t / 1e9 / peaks["hbm_gbs"],
                     "rel_residual_max": float((st[:, 0].sqrt() / st[:, 1].sqrt()).max())})
        del a, l, out, work
        torch.cuda.empty_cache()
    return rows


def _grid_summary(name, ms_step, shapes):
    """The reference leaderboard's ranking figure (AGENTS.md:58-64): the geometric mean of the
    per-call runtimes over the benchmark-grid entries, ours and the reference's published,
    over the same entries."""
    ms = {k: v[0] for k, v in shapes.items() if k in REFERENCE_PUBLISHED_S}
    ms[name] = ms_step
    names = [k for k in ms if k in REFERENCE_PUBLISHED_S]
    ours = math.exp(sum(math.log(ms[k]) for k in names) / len(names))
    ref = math.exp(sum(math.log(REFERENCE_PUBLISHED_S[k] * 1e3) for k in names) / len(names))
    return {"entries": len(names), "geomean_ms": _sig(ours), "reference_geomean_ms": _sig(ref),
            "vs_reference_published": _sig(ref / ours)}


GEMM_PROBES = {
    # name: (m, ncols, K, lower_only, alpha, beta) of one C -= P Q^T launch on an 8192-row
    # panel; the roles of the blocked schedule's three GEMMs at n = 16384 scale
    "trailing": (8192, 8192, 512, 1, -1.0, 1.0),
    "inpanel": (8192, 448, 64, 1, -1.0, 1.0),
    "solve": (8192, 64, 64, 0, 1.0, 0.0),
}


def run_kernel_probe(args):
    """Time the tensor-core GEMM alone in each role (CUDA events, 10 launches after 3 warm)."""
    from linalg_kernels_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    peaks, peak_kind = _peaks()
    out = {}
    for name in args.probe.split(","):
        m, nc, k, lower, alpha, beta = GEMM_PROBES[name]
        g = torch.Generator(device=dev).manual_seed(1)
        p = torch.randn(m, k, device=dev, generator=g)
        c = torch.randn(m, nc, device=dev, generator=g)
        q = ctypes.c_void_p(_lib.current_queue(dev))

        def launch():
            st = lib.chol_gemm_nt_f32(ctypes.c_void_p(c.data_ptr()), 1, m * nc, nc, m, nc, k,
                                      ctypes.c_void_p(p.data_ptr()), m * k, k,
                                      ctypes.c_void_p(p.data_ptr()), m * k, k,
                                      alpha, beta, 0, lower, q)
            _lib.check(st, "chol_gemm_nt_f32")

        for _ in range(args.warmup):
            launch()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            launch()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / args.steps / 1e3
        if lower:
            flops = 2.0 * k * sum(min(r + 1, nc) for r in range(0, m, 1))
            cbytes = 8.0 * sum(min(r + 1, nc) for r in range(0, m, 1))
        else:
            flops = 2.0 * m * nc * k
            cbytes = (8.0 if beta else 4.0) * m * nc
        out[name] = {"m": m, "ncols": nc, "K": k, "ms": t * 1e3,
                     "tflops": flops / t / 1e12,
                     "tf32_frac_of_measured": flops / t / 1e12 / (peaks["bf16_tflops"] / 2.0),
                     "c_gbs": cbytes / t / 1e9, "hbm_frac_of_measured": cbytes / t / 1e9 / peaks["hbm_gbs"]}
    print(json.dumps({"kernel_probe": out, "peaks": peak_kind}), flush=True)


class _NoDist(Dist):
    def __init__(self):
        self.world, self.rank, self.local, self.pg = 1, 0, 0, None


def run_ncu_target(args):
    """The program the profiles/ ncu captures run: one input of the config (generated on the
    host for n <= 1024, so the only GPU kernels are ours), warm-up + steps calls of
    custom_kernel, nothing else (no timing, no baselines)."""
    from linalg_kernels_b200 import inputs
    from linalg_kernels_b200.cholesky import custom_kernel

    if args.config in inputs.GRID:
        cfg = inputs.GRID[args.config]
    else:  # any other shape, "b<batch>n<n>": spectral inputs, condition 1e3
        m = re.fullmatch(r"b(\d+)n(\d+)", args.config)
        if m is None:
            raise SystemExit(f"--ncu-run: unknown config {args.config!r}")
        cfg = inputs.Config(args.config, int(m.group(1)), int(m.group(2)), "spectral", 1e3, 7)
    dev = torch.device("cuda", 0)
    if not args.overlap:
        from linalg_kernels_b200 import _lib

        _lib.load().chol_set_option(_lib.CHOL_OPT_OVERLAP_CALLS, 0)
    gen_dev = "cpu" if cfg.n <= 1024 else dev
    a, _ = inputs.config_input(cfg, device=gen_dev)
    a = a.to(dev)
    torch.cuda.synchronize()
    for _ in range(args.warmup + args.steps):
        custom_kernel(a)
    torch.cuda.synchronize()
    print(json.dumps({"ncu_run": cfg.name, "calls": args.warmup + args.steps}))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default=DEFAULT_CONFIG)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=10.0,
                    help="seconds of CPU work for the cpu_baseline sample")
    ap.add_argument("--shapes", action=argparse.BooleanOptionalAction, default=True,
                    help="also time the other benchmark shapes (N=1 only)")
    ap.add_argument("--big", action=argparse.BooleanOptionalAction, default=True,
                    help="include b1n32768 in --shapes")
    ap.add_argument("--multi", action=argparse.BooleanOptionalAction, default=True,
                    help="N>1: also run the multi-GPU schedules (b1n32768 block-cyclic, batch "
                         "sharding of b640n512 and b60n1024 from rank 0's GPU) after a parity "
                         "gate of each against the one-GPU factor")
    ap.add_argument("--validate", action="store_true",
                    help="also time the device-side checker (chol_validate_f32) (N=1 only)")
    ap.add_argument("--cyclic", action="store_true",
                    help="b1n32768 through the block-cyclic driver even on one GPU")
    ap.add_argument("--probe", default=None,
                    help="time the tensor-core GEMM alone in the given roles "
                         "(comma list of trailing,inpanel,solve) and exit")
    ap.add_argument("--overlap", action=argparse.BooleanOptionalAction, default=True,
                    help="with --ncu-run: --no-overlap makes every n <= 64 call wait for the "
                         "one before it (CHOL_OPT_OVERLAP_CALLS = 0), the single-launch case "
                         "a serialising profiler sees anyway")
    ap.add_argument("--ncu-run", action="store_true",
                    help="only call custom_kernel warmup + steps times on one input of --config "
                         "(the target of the ncu captures in profiles/)")
    args = ap.parse_args(argv)
    if args.ncu_run:
        run_ncu_target(args)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.probe:
        run_kernel_probe(args)
        return
    if args.impl == "reference":
        # the CPU reference arm runs on rank 0 only; other ranks exit without work
        nd = _NoDist()
        nd.rank = int(os.environ.get("RANK", "0"))
        run_reference(args, nd)
        return
    dist = Dist()
    try:
        if args.config == "b1n32768" and (dist.world > 1 or args.cyclic):
            run_cyclic(args, dist)
        else:
            run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
