#!/usr/bin/env python
"""Benchmark of the fused SwiGLU hot path on B200 (one JSON line on stdout).

Workload (the configuration the headline metric is quoted on): Llama-7B
prefill SwiGLU, X[2048,4096] x Wg,Wu[4096,11008] bf16, f32 accumulation,
Y bf16.  One step = one launch of the fused kernel over the whole problem
(at N GPUs: this rank's column shard, 128-column tiles dealt out evenly; no
collective on the data path).  Inputs are seeded synthetic tensors of the
configured shapes and distributions.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

value: whole-job TFLOP/s = 4*M*N*K / (max over ranks of the summed
K back-to-back steps, one CUDA event pair), inputs resident in HBM; steps
cycle through enough distinct input sets that their total exceeds 2x L2, so
no step finds its inputs in L2.  e2e: the same metric through the C ABI
``llk_swiglu`` with pinned HOST buffers (H2D of X, Wg, Wu and D2H of Y in
the timed region, every step).  --impl reference times the CPU restatement
of the reference's fused AVX2 schedule on this host's cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIG = dict(name="c3", M=2048, K=4096, N=11008, x_std=1.0, w_std=0.02)
METRIC = "fused SwiGLU BF16 TFLOP/s (Llama-7B prefill shape, config 3)"
UNIT = "TFLOP/s"


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def measured_peaks():
    """{"burst", "sustained", "hbm", "source"} from MEASURED_PEAKS.json: bf16
    TFLOP/s of a cuBLAS GEMM timed alone (burst) and held for seconds under
    the power cap (sustained), and the HBM copy bandwidth in GB/s.  Without
    the file, the pool's earlier measurement (1590 / 1400 TFLOP/s, 6650 GB/s)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        burst = d.get("bf16_tflops") or d.get("bf16_tflops_sustained")
        return {"burst": burst, "sustained": d.get("bf16_tflops_sustained") or burst, "hbm": d.get("hbm_gbs"),
                "source": "measured"}
    return {"burst": 1590.0, "sustained": 1400.0, "hbm": 6650.0, "source": "fallback"}


def choose_peak(peaks, region_s, clocks):
    """The bf16 denominator for a timed region: the sustained figure when its
    own clock samples show sw_power_cap AND the cap held the clock down (the
    region ran over one second, or its median SM clock was under 0.9 of the
    maximum); the burst figure otherwise."""
    capped = bool(clocks) and "sw_power_cap" in (clocks.get("reasons") or [])
    held = False
    if capped:
        med, top = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
        held = region_s > 1.0 or (med is not None and top and med < 0.9 * top)
    if held:
        return peaks["sustained"], "sustained", (f"region {region_s:.3f} s with sw_power_cap in its clock samples, "
                                                 f"median SM clock {clocks.get('sm_mhz')} of {clocks.get('sm_max_mhz')} MHz")
    why = "no sw_power_cap in its clock samples" if not capped else "the power cap did not hold the clock down"
    return peaks["burst"], "burst", f"region {region_s:.3f} s, {why}"


def profile_traffic(kernel, shard_cols):
    """DRAM bytes (read + write) per launch of `kernel` on a shard of
    `shard_cols` columns, from the machine-readable ncu summary
    profiles/<kernel>.json ({"launches": [{"N": .., "dram_bytes": ..}, ..]});
    None when no capture of that width is recorded."""
    p = os.path.join(ROOT, "profiles", kernel + ".json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    for e in d.get("launches", []):
        if int(e.get("N", -1)) == int(shard_cols):
            return {"bytes": float(e["dram_bytes"]), "source": f"profiles/{kernel}.json ({e.get('what', '')})"}
    return None


_SAMPLER_SRC = r"""
import sys, time, pynvml
uuids, period, out = sys.argv[1].split(","), float(sys.argv[2]), sys.argv[3]
pynvml.nvmlInit()
hs = []
for i, u in enumerate(uuids):
    try:
        h = pynvml.nvmlDeviceGetHandleByUUID(u)
    except Exception:
        h = pynvml.nvmlDeviceGetHandleByIndex(i)
    hs.append((i, h, pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)))
rs = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
with open(out, "w", buffering=1) as f:
    while True:
        now = time.monotonic()
        for i, h, mx in hs:
            try:
                f.write("%.6f %d %d %d %.3f %d\n" % (now, i, pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), mx,
                                                     pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0, int(rs(h))))
            except Exception:
                pass
        time.sleep(period)
"""


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of the given CUDA
    devices, polled through NVML every few milliseconds by a separate
    process (so the sampling never competes with the launching thread for
    the interpreter lock), each sample time-stamped on the system-wide
    monotonic clock so that the samples inside the timed region can be told
    from those of the warm-up around it."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_devices, period_s=0.004):
        self.devs = list(cuda_devices)
        self.period = period_s
        self.rows = []  # (t, dev, sm_mhz, max_mhz, power_w, reason_bits)
        self.marks = {}
        self.proc = None
        self.path = None
        self.error = None

    def __enter__(self):
        try:
            import tempfile

            import torch

            uuids = []
            for d in self.devs:
                u = str(torch.cuda.get_device_properties(d).uuid)
                uuids.append(u if u.startswith("GPU-") else "GPU-" + u)
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".txt")
            os.close(fd)
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER_SRC, ",".join(uuids), str(self.period),
                                          self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.2)  # NVML initialised and sampling before the window opens
        except Exception as e:  # noqa: BLE001
            self.error = f"{type(e).__name__}: {e}"[:200]
        return self

    def mark(self, name):
        self.marks[name] = time.monotonic()

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()
            self.proc = None
        if self.path and os.path.exists(self.path):
            with open(self.path) as f:
                for line in f:
                    p = line.split()
                    if len(p) == 6:
                        try:
                            self.rows.append((float(p[0]), self.devs[int(p[1])], int(p[2]), int(p[3]), float(p[4]),
                                              int(p[5])))
                        except (ValueError, IndexError):
                            pass
            os.unlink(self.path)
            self.path = None

    def summary(self, begin="timed_begin", end="timed_end"):
        """Samples inside [begin, end]; when the region is shorter than the
        polling period and holds none, the samples of the whole loaded
        window (warm-up start to region end) stand in, and say so."""
        if self.error and not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "error": self.error}
        t0, t1 = self.marks.get(begin), self.marks.get(end)
        rows = [r for r in self.rows if t0 is not None and t1 is not None and t0 <= r[0] <= t1]
        scope = "timed region"
        if not rows:
            w0 = self.marks.get("window_begin", t0)
            rows = [r for r in self.rows if w0 is not None and t1 is not None and w0 <= r[0] <= t1]
            scope = "warm-up + timed region (region shorter than the polling period)"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "scope": scope}
        reasons = sorted({name for r in rows for bit, name in self.REASONS.items() if r[5] & bit})
        return {"sm_mhz": statistics.median(r[2] for r in rows), "sm_max_mhz": max(r[3] for r in rows),
                "sm_mhz_min": min(r[2] for r in rows), "reasons": reasons, "samples": len(rows),
                "power_w_max": max(r[4] for r in rows), "scope": scope, "source": "NVML, polled every "
                f"{self.period * 1e3:.0f} ms by a separate process"}


def cpu_port_run(x, wg, wu, rows, threads):
    import oracle

    t0 = time.perf_counter()
    oracle.port_swiglu(x[:rows], wg, wu, "bf16", threads=threads)
    return time.perf_counter() - t0


def cpu_baseline(x, wg, wu, budget_s=12.0):
    """The threaded fused-schedule CPU port on this host, on a bounded row
    sample of the workload, repeated for about `budget_s` seconds."""
    import oracle

    oracle.build()
    threads = os.cpu_count() or 1
    rows = 64
    K, N = wg.shape
    t = cpu_port_run(x, wg, wu, rows, threads)  # warm-up + size probe
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or not times:
        times.append(cpu_port_run(x, wg, wu, rows, threads))
    best = min(times)
    return {"value": 4.0 * rows * N * K / best / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{rows} of {x.shape[0]} token rows x full N={N}, K={K}; best of {len(times)} runs "
                      f"(~{sum(times) + t:.0f} s); oracle/swiglu_port.c fused schedule BM=32 BN=64 BK=64"}


def reference_naive_baseline():
    """The reference's own naive f32 swiglu_reference (its test oracle,
    compiled from the reference's sources into oracle/_ref/ref_driver when
    the reference tree was present at build time), one thread, on configs 1
    and 4 (M = 1): what the reference runs on the CPU for this op.  None when
    the binary is absent."""
    exe = os.path.join(ROOT, "oracle", "_ref", "ref_driver")
    if not os.access(exe, os.X_OK):
        return None
    out = {}
    for name, (M, N, K, reps) in {"c1": (64, 512, 256, 5), "c4_m1": (1, 14336, 4096, 2)}.items():
        try:
            r = subprocess.run([exe, "time", str(M), str(N), str(K), str(reps)], capture_output=True, text=True,
                               timeout=120)
            sec = float(r.stdout.split()[0])
        except Exception as e:  # noqa: BLE001
            out[name] = {"error": str(e)[:200]}
            continue
        out[name] = {"gflops": 4.0 * M * N * K / sec / 1e9, "ms": sec * 1e3, "threads": 1,
                     "shape": f"M={M} N={N} K={K}"}
    return {"kind": "reference", "what": "test/Execution/swiglu_reference.cpp swiglu_reference (naive f32 loops)",
            "configs": out}


def reference_arm(args):
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    from dslcompiler_b200 import datagen as dg
    import oracle

    oracle.build()
    M, K, N = CONFIG["M"], CONFIG["K"], CONFIG["N"]
    x, wg, wu = dg.swiglu_inputs(M, K, N, CONFIG["x_std"], CONFIG["w_std"], seed=42)
    threads = os.cpu_count() or 1
    rows = 32
    for _ in range(args.warmup):
        cpu_port_run(x, wg, wu, rows, threads)
    times = [cpu_port_run(x, wg, wu, rows, threads) for _ in range(args.steps)]
    mean = sum(times) / len(times)
    value = 4.0 * rows * N * K / mean / 1e12
    sample = (f"each step: {rows} of {M} token rows x full N={N}, K={K} (bounded sample of the workload); "
              f"CPU restatement of the reference's fused AVX2 schedule (oracle/swiglu_port.c) on {threads} threads")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean * 1e3, "sample_rows": rows,
            "ms_per_step_what": f"measured time of one step as run: {rows} token rows x full N, K (the rate "
                                f"`value` is 4*rows*N*K / that time); the whole {M}-row workload would take "
                                f"about {mean * 1e3 * M / rows:.0f} ms per step at this rate",
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded splitmix64/Box-Muller, X~N(0,1), W~N(0,0.02), bf16)",
            "config": {"workload": "c3 llama7b-prefill swiglu", "M": M, "K": K, "N": N, "math_mode": "strict", "sample_rows": rows},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's own path (MLIR/LLVM ORC JIT) cannot be built here; its naive test oracle is "
                    "slower than this port, so the port is the faster, conservative CPU arm"}
    print(json.dumps(line), flush=True)
    return 0


class stdout_to_stderr:
    """Points file descriptor 1 at stderr for the duration (C libraries
    included)."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *a):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)


def bf16_tensor(a_u16, pin=False):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a_u16).view(np.int16)).view(torch.bfloat16)
    return t.pin_memory() if pin else t


def input_sets(dev, tensors, l2_bytes):
    """Enough distinct copies of a step's device tensors that together they
    exceed twice the L2: back-to-back steps cycling through them never find
    their inputs in L2 from an earlier step."""
    import torch

    per = sum(t.numel() * t.element_size() for t in tensors)
    n = max(1, min(16, -(-2 * l2_bytes // per)))
    sets = [tuple(tensors)] + [tuple(t.clone() for t in tensors) for _ in range(n - 1)]
    torch.cuda.synchronize(dev)
    return sets, per


def time_back_to_back(fn, steps, stream):
    """Total CUDA-event time (ms) of `steps` back-to-back calls fn(i)."""
    import torch

    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(steps):
        fn(i)
    e.record(stream)
    torch.cuda.synchronize()
    return s.elapsed_time(e)


def time_steps(fn, flush, steps, stream):
    """Per-step CUDA-event durations (ms) of fn() (host-synchronous steps such
    as the host-buffer e2e calls); flush, if given, runs before each step."""
    import torch

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for s, e in evs:
        if flush is not None:
            flush()
        s.record(stream)
        fn()
        e.record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in evs]


def _bits(t):
    """bf16 torch tensor (any device) -> numpy uint16 bit patterns."""
    import torch

    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def points_rel_err(x, wg, wu, y, rows, cols):
    """max |y - ref| / max |ref| over the points (rows[i], cols[i]) of y,
    ref = the FP64 oracle (oracle/swiglu_oracle.c, the checker) on the same
    bf16 inputs.  x [M, K], wg / wu [K, n] (numpy uint16 bit patterns or
    bf16 torch tensors on any device), y [M, n] torch (bf16 or f32).  Only
    the rows of X and columns of W the points touch are copied to the host."""
    import torch

    import oracle

    rows = np.asarray(rows, np.int64)
    cols = np.asarray(cols, np.int64)
    ur, ri = np.unique(rows, return_inverse=True)
    uc, ci = np.unique(cols, return_inverse=True)

    def take(t, idx, dim):
        if isinstance(t, np.ndarray):
            return np.ascontiguousarray(np.take(t, idx, axis=dim))
        return _bits(t.index_select(dim, torch.as_tensor(idx, device=t.device)))

    xc, gc, uc_ = take(x, ur, 0), take(wg, uc, 1), take(wu, uc, 1)
    ref = oracle.swiglu_fp64_points(xc, gc, uc_, ri, ci)
    yv = y[torch.as_tensor(rows, device=y.device), torch.as_tensor(cols, device=y.device)]
    yv = yv.double().cpu().numpy()
    if not np.all(np.isfinite(yv)):
        return float("inf")
    return float(np.abs(yv - ref).max() / max(np.abs(ref).max(), 1e-30))


def parity_points(M, n, seed, boundaries=(), n_random=2048):
    """Check points of an [M, n] output: n_random seeded random points, one
    whole row, and the two columns on either side of every boundary (shard
    edges) at 64 rows."""
    rng = np.random.default_rng(seed)
    rows = [rng.integers(0, M, n_random), np.full(n, int(rng.integers(0, M)))]
    cols = [rng.integers(0, n, n_random), np.arange(n)]
    for b in boundaries:
        for c in (b - 1, b):
            if 0 <= c < n:
                r = rng.integers(0, M, 64)
                rows.append(r)
                cols.append(np.full(64, c))
    return np.concatenate(rows), np.concatenate(cols)


TOL_BF16 = 1e-2  # bf16 Y: max |y - ref| <= 1e-2 * max |ref| (the north star's tolerance)


def our_arm(args):
    import torch
    import torch.distributed as dist

    import dslcompiler_b200 as llk
    from dslcompiler_b200 import datagen as dg

    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        # NCCL may print its banner on stdout when the communicator comes up;
        # keep stdout for the one JSON line.
        with stdout_to_stderr():
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
            dist.barrier(device_ids=[local])
            torch.cuda.synchronize()
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)

    M, K, N = CONFIG["M"], CONFIG["K"], CONFIG["N"]
    x, wg, wu = dg.swiglu_inputs(M, K, N, CONFIG["x_std"], CONFIG["w_std"], seed=42)
    b, e = llk.shard_columns(N, world, rank)
    n_r = e - b
    wg_s = np.ascontiguousarray(wg[:, b:e])
    wu_s = np.ascontiguousarray(wu[:, b:e])

    xd, gd, ud = bf16_tensor(x).to(dev), bf16_tensor(wg_s).to(dev), bf16_tensor(wu_s).to(dev)
    yd = torch.empty((M, n_r), dtype=torch.bfloat16, device=dev)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    sets, set_bytes = input_sets(dev, [xd, gd, ud, yd], l2)

    def step(i):
        a, b, c, d = sets[i % len(sets)]
        llk.fused_swiglu(a, b, c, out=d)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def reduce_over_ranks(v, op):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=op)
        return float(t.item())

    def max_over_ranks(v):
        return reduce_over_ranks(v, dist.ReduceOp.MAX if world > 1 else None)

    def sum_over_ranks(v):
        return reduce_over_ranks(v, dist.ReduceOp.SUM if world > 1 else None)

    # ---------------------------------------------------------- value
    sampler = ClockSampler(range(world)) if local == 0 else None
    if sampler:
        sampler.__enter__()
        sampler.mark("window_begin")
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    llk.synchronize(local)
    barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.mark("timed_begin")
    t_wall0 = time.perf_counter()
    kernel_ms = time_back_to_back(step, args.steps, stream)
    t_wall = time.perf_counter() - t_wall0
    if sampler:
        sampler.mark("timed_end")
    barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__()
    llk.synchronize(local)
    job_ms = max_over_ranks(kernel_ms) / args.steps
    total_flops = 4.0 * M * N * K
    value = total_flops / (job_ms * 1e-3) / 1e12
    clocks = sampler.summary() if sampler else None

    # ------------------------------------------------------- parity (this rank's shard)
    parity = {}
    rows, cols = parity_points(M, n_r, seed=1000 + rank)
    err = points_rel_err(x, wg_s, wu_s, sets[0][3], rows, cols)
    parity["headline_shard"] = {"max_rel_err": max_over_ranks(err), "points_per_rank": int(rows.size)}

    # ------------------------------------------------------- roofline
    peaks = measured_peaks()
    peak_tf, peak_kind, peak_why = choose_peak(peaks, kernel_ms * 1e-3, clocks)
    my_ms = kernel_ms / args.steps
    achieved = 4.0 * M * n_r * K / (my_ms * 1e-3) / 1e12
    traffic = profile_traffic("tc2_swiglu_c3", n_r)
    alg_bytes = 2 * M * K + 4 * K * n_r + 2 * M * n_r

    # ----------------------------------------------------------- e2e
    # Through the reference-facing C ABI (llk_swiglu) with pinned host
    # buffers: every step copies X, Wg, Wu (this rank's shard) in and Y out.
    xh, gh, uh = bf16_tensor(x, pin=True), bf16_tensor(wg_s, pin=True), bf16_tensor(wu_s, pin=True)
    yh = torch.empty((M, n_r), dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(3, min(args.steps, 30))
    torch.cuda.set_device(local)

    def e2e_step():
        st = llk.swiglu_c_abi(xh, gh, uh, yh)
        if st != 0:
            raise RuntimeError(f"llk_swiglu failed: {st}")

    for _ in range(2):
        e2e_step()
    barrier()
    dstream = torch.cuda.default_stream(dev)
    e2e_times = time_steps(e2e_step, None, e2e_steps, dstream)
    barrier()
    e2e_ms = max_over_ranks(sum(e2e_times)) / e2e_steps
    h2d = sum_over_ranks(float(xh.numel() * 2 + gh.numel() * 2 + uh.numel() * 2))
    d2h = sum_over_ranks(float(yh.numel() * 2))
    e2e = {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
           "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_ms,
           "path": "llk_swiglu C ABI, pinned host X/Wg/Wu/Y, copies in the timed region"}
    parity["e2e_host_buffers"] = {"max_rel_err": max_over_ranks(points_rel_err(x, wg_s, wu_s, yh, rows, cols))}
    # Packed weights (PackedWeights + L4-cache role): weights resident,
    # X in / Y out per step.
    pw = llk.PackedWeights(gd, ud)

    def e2e_packed_step():
        pw(xh, out=yh)

    for _ in range(2):
        e2e_packed_step()
    p_times = time_steps(e2e_packed_step, None, e2e_steps, dstream)
    p_ms = max_over_ranks(sum(p_times)) / e2e_steps
    e2e_packed = {"value": total_flops / (p_ms * 1e-3) / 1e12, "unit": UNIT,
                  "h2d_bytes_per_step": int(sum_over_ranks(float(xh.numel() * 2))),
                  "d2h_bytes_per_step": int(d2h), "ms_per_step": p_ms}
    pw.close()

    extras = {}
    n_sets = len(sets)
    if world > 1:
        extras["gather_y"] = secondary(lambda: gather_timing(args, dev, stream, yd, N, world, barrier, max_over_ranks,
                                                             (x, wg, wu)))
        if "error" not in extras["gather_y"]:
            extras["fused_allgather"] = secondary(lambda: fused_allgather_timing(
                args, dev, stream, xd, gd, ud, N, barrier, max_over_ranks, job_ms, extras["gather_y"]["ms"],
                (x, wg, wu)))
    cpu = None
    if not args.quick:
        del sets, xd, gd, ud, yd
        torch.cuda.empty_cache()
        extras.update(secondary(lambda: sharded_extras(args, dev, stream, rank, world, peaks, barrier,
                                                       max_over_ranks), "sharded_extras"))
        if world == 1:
            extras.update(secondary(lambda: single_gpu_extras(args, dev, stream, peaks, value),
                                    "single_gpu_extras"))
            if not args.no_cpu_baseline:
                cpu = cpu_baseline(x, wg, wu)
                naive = secondary(reference_naive_baseline)
                if naive:
                    cpu["reference_naive"] = naive

    # every parity figure of the run, headline and secondary, in one place
    for key, v in extras.items():
        if isinstance(v, dict):
            if "parity" in v:
                parity[key] = v["parity"]
            for cfg, r in v.items():
                if isinstance(r, dict) and "parity" in r:
                    parity[f"{key}.{cfg}"] = r["parity"]
    expected = ["headline_shard", "e2e_host_buffers"]
    if world > 1:
        expected += ["gather_y", "fused_allgather"]
    if not args.quick:
        expected += ["decode_c4.c4_m1", "decode_c4.c4_m4", "decode_c4.c4_m16", "decode_c4.c4_m1_f32", "swiglu_c5"]
        if world == 1:
            expected += ["matmul_c2", "rope", "attention"]
    missing = [k for k in expected if k not in parity]
    worst = max((p["max_rel_err"] for p in parity.values()), default=float("inf"))
    # each check against its own tolerance (FP32 outputs carry a tighter one)
    within = all(p["max_rel_err"] <= p.get("tol", TOL_BF16) for p in parity.values())
    parity_line = {"max_rel_err": worst, "tol": TOL_BF16, "ok": bool(within and not missing),
                   "missing": missing, "checks": parity,
                   "oracle": "FP64 at sampled points (oracle/swiglu_oracle.c), every rank its own columns; full-Y "
                             "paths: every rank the whole Y incl. both sides of each shard boundary"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": job_ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded splitmix64/Box-Muller, X~N(0,1), W~N(0,0.02), rounded to bf16)",
            "config": {"workload": "c3 llama7b-prefill swiglu", "M": M, "K": K, "N": N,
                       "parallelism": f"N-column-sharded x{world} (no collective)" if world > 1 else "single GPU",
                       "shard_cols_rank0": n_r,
                       "l2": f"no flush: back-to-back steps cycle {n_sets} distinct input sets of "
                             f"{set_bytes / 2**20:.0f} MiB (together >= 2 x the {l2 / 2**20:.0f} MiB L2)",
                       "timing": "one CUDA event pair around all timed steps (launches back to back), "
                                 "max over ranks"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved / peak_tf, "peak_kind": peak_kind,
                         "peak_why": f"{peaks['source']} bf16 {peak_kind}: {peak_why}",
                         "frac_of_burst": achieved / peaks["burst"],
                         "frac_of_sustained": achieved / peaks["sustained"],
                         "traffic": traffic["bytes"] if traffic else None,
                         "traffic_source": traffic["source"] if traffic else "no ncu capture of this shard width",
                         "algorithmic_bytes": alg_bytes,
                         "kernel": "tc2_kernel<TC_SWIGLU_BF16> (CTA pairs)" if M > 128 else
                                   "tc_swiglu_kernel<TC_SWIGLU_BF16>",
                         "algorithmic_work": "4*M*N_rank*K FLOP per launch (rank 0's shard)"},
            "e2e": e2e, "e2e_packed_weights": e2e_packed,
            "parity": parity_line,
            "gpu_launches": args.steps,
            "clocks": clocks,
            "wall_s_timed_region": t_wall,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if not parity_line["ok"]:
        print(f"PARITY FAILURE: max rel err {worst:.3e} > {TOL_BF16}: {json.dumps(parity)}", file=sys.stderr)
        return 3
    return 0


def full_y_parity(y_full, host_inputs, bounds, rank, max_over_ranks):
    """Every rank checks the whole Y it holds: random points, one whole row
    and both sides of every shard boundary, against the FP64 oracle."""
    x, wg, wu = host_inputs
    M, N = y_full.shape
    rows, cols = parity_points(M, N, seed=2000 + rank, boundaries=[b for b, _ in bounds[1:]])
    err = points_rel_err(x, wg, wu, y_full, rows, cols)
    return {"max_rel_err": max_over_ranks(err), "points_per_rank": int(rows.size)}


def gather_timing(args, dev, stream, yd, N, world, barrier, max_over_ranks, host_inputs):
    """Optional full-Y path: NCCL all-gather of the padded shards plus the
    llk_gather_columns relayout -- timed apart from the kernel."""
    import torch
    import torch.distributed as dist

    from dslcompiler_b200.sharding import gather_columns, shard_bounds

    bounds = shard_bounds(N, world)
    width = max(e - b for b, e in bounds)
    M = yd.shape[0]
    buf = torch.zeros((M, width), dtype=yd.dtype, device=dev)
    buf[:, : yd.shape[1]].copy_(yd)
    gathered = torch.empty((world, M, width), dtype=yd.dtype, device=dev)
    y_full = torch.empty((M, N), dtype=yd.dtype, device=dev)

    def step():
        dist.all_gather_into_tensor(gathered, buf)
        gather_columns(gathered, bounds, y_full)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    barrier()
    steps = max(5, min(args.steps, 50))
    t = time_steps(step, None, steps, stream)
    ms = max_over_ranks(sum(t)) / steps
    recv = (world - 1) * M * width * yd.element_size()
    torch.cuda.synchronize()
    rank = dist.get_rank()
    par = full_y_parity(y_full, host_inputs, bounds, rank, max_over_ranks)
    return {"ms": ms, "bytes_received_per_gpu": recv, "GB/s_per_gpu": recv / (ms * 1e-3) / 1e9,
            "what": "all_gather_into_tensor (NCCL) of padded Y shards + llk_gather_columns relayout",
            "parity": par}


def secondary(fn, key=None):
    """Runs a secondary measurement; an exception is reported in the JSON
    line (under `key` when given) instead of ending the run, so the headline
    line is always printed.  Every rank runs the same measurements, so they
    fail alike and no rank is left waiting in a collective."""
    try:
        return fn()
    except Exception as e:  # noqa: BLE001
        import traceback

        traceback.print_exc(file=sys.stderr)
        err = {"error": f"{type(e).__name__}: {e}"[:300]}
        return {key: err} if key else err


def fused_allgather_timing(args, dev, stream, xd, gd, ud, N, barrier, max_over_ranks, kernel_ms, gather_ms,
                           host_inputs):
    """The full-Y path with the all-gather fused into the kernel
    (llk_swiglu_column_parallel: each rank's epilogue stores its columns
    into every rank's Y over NVLink, plus the entry / exit barriers), against
    kernel + NCCL all-gather + relayout."""
    import torch

    from dslcompiler_b200.sharding import PeerGroupSwiGLU

    M, K = xd.shape
    layer = PeerGroupSwiGLU(gd, ud, N, max_rows=M, already_sharded=True, pack=False, device=dev.index)
    for _ in range(3):
        layer(xd)
    torch.cuda.synchronize()
    barrier()
    steps = max(5, min(args.steps, 200))
    ms = max_over_ranks(time_back_to_back(lambda i: layer(xd), steps, stream)) / steps
    torch.cuda.synchronize()
    barrier()
    # The Y of the last timed call, as this rank holds it (its own columns
    # written locally, every other rank's columns stored by that rank's kernel
    # over NVLink).
    y_last = layer.y(M).clone()
    torch.cuda.synchronize()
    barrier()
    layer.close()
    from dslcompiler_b200.sharding import shard_bounds

    par = full_y_parity(y_last, host_inputs, shard_bounds(N, layer.world), layer.rank, max_over_ranks)
    flops = 4.0 * M * N * K
    bytes_out = (layer.world - 1) * M * (layer.end - layer.begin) * 2
    return {"ms": ms, "tflops_whole_job": flops / (ms * 1e-3) / 1e12, "parity": par,
            "nvlink_bytes_out_per_gpu": bytes_out, "GB/s_out_per_gpu": bytes_out / (ms * 1e-3) / 1e9,
            "kernel_plus_nccl_gather_ms": kernel_ms + gather_ms,
            "tflops_kernel_plus_nccl_gather": flops / ((kernel_ms + gather_ms) * 1e-3) / 1e12,
            "what": "llk_swiglu_column_parallel: full Y on every GPU, shards stored to peers by the kernel epilogue"}


def single_gpu_extras(args, dev, stream, peaks, headline_tflops):
    """Secondary measurements on one GPU, same timing rules: the micro.mma
    matmul (config 2), and a cuBLAS yardstick (torch.matmul, a library GEMM
    timed beside ours, not part of the product) for both config 3 -- the
    same FLOPs as X.[Wg|Wu] with no epilogue -- and config 2."""
    import torch

    import dslcompiler_b200 as llk
    from dslcompiler_b200 import datagen as dg

    out = {}
    steps = max(5, min(args.steps, 200))
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    a, b = dg.config_inputs("c2")
    ad, bd = bf16_tensor(a).to(dev), bf16_tensor(b).to(dev)
    cd = torch.empty((4096, 4096), dtype=torch.float32, device=dev)
    msets, _ = input_sets(dev, [ad, bd, cd], l2)

    def fn(i):
        x_, w_, c_ = msets[i % len(msets)]
        llk.matmul(x_, w_, c_)

    for i in range(3):
        fn(i)
    ms = time_back_to_back(fn, steps, stream) / steps
    torch.cuda.synchronize()
    llk.synchronize(dev.index)
    mm_tf = 2.0 * 4096 ** 3 / (ms * 1e-3) / 1e12
    # parity: 2048 points of C against an f64 dot product of the bf16 operands
    rng = np.random.default_rng(7)
    r, c = rng.integers(0, 4096, 2048), rng.integers(0, 4096, 2048)
    af = torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).double()
    bf = torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).double()
    ref = (af[torch.as_tensor(r)] * bf[:, torch.as_tensor(c)].T).sum(1).numpy()
    got = msets[0][2][torch.as_tensor(r, device=dev), torch.as_tensor(c, device=dev)].double().cpu().numpy()
    mm_err = float(np.abs(got - ref).max() / np.abs(ref).max())

    # cuBLAS on the same shapes and rotation
    def cublas_ms(A, B, out_dtype):
        sets_, _ = input_sets(dev, [A, B], l2)
        kw = {"out_dtype": out_dtype} if out_dtype is not None else {}

        def g(i):
            x_, w_ = sets_[i % len(sets_)]
            torch.mm(x_, w_, **kw)

        for i in range(3):
            g(i)
        return time_back_to_back(g, steps, stream) / steps

    try:
        cb2_ms = cublas_ms(ad, bd, torch.float32)
        cb2_what = "torch.mm bf16 x bf16 -> f32 (out_dtype)"
    except (TypeError, RuntimeError):
        cb2_ms = cublas_ms(ad, bd, None)
        cb2_what = "torch.mm bf16 x bf16 -> bf16"
    cb2_tf = 2.0 * 4096 ** 3 / (cb2_ms * 1e-3) / 1e12
    out["matmul_c2"] = {"tflops": mm_tf, "ms": ms, "frac_of_burst": mm_tf / peaks["burst"],
                        "frac_of_sustained": mm_tf / peaks["sustained"], "parity": {"max_rel_err": mm_err},
                        "cublas_tflops": cb2_tf, "vs_cublas": mm_tf / cb2_tf, "cublas_what": cb2_what}
    del ad, bd, cd, msets
    torch.cuda.empty_cache()

    c = CONFIG
    g = torch.Generator(device=dev).manual_seed(3)
    X = (torch.randn((c["M"], c["K"]), generator=g, device=dev) * c["x_std"]).bfloat16()
    # the headline's kernel with the fast epilogue (math_mode bounded_fast)
    Wg = (torch.randn((c["K"], c["N"]), generator=g, device=dev) * c["w_std"]).bfloat16()
    Wu = (torch.randn((c["K"], c["N"]), generator=g, device=dev) * c["w_std"]).bfloat16()
    Y = torch.empty((c["M"], c["N"]), dtype=torch.bfloat16, device=dev)
    fsets, _ = input_sets(dev, [X, Wg, Wu, Y], l2)

    def fast(i):
        a_, b_, c_, d_ = fsets[i % len(fsets)]
        llk.fused_swiglu(a_, b_, c_, out=d_, math_mode="bounded_fast")

    def strict(i):
        a_, b_, c_, d_ = fsets[i % len(fsets)]
        llk.fused_swiglu(a_, b_, c_, out=d_)

    # the headline kernel again with this function's step count, so that it
    # and cuBLAS below run timed regions of the same length (same clock regime)
    for i in range(3):
        strict(i)
    sms = time_back_to_back(strict, steps, stream) / steps
    strict_tf = 4.0 * c["M"] * c["N"] * c["K"] / (sms * 1e-3) / 1e12
    for i in range(3):
        fast(i)
    fms = time_back_to_back(fast, steps, stream) / steps
    llk.synchronize(dev.index)
    out["c3_bounded_fast"] = {"tflops": 4.0 * c["M"] * c["N"] * c["K"] / (fms * 1e-3) / 1e12, "ms": fms,
                              "what": "config 3 with math_mode bounded_fast (__expf / __fdividef epilogue); the "
                                      "headline runs the strict epilogue (expf, IEEE division)"}
    del fsets, Wg, Wu, Y
    W = (torch.randn((c["K"], 2 * c["N"]), generator=g, device=dev) * c["w_std"]).bfloat16()
    cb3_ms = cublas_ms(X, W, None)
    cb3_tf = 4.0 * c["M"] * c["N"] * c["K"] / (cb3_ms * 1e-3) / 1e12
    out["cublas_c3"] = {"tflops": cb3_tf, "ms": cb3_ms, "ours_tflops": strict_tf, "headline_tflops": headline_tflops,
                        "vs_cublas": strict_tf / cb3_tf, "steps": steps,
                        "what": "torch.mm X[2048,4096] x [Wg|Wu][4096,22016] bf16 -> bf16 (same FLOPs, no SiLU "
                                "epilogue) against the headline kernel (strict epilogue), both timed right here "
                                "with the same rotation and the same number of back-to-back steps"}
    del X, W
    torch.cuda.empty_cache()
    out.update(rope_attention_extras(args, dev, stream, peaks))
    return out


def rope_attention_extras(args, dev, stream, peaks):
    """The reference's other two LLK ops at Llama-7B attention shapes (32
    heads of 128, f32 as the ops are): RoPE over [1, 32, 4096, 128]
    (HBM-bound: read x, write y) and causal attention over [1, 32, 2048, 128]
    (FLOP-bound on the CUDA cores: the op is f32).  Same rotation / timing
    rules as the headline; parity at sampled rows against the CPU oracle."""
    import torch

    import dslcompiler_b200 as llk
    import oracle

    out = {}
    steps = max(5, min(args.steps, 100))
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    g = torch.Generator(device=dev).manual_seed(9)
    B, H, L, D = 1, 32, 4096, 128
    x = torch.randn((B, H, L, D), generator=g, device=dev)
    pos = torch.arange(L, device=dev, dtype=torch.int64)
    y = torch.empty_like(x)
    sets, _ = input_sets(dev, [x, y], l2)

    def rope_step(i):
        a, b_ = sets[i % len(sets)]
        llk.rope(a, pos, out=b_)

    for i in range(3):
        rope_step(i)
    ms_eager = time_back_to_back(rope_step, steps, stream) / steps
    # the same launches replayed from one CUDA graph: the GPU time without
    # the host's per-call cost (about the kernel time at this size)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side, capture_error_mode="thread_local"):
            for i in range(steps):
                rope_step(i)
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    ms = time_back_to_back(lambda i: graph.replay(), 3, stream) / (3 * steps)
    del graph
    byts = 2 * x.numel() * 4 + L * 8
    hs = [0, 17, 31]
    ref = oracle.rope_f32(x[:, hs].cpu().numpy(), pos.cpu().numpy(), 10000.0)
    err = float(np.abs(sets[0][1][:, hs].cpu().numpy() - ref).max() / np.abs(ref).max())
    out["rope"] = {"shape": [B, H, L, D], "us": ms * 1e3, "us_eager": ms_eager * 1e3,
                   "timing": "us: back-to-back calls replayed from one CUDA graph; us_eager: issued from Python",
                   "GB/s": byts / (ms * 1e-3) / 1e9,
                   "frac_of_hbm": byts / (ms * 1e-3) / 1e9 / peaks["hbm"], "parity": {"max_rel_err": err},
                   "what": "llk_rope, f32 [1,32,4096,128], positions 0..4095, theta 1e4, strict cos/sin"}
    del sets, x, y
    Lq = 2048
    q = torch.randn((B, H, Lq, D), generator=g, device=dev)
    k = torch.randn((B, H, Lq, D), generator=g, device=dev)
    v = torch.randn((B, H, Lq, D), generator=g, device=dev)
    o = torch.zeros_like(q)
    asteps = max(3, min(args.steps, 10))

    def attn_step(i):
        llk.attention(q, k, v, causal=True, out=o)

    attn_step(0)
    ams = time_back_to_back(attn_step, asteps, stream) / asteps
    flops = 4.0 * B * H * Lq * Lq * D / 2  # causal: half the score matrix
    o.zero_()
    attn_step(0)
    torch.cuda.synchronize()
    hs = [0, 31]
    ref = oracle.attention_f32(q[:, hs].cpu().numpy(), k[:, hs].cpu().numpy(), v[:, hs].cpu().numpy(),
                               1.0 / np.sqrt(D), True)
    err = float(np.abs(o[:, hs].cpu().numpy() - ref).max() / np.abs(ref).max())
    sm_clock_ghz = 1.965
    f32_peak = 148 * 128 * 2 * sm_clock_ghz * 1e9 / 1e12
    out["attention"] = {"shape": [B, H, Lq, Lq, D], "causal": True, "ms": ams,
                        "tflops": flops / (ams * 1e-3) / 1e12,
                        "frac_of_f32_fma_peak": flops / (ams * 1e-3) / 1e12 / f32_peak,
                        "f32_fma_peak_tflops": f32_peak, "parity": {"max_rel_err": err},
                        "what": "llk_attention f32 on the CUDA cores; peak = 148 SMs x 128 FMA lanes x 2 x 1.965 GHz "
                                "(nominal, not measured)"}
    llk.synchronize(dev.index)
    del q, k, v, o
    torch.cuda.empty_cache()
    return out


def device_normal_bf16(shape, std, seed, dev):
    """Seeded N(0, std) bf16 tensor drawn on the device (torch's Philox
    generator): the multi-GB secondary configurations would take minutes to
    draw on the host."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * std).to(torch.bfloat16)


def sharded_extras(args, dev, stream, rank, world, peaks, barrier, max_over_ranks):
    """Secondary configurations at every GPU count, column-sharded like the
    headline (rank r computes its llk_shard_columns share, no collective):
    config 5 (Llama-70B prefill SwiGLU, 7.7 TFLOP) and the config-4 decode
    shapes.  Whole-job figures from the max over ranks of back-to-back
    CUDA-event time, inputs rotating over sets larger than 2x L2.  Every
    rank checks its shard against the FP64 oracle at sampled points."""
    import torch

    import dslcompiler_b200 as llk
    from dslcompiler_b200 import datagen as dg

    out = {}
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size

    def graph_ms(fn, steps):
        """Per-launch time of `steps` back-to-back launches replayed from
        one CUDA graph (captured on a side stream, replayed on `stream`):
        the launches without the host's per-call cost, as a decode loop
        runs them."""
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side, capture_error_mode="thread_local"):
                for i in range(steps):
                    fn(i)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        barrier()
        ms = time_back_to_back(lambda i: g.replay(), 3, stream) / (3 * steps)
        del g
        return ms

    def run(cfg, steps, seed, graph=False, y_f32=False):
        c = dg.CONFIGS[cfg]
        M, K, N = c["M"], c["K"], c["N"]
        b, e = llk.shard_columns(N, world, rank)
        xd = device_normal_bf16((M, K), c["x_std"], seed, dev)
        gd = device_normal_bf16((K, e - b), c["w_std"], seed * 1000 + 2 * rank + 1, dev)
        ud = device_normal_bf16((K, e - b), c["w_std"], seed * 1000 + 2 * rank + 2, dev)
        yd = torch.empty((M, e - b), dtype=torch.float32 if y_f32 else torch.bfloat16, device=dev)
        sets, _ = input_sets(dev, [xd, gd, ud, yd], l2)
        out_dtype = "f32" if y_f32 else "bf16"

        def fn(i):
            a_, b_, c_, d_ = sets[i % len(sets)]
            llk.fused_swiglu(a_, b_, c_, out=d_, out_dtype=out_dtype)

        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(time_back_to_back(fn, steps, stream)) / steps
        gms = max_over_ranks(graph_ms(fn, steps)) if graph else None
        torch.cuda.synchronize()
        llk.synchronize(dev.index)
        rows, cols = parity_points(M, e - b, seed=seed + 17 * rank, n_random=1024)
        err = max_over_ranks(points_rel_err(xd, gd, ud, sets[0][3], rows, cols))
        del sets, xd, gd, ud, yd
        torch.cuda.empty_cache()
        return M, K, N, e - b, ms, gms, {"max_rel_err": err, "points_per_rank": int(rows.size)}

    dec = {}
    for i, (cfg, y_f32) in enumerate((("c4_m1", False), ("c4_m4", False), ("c4_m16", False), ("c4_m1", True))):
        M, K, N, n_r, ms_eager, ms, par = run(cfg, max(5, min(args.steps, 200)), 41 + i, graph=True, y_f32=y_f32)
        byts = 2 * M * K + 4 * K * N + (4 if y_f32 else 2) * M * N
        if y_f32:
            par["tol"] = 2e-3  # FP32 Y
        dec[cfg + ("_f32" if y_f32 else "")] = {"us": ms * 1e3, "GB/s": byts / (ms * 1e-3) / 1e9,
                    "frac_of_hbm_per_gpu": byts / (ms * 1e-3) / 1e9 / world / peaks["hbm"],
                    "shard_cols_rank0": n_r, "tflops": 4.0 * M * N * K / (ms * 1e-3) / 1e12, "parity": par,
                    "us_eager": ms_eager * 1e3,
                    "timing": "us: back-to-back launches replayed from one CUDA graph (inputs rotating over sets "
                              "> 2x L2), max over ranks; us_eager: the same launches issued one by one from Python "
                              "(includes the host's ~13 us per call)", "y": "f32" if y_f32 else "bf16"}
    out["decode_c4"] = dec
    # config 5 after the decode shapes: its seconds at the power cap lower the
    # SM clock for a few seconds afterwards, which slows the decode kernel.
    M, K, N, n_r, ms, _, par = run("c5", max(5, min(args.steps, 40)), 55)
    tf = 4.0 * M * N * K / (ms * 1e-3) / 1e12
    out["swiglu_c5"] = {"workload": "c5 llama70b-prefill swiglu X[8192,8192] W[8192,28672] bf16",
                        "tflops": tf, "ms": ms, "frac_of_sustained_per_gpu": tf / world / peaks["sustained"],
                        "frac_of_burst_per_gpu": tf / world / peaks["burst"], "shard_cols_rank0": n_r,
                        "parity": par,
                        "data": "synthetic, drawn on the device (torch Philox, seeded), X~N(0,1), W~N(0,0.015)"}
    return out


def profile_case(args):
    """Runs one configuration's kernel a few times on cuda:0 with per-launch
    CUDA-event times, for ncu captures and quick timing.  Inputs are seeded
    random tensors of the configuration's shapes, drawn on the device;
    --shape M,K,N runs a SwiGLU of that shape instead (e.g. a column shard)."""
    import torch

    import dslcompiler_b200 as llk
    from dslcompiler_b200 import datagen as dg

    if args.profile_case == "attention":
        # --shape B,H,L,D: causal self-attention, f32 (the Llama-7B attention
        # shape is 1,32,2048,128)
        B_, H_, L_, D_ = (int(v) for v in (args.shape or "1,32,2048,128").split(","))
        g = torch.Generator(device="cuda").manual_seed(42)
        q, k, v = (torch.randn((B_, H_, L_, D_), generator=g, device="cuda") for _ in range(3))
        o = torch.zeros_like(q)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        times = []
        for _ in range(args.launches):
            s.record()
            llk.attention(q, k, v, scale=D_ ** -0.5, causal=True, out=o)
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        llk.synchronize(0)
        print(f"attention B={B_} H={H_} L={L_} D={D_}: {args.launches} launches, ms per launch "
              f"{[round(t, 4) for t in times]}", file=sys.stderr)
        return 0
    if args.profile_case == "shape":
        M_, K_, N_ = (int(v) for v in args.shape.split(","))
        c = dict(kind="swiglu", M=M_, K=K_, N=N_, x_std=1.0, w_std=0.02, y="bf16")
    else:
        c = dg.CONFIGS[args.profile_case]
    g = torch.Generator(device="cuda").manual_seed(42)
    M, K, N = c["M"], c["K"], c["N"]
    if c["kind"] == "matmul":
        A = (torch.rand((M, K), generator=g, device="cuda") * 2 - 1).bfloat16()
        B = (torch.rand((K, N), generator=g, device="cuda") * 2 - 1).bfloat16()
        C = torch.empty((M, N), dtype=torch.float32, device="cuda")
        run = lambda: llk.matmul(A, B, C, variant=args.variant)  # noqa: E731
    else:
        X = (torch.randn((M, K), generator=g, device="cuda") * c["x_std"]).bfloat16()
        Wg = (torch.randn((K, N), generator=g, device="cuda") * c["w_std"]).bfloat16()
        Wu = (torch.randn((K, N), generator=g, device="cuda") * c["w_std"]).bfloat16()
        Y = torch.empty((M, N), dtype=torch.float32 if c["y"] == "f32" else torch.bfloat16, device="cuda")
        run = lambda: llk.fused_swiglu(X, Wg, Wu, out=Y, out_dtype=c["y"], variant=args.variant)  # noqa: E731
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(args.launches):
        s.record()
        run()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    llk.synchronize(0)
    print(f"{args.profile_case} M={M} K={K} N={N}: {args.launches} launches, ms per launch "
          f"{[round(t, 4) for t in times]}", file=sys.stderr)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--quick", action="store_true", help="skip the single-GPU extras and the CPU baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-case", default=None, metavar="CFG",
                    help="run one configuration's kernel --launches times on cuda:0 (for ncu) and exit; CFG is a "
                         "config name (c1 .. c5, c4_m1 ..), 'shape' with --shape M,K,N, or 'attention' with "
                         "--shape B,H,L,D (causal f32 attention)")
    ap.add_argument("--shape", default=None)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--variant", default="auto")
    args = ap.parse_args(argv)
    if args.profile_case:
        return profile_case(args)
    if args.warmup < 3:
        args.warmup = 3
    rank, _, world = dist_env()
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        return reference_arm(args)
    return our_arm(args)


if __name__ == "__main__":
    sys.exit(main())
