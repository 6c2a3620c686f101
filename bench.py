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
import threading
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
    """(bf16 TFLOP/s, HBM GB/s, source).  The bf16 figure is the SUSTAINED
    one: the timed loop runs back to back for a sizeable fraction of a
    second, long enough for the 1 kW power cap to set the clock, which is the
    regime of the seconds-long cuBLAS loop the sustained figure measures."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops_sustained") or d.get("bf16_tflops"), d.get("hbm_gbs"), "measured"
    return 1400.0, 6650.0, "fallback"


def profile_traffic(name):
    """dram bytes per launch recorded from an ncu capture in profiles/<name>.md
    (a line 'traffic_bytes_per_launch: <int>')."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(p):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            f = [s.strip() for s in line.split(",")]
            if len(f) == 9:
                self.rows.append(f)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = [r for r in self.rows if r[0].isdigit() and int(r[0]) in self.gpus]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        pw = [float(r[3]) for r in rows if re.match(r"^[0-9.]+$", r[3])]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(pw) if pw else None}


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
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean * 1e3 * M / rows,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded splitmix64/Box-Muller, X~N(0,1), W~N(0,0.02), bf16)",
            "config": {"workload": "c3 llama7b-prefill swiglu", "M": M, "K": K, "N": N, "sample_rows": rows},
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

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    # ---------------------------------------------------------- value
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    llk.synchronize(local)
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(range(world)) if local == 0 else None
    if sampler:
        sampler.__enter__()
    t_wall0 = time.perf_counter()
    kernel_ms = time_back_to_back(step, args.steps, stream)
    t_wall = time.perf_counter() - t_wall0
    barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__()
    llk.synchronize(local)
    job_ms = max_over_ranks(kernel_ms) / args.steps
    total_flops = 4.0 * M * N * K
    value = total_flops / (job_ms * 1e-3) / 1e12

    # ------------------------------------------------------- roofline
    peak_tf, peak_gbs, peak_src = measured_peaks()
    my_ms = kernel_ms / args.steps
    achieved = 4.0 * M * n_r * K / (my_ms * 1e-3) / 1e12
    traffic = profile_traffic("tc2_swiglu_c3") if world == 1 else None

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
        extras["gather_y"] = secondary(lambda: gather_timing(args, dev, stream, yd, N, world, barrier, max_over_ranks))
        if "error" not in extras["gather_y"]:
            extras["fused_allgather"] = secondary(lambda: fused_allgather_timing(
                args, dev, stream, xd, gd, ud, N, barrier, max_over_ranks, job_ms, extras["gather_y"]["ms"]))
    cpu = None
    if not args.quick:
        del sets, xd, gd, ud, yd
        torch.cuda.empty_cache()
        extras.update(secondary(lambda: sharded_extras(args, dev, stream, rank, world, peak_tf, peak_gbs, barrier,
                                                       max_over_ranks), "sharded_extras"))
        if world == 1:
            extras.update(secondary(lambda: single_gpu_extras(args, dev, stream, peak_tf, peak_gbs),
                                    "single_gpu_extras"))
            if not args.no_cpu_baseline:
                cpu = cpu_baseline(x, wg, wu)
                naive = secondary(reference_naive_baseline)
                if naive:
                    cpu["reference_naive"] = naive

    clocks = sampler.summary() if sampler else None
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
                         "frac": achieved / peak_tf, "traffic": traffic,
                         "peak_source": f"{peak_src} bf16 sustained (MEASURED_PEAKS.json bf16_tflops_sustained): "
                                        "the timed loop is back to back and power-capped",
                         "kernel": "tc2_kernel<TC_SWIGLU_BF16> (CTA pairs)" if M > 128 else "tc_swiglu_kernel<TC_SWIGLU_BF16>",
                         "algorithmic_work": "4*M*N_rank*K FLOP per launch"},
            "e2e": e2e, "e2e_packed_weights": e2e_packed,
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
    return 0


def gather_timing(args, dev, stream, yd, N, world, barrier, max_over_ranks):
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
    return {"ms": ms, "bytes_received_per_gpu": recv, "GB/s_per_gpu": recv / (ms * 1e-3) / 1e9,
            "what": "all_gather_into_tensor (NCCL) of padded Y shards + llk_gather_columns relayout"}


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


def fused_allgather_timing(args, dev, stream, xd, gd, ud, N, barrier, max_over_ranks, kernel_ms, gather_ms):
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
    layer.close()
    flops = 4.0 * M * N * K
    return {"ms": ms, "tflops_whole_job": flops / (ms * 1e-3) / 1e12,
            "kernel_plus_nccl_gather_ms": kernel_ms + gather_ms,
            "tflops_kernel_plus_nccl_gather": flops / ((kernel_ms + gather_ms) * 1e-3) / 1e12,
            "what": "llk_swiglu_column_parallel: full Y on every GPU, shards stored to peers by the kernel epilogue"}


def single_gpu_extras(args, dev, stream, peak_tf, peak_gbs):
    """Secondary measurement on one GPU: the micro.mma matmul (config 2),
    same timing rules."""
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
    out["matmul_c2"] = {"tflops": 2.0 * 4096 ** 3 / (ms * 1e-3) / 1e12, "ms": ms,
                        "frac_of_peak": 2.0 * 4096 ** 3 / (ms * 1e-3) / 1e12 / peak_tf}
    del ad, bd, cd, msets
    torch.cuda.synchronize()
    llk.synchronize(dev.index)
    return out


def device_normal_bf16(shape, std, seed, dev):
    """Seeded N(0, std) bf16 tensor drawn on the device (torch's Philox
    generator): the multi-GB secondary configurations would take minutes to
    draw on the host."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * std).to(torch.bfloat16)


def sharded_extras(args, dev, stream, rank, world, peak_tf, peak_gbs, barrier, max_over_ranks):
    """Secondary configurations at every GPU count, column-sharded like the
    headline (rank r computes its llk_shard_columns share, no collective):
    config 5 (Llama-70B prefill SwiGLU, 7.7 TFLOP) and the config-4 decode
    shapes.  Whole-job figures from the max over ranks of back-to-back
    CUDA-event time, inputs rotating over sets larger than 2x L2."""
    import torch

    import dslcompiler_b200 as llk
    from dslcompiler_b200 import datagen as dg

    out = {}
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size

    def run(cfg, steps, seed):
        c = dg.CONFIGS[cfg]
        M, K, N = c["M"], c["K"], c["N"]
        b, e = llk.shard_columns(N, world, rank)
        xd = device_normal_bf16((M, K), c["x_std"], seed, dev)
        gd = device_normal_bf16((K, e - b), c["w_std"], seed * 1000 + 2 * rank + 1, dev)
        ud = device_normal_bf16((K, e - b), c["w_std"], seed * 1000 + 2 * rank + 2, dev)
        yd = torch.empty((M, e - b), dtype=torch.bfloat16, device=dev)
        sets, _ = input_sets(dev, [xd, gd, ud, yd], l2)

        def fn(i):
            a_, b_, c_, d_ = sets[i % len(sets)]
            llk.fused_swiglu(a_, b_, c_, out=d_)

        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(time_back_to_back(fn, steps, stream)) / steps
        llk.synchronize(dev.index)
        del sets, xd, gd, ud, yd
        torch.cuda.empty_cache()
        return M, K, N, ms

    dec = {}
    for i, cfg in enumerate(("c4_m1", "c4_m4", "c4_m16")):
        M, K, N, ms = run(cfg, max(5, min(args.steps, 200)), 41 + i)
        byts = 2 * M * K + 4 * K * N + 2 * M * N
        dec[cfg] = {"us": ms * 1e3, "GB/s": byts / (ms * 1e-3) / 1e9,
                    "frac_of_hbm_per_gpu": byts / (ms * 1e-3) / 1e9 / world / peak_gbs,
                    "tflops": 4.0 * M * N * K / (ms * 1e-3) / 1e12}
    out["decode_c4"] = dec
    # config 5 after the decode shapes: its seconds at the power cap lower the
    # SM clock for a few seconds afterwards, which slows the decode kernel.
    M, K, N, ms = run("c5", max(5, min(args.steps, 40)), 55)
    tf = 4.0 * M * N * K / (ms * 1e-3) / 1e12
    out["swiglu_c5"] = {"workload": "c5 llama70b-prefill swiglu X[8192,8192] W[8192,28672] bf16",
                        "tflops": tf, "ms": ms, "frac_of_peak_per_gpu": tf / world / peak_tf,
                        "data": "synthetic, drawn on the device (torch Philox, seeded), X~N(0,1), W~N(0,0.015)"}
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--quick", action="store_true", help="skip the single-GPU extras and the CPU baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
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
