"""llk-bench for the B200 target.

Flags of ``tools/llk-bench/llk-bench.cpp:21-35`` (--M --N --K --threads
--warmup-ms --measure-ms --reps) with the same method (warm up for
warmup-ms, then `reps` windows of measure-ms, report the best GFLOPS with the
op's FLOP count) and the same two output lines.  Unlike the reference, which
times a stand-in loop (llk-bench.cpp:37-53), this times the real fused SwiGLU
(4MNK FLOP) or matmul (2MNK) kernel on the GPU; each window is timed with CUDA
events.  (The CPU baseline with the same flags and output lines is
``python -m oracle.cpu_bench``, test infrastructure outside this package.)
"""
from __future__ import annotations

import argparse
import json
import sys
import time


def gpu_window(fn, ms_budget):
    import torch

    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    iters, total = 0, 0.0
    t_end = time.perf_counter() + ms_budget / 1e3
    while True:
        s.record()
        fn()
        e.record()
        e.synchronize()
        total += s.elapsed_time(e)
        iters += 1
        if time.perf_counter() >= t_end:
            return total, iters


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="llk-bench")
    ap.add_argument("--M", type=int, default=128)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--threads", type=int, default=8)
    ap.add_argument("--warmup-ms", type=int, default=500)
    ap.add_argument("--measure-ms", type=int, default=2000)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--op", choices=["swiglu", "matmul"], default="swiglu")
    ap.add_argument("--variant", choices=["auto", "tc", "decode", "simt"], default="auto")
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--packed", action="store_true", help="use packed (slab-major) weights")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    M, N, K = a.M, a.N, a.K
    flop = (4.0 if a.op == "swiglu" else 2.0) * M * N * K
    print(f"LLK Bench — M={M} N={N} K={K} threads={a.threads}")

    import torch

    import dslcompiler_b200 as llk

    torch.cuda.set_device(a.device)
    g = torch.Generator(device="cuda").manual_seed(1)
    X = torch.randn((M, K), generator=g, device="cuda").bfloat16()
    Wg = (torch.randn((K, N), generator=g, device="cuda") * 0.02).bfloat16()
    if a.op == "swiglu":
        Wu = (torch.randn((K, N), generator=g, device="cuda") * 0.02).bfloat16()
        Y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        if a.packed:
            pw = llk.PackedWeights(Wg, Wu)
            fn = lambda: pw(X, out=Y, variant=a.variant)  # noqa: E731
        else:
            fn = lambda: llk.fused_swiglu(X, Wg, Wu, out=Y, variant=a.variant)  # noqa: E731
    else:
        C = torch.empty((M, N), dtype=torch.float32, device="cuda")
        fn = lambda: llk.matmul(X, Wg, C, variant=a.variant)  # noqa: E731

    def window(budget):
        return gpu_window(fn, budget)

    window(a.warmup_ms)
    best_gflops, best_ms = 0.0, 0.0
    for _ in range(a.reps):
        total_ms, iters = window(a.measure_ms)
        ms = total_ms / iters
        gf = flop / (ms * 1e-3) / 1e9
        if gf > best_gflops:
            best_gflops, best_ms = gf, ms
    llk.synchronize(a.device)
    print(f"Best: {best_gflops} GFLOPS ({best_ms} ms/iter, {a.reps} reps)")
    if a.json:
        print(json.dumps({"M": M, "N": N, "K": K, "op": a.op, "gflops": best_gflops, "ms": best_ms,
                          "device": "b200"}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
