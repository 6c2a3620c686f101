"""CPU baseline in llk-bench's form: the threaded restatement of the
reference's fused AVX2 schedule (swiglu_port.c) timed with the flags and
output lines of ``tools/llk-bench/llk-bench.cpp:21-35`` -- warm up for
warmup-ms, then `reps` windows of measure-ms, best GFLOPS.

TEST INFRASTRUCTURE: a timed CPU baseline, never the product.

    python -m oracle.cpu_bench --M 8 --N 256 --K 256 --threads 16
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main(argv=None) -> int:
    import oracle
    from dslcompiler_b200 import datagen as dg

    ap = argparse.ArgumentParser(prog="llk-bench (CPU port)")
    ap.add_argument("--M", type=int, default=128)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--threads", type=int, default=8)
    ap.add_argument("--warmup-ms", type=int, default=500)
    ap.add_argument("--measure-ms", type=int, default=2000)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--op", choices=["swiglu", "matmul"], default="swiglu")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    M, N, K = a.M, a.N, a.K
    flop = (4.0 if a.op == "swiglu" else 2.0) * M * N * K
    print(f"LLK Bench — M={M} N={N} K={K} threads={a.threads}")
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0, 0.02, seed=1)
    fn = (lambda: oracle.port_swiglu(x, wg, wu, "bf16", threads=a.threads)) if a.op == "swiglu" else \
        (lambda: oracle.port_matmul(x, wg, threads=a.threads))

    def window(budget_ms):
        t0, it = time.perf_counter(), 0
        while True:
            fn()
            it += 1
            el = (time.perf_counter() - t0) * 1e3
            if el >= budget_ms:
                return el, it

    window(a.warmup_ms)
    best_gflops, best_ms = 0.0, 0.0
    for _ in range(a.reps):
        total_ms, iters = window(a.measure_ms)
        ms = total_ms / iters
        gf = flop / (ms * 1e-3) / 1e9
        if gf > best_gflops:
            best_gflops, best_ms = gf, ms
    print(f"Best: {best_gflops} GFLOPS ({best_ms} ms/iter, {a.reps} reps)")
    if a.json:
        print(json.dumps({"M": M, "N": N, "K": K, "op": a.op, "gflops": best_gflops, "ms": best_ms,
                          "device": "cpu", "threads": a.threads}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
