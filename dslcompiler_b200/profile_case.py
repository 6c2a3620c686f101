"""Runs one benchmark configuration's kernel a few times on cuda:0, for
profiling (ncu) and quick timing.  Inputs are seeded random tensors of the
configuration's shapes drawn on the device.

    python -m dslcompiler_b200.profile_case c3 [--launches 3] [--variant auto]
"""
from __future__ import annotations

import argparse
import sys

import torch

import dslcompiler_b200 as llk
from dslcompiler_b200 import datagen as dg


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("config", choices=sorted(dg.CONFIGS) + ["shape"])
    ap.add_argument("--shape", default=None, help="M,K,N for config 'shape' (SwiGLU, bf16 Y)")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--variant", default="auto")
    a = ap.parse_args(argv)
    if a.config == "shape":
        M_, K_, N_ = (int(v) for v in a.shape.split(","))
        c = dict(kind="swiglu", M=M_, K=K_, N=N_, x_std=1.0, w_std=0.02, y="bf16")
    else:
        c = dg.CONFIGS[a.config]
    g = torch.Generator(device="cuda").manual_seed(42)
    M, K, N = c["M"], c["K"], c["N"]
    if c["kind"] == "matmul":
        A = (torch.rand((M, K), generator=g, device="cuda") * 2 - 1).bfloat16()
        B = (torch.rand((K, N), generator=g, device="cuda") * 2 - 1).bfloat16()
        C = torch.empty((M, N), dtype=torch.float32, device="cuda")
        run = lambda: llk.matmul(A, B, C, variant=a.variant)  # noqa: E731
    else:
        X = (torch.randn((M, K), generator=g, device="cuda") * c["x_std"]).bfloat16()
        Wg = (torch.randn((K, N), generator=g, device="cuda") * c["w_std"]).bfloat16()
        Wu = (torch.randn((K, N), generator=g, device="cuda") * c["w_std"]).bfloat16()
        Y = torch.empty((M, N), dtype=torch.float32 if c["y"] == "f32" else torch.bfloat16, device="cuda")
        run = lambda: llk.fused_swiglu(X, Wg, Wu, out=Y, out_dtype=c["y"], variant=a.variant)  # noqa: E731
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(a.launches):
        s.record()
        run()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    llk.synchronize(0)
    print(f"{a.config}: {a.launches} launches, ms per launch {[round(t, 4) for t in times]}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
