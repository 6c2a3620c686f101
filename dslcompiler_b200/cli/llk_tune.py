"""llk-tune for the B200 target.

Flags of ``tools/llk-tune/llk-tune.cpp:21-32`` (--M --N --K -o --dry-run) and
its output: the top-3 configurations as schedule-DB entries.  Where the
reference writes its candidates unmeasured (llk-tune.cpp:226-232), this one
measures every sm_100a candidate on the GPU (CUDA events, L2 evicted before
each launch, median of --iters) and records measured_gflops.

Candidates: the legal launch plans of the op's ``micro.search_space``
(``dslcompiler_b200.micro``: CTA pairs or single CTAs, the tail split of
the leftover tiles along N or K, static or dynamic schedule, persistent grid
sizes; for small-M SwiGLU the decode kernel's stages, grid and cluster
split), or of a stored space given with ``--search-space FILE`` (the output
of ``llk-compile --emit micro-search-space``).
--install merges the results into a schedule DB file.
"""
from __future__ import annotations

import argparse
import statistics
import sys

from .. import micro, schedule


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="llk-tune")
    ap.add_argument("--M", type=int, default=128)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("-o", dest="output", default="tune_result.json")
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--op", choices=["swiglu", "matmul"], default="swiglu")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--install", default=None, help="merge the top entries into this schedule DB")
    ap.add_argument("--search-space", default=None, help="micro.search_space file to draw the candidates from")
    a = ap.parse_args(argv)
    M, N, K = a.M, a.N, a.K
    from .. import capi
    from ..swiglu import KernelKey

    opname = "fused_swiglu" if a.op == "swiglu" else "matmul"
    opcode = schedule.OPS[opname]
    out_t = capi.LLK_DTYPE_BF16 if a.op == "swiglu" else capi.LLK_DTYPE_FP32
    bucket = schedule.classify_m(M)
    key_tc = KernelKey(operation=opcode, output_type=out_t, M_bucket=bucket, N=N, K=K, thread_count=capi.VARIANTS["tc"])
    key_dec = KernelKey(operation=opcode, output_type=out_t, M_bucket=bucket, N=N, K=K,
                        thread_count=capi.VARIANTS["decode"]) if (a.op == "swiglu" and M <= 128) else None
    base_tc = key_tc.plan(M)
    base_dec = key_dec.plan(M) if key_dec else None
    if a.search_space:
        space = micro.parse_search_space(open(a.search_space).read())
        if (space.M, space.N, space.K) != (M, N, K) or space.workload != opname:
            print(f"error: {a.search_space} is the space of {space.workload} M={space.M} N={space.N} K={space.K}",
                  file=sys.stderr)
            return 1
    else:
        space = micro.search_space(opname, M, N, K)
    cands = micro.candidates(space)
    if key_dec is None:
        cands = [c for c in cands if c["variant"] != capi.VARIANTS["decode"]]
    print(f"M={M} (bucket {bucket}) N={N} K={K}")
    print(f"Generated {len(cands)} candidate configs (sm_100a launch plans)")
    results = []
    if a.dry_run:
        print("\nTop candidate configs (unmeasured):")
        for i, c in enumerate(cands[:5]):
            print(f"  [{i}] {c}")
        results = [(0.0, c) for c in cands]
    else:
        import torch

        import dslcompiler_b200 as llk

        g = torch.Generator(device="cuda").manual_seed(1)
        X = torch.randn((M, K), generator=g, device="cuda").bfloat16()
        Wg = (torch.randn((K, N), generator=g, device="cuda") * 0.02).bfloat16()
        Wu = (torch.randn((K, N), generator=g, device="cuda") * 0.02).bfloat16()
        Y = torch.empty((M, N), dtype=torch.bfloat16 if a.op == "swiglu" else torch.float32, device="cuda")
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda").view(torch.float32)
        flop = (4.0 if a.op == "swiglu" else 2.0) * M * N * K
        for c in cands:
            v = "decode" if c["variant"] == capi.VARIANTS["decode"] else "tc"
            key = key_dec if v == "decode" else key_tc
            key.insert_plan(**c)
            fn = (lambda: llk.fused_swiglu(X, Wg, Wu, out=Y, variant=v)) if a.op == "swiglu" else \
                (lambda: llk.matmul(X, Wg, Y, variant="tc"))
            for _ in range(3):
                fn()
            ts = []
            for _ in range(a.iters):
                flush.sum()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                fn()
                e.record()
                e.synchronize()
                ts.append(s.elapsed_time(e))
            gf = flop / (statistics.median(ts) * 1e-3) / 1e9
            results.append((gf, c))
        key_tc.insert_plan(**base_tc)
        if key_dec:
            key_dec.insert_plan(**base_dec)
        llk.synchronize(0)
    results.sort(key=lambda r: -r[0])
    entries = []
    for gf, c in results[:3]:
        sched = {f: c[f] for f in schedule.PLAN_FIELDS if f != "variant"}
        sched["variant"] = schedule.VARIANT_NAMES[c["variant"]]
        entries.append(schedule.ScheduleEntry(opname, schedule.TARGET, bucket, N, K,
                                              "bf16" if a.op == "swiglu" else "f32", "strict", sched,
                                              round(gf, 1) if not a.dry_run else 0.0))
    schedule.write_db(entries, a.output, merge=False)
    print(f"Wrote top-{len(entries)} configs to {a.output}")
    for gf, c in results[:3]:
        print(f"  {gf:.1f} GFLOPS  {c}")
    if a.install:
        schedule.write_db(entries[:1], a.install, merge=True)
        print(f"Installed the best config into {a.install}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
