"""llk-compile for the B200 target.

Same interface as ``tools/llk-compile/llk-compile.cpp:76-82,209-319``: a
positional input .mlir and ``--M/--N/--K`` for dynamic dimensions; prints
"Compilation successful" and exits 0, or reports "Failed to parse <file>" /
"Compilation pipeline failed" and exits 1.  Instead of JIT-compiling CPU code
it verifies the op, lowers it to the micro.kernel that dispatches to the
sm_100a kernel (``--emit=micro`` prints it; ``dslcompiler_b200.micro.run_micro``
runs it) and resolves the launch plan (the "object code" of this backend).
``--emit=micro-search-space`` prints the ``micro.search_space`` of legal
launch-plan choices for each op instead (the spec's
``--llk-to-micro-search-space``), which ``llk-tune --search-space`` reads.
"""
from __future__ import annotations

import argparse
import json
import sys

from .. import compiler, micro, schedule


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="llk-compile", description="LLK compiler (B200 backend)")
    ap.add_argument("input")
    ap.add_argument("--M", type=int, default=0)
    ap.add_argument("--N", type=int, default=0)
    ap.add_argument("--K", type=int, default=0)
    ap.add_argument("--emit", choices=["none", "micro", "plan", "micro-search-space"], default="none")
    ap.add_argument("--variant", choices=["auto", "tc", "decode"], default="auto")
    ap.add_argument("--schedule-db", default=None, help="install B200 schedules from this DB first")
    ap.add_argument("-o", "--output", default=None, help="write the emitted text here")
    a = ap.parse_args(argv)
    try:
        text = open(a.input).read()
    except OSError:
        print(f"Failed to parse {a.input}", file=sys.stderr)
        return 1
    ops = compiler.parse_llk(text)
    if not ops:
        print(f"Failed to parse {a.input}", file=sys.stderr)
        return 1
    if a.schedule_db:
        schedule.install(a.schedule_db)
    out = []
    try:
        for op in ops:
            compiler.verify(op)
            M, N, K = compiler.resolve_shape(op, a.M, a.N, a.K)
            if a.emit == "micro-search-space":
                out.append(micro.emit_search_space(micro.search_space(op.op, M, N, K)))
                continue
            low = compiler.lower_to_micro(op, M, N, K, a.variant)
            if a.emit == "micro":
                out.append(low.text)
            elif a.emit == "plan":
                out.append(json.dumps({"kernel": low.name, "plan": low.plan}))
    except compiler.VerifyError as e:
        print(f"error: 'llk.{ops[0].op}' op {e}", file=sys.stderr)
        print("Compilation pipeline failed", file=sys.stderr)
        return 1
    if out:
        if a.output:
            with open(a.output, "w") as f:
                f.write("\n".join(out))
        else:
            print("\n".join(out))
    print("Compilation successful")
    return 0


if __name__ == "__main__":
    sys.exit(main())
