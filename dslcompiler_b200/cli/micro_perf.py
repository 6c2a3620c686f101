"""micro-perf: L0 static bound of a micro.kernel on a MachineModel
(``--machine``, ``--level``, ``--format``, positional input; the CLI of the
reference's simulator spec, section 10).  Only level 0 is implemented."""
from __future__ import annotations

import argparse
import os
import sys

from .. import microperf

DEFAULT_MACHINE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "machines",
                               "b200-sm100a.yaml")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="micro-perf")
    ap.add_argument("input")
    ap.add_argument("--machine", default=DEFAULT_MACHINE)
    ap.add_argument("--level", type=int, default=0, choices=[0])
    ap.add_argument("--format", choices=["yaml", "text"], default="yaml")
    a = ap.parse_args(argv)
    try:
        machine = microperf.load_machine(a.machine)
    except microperf.MachineModelError as e:
        print(f"error: {a.machine}: {e}", file=sys.stderr)
        return 1
    rep = microperf.l0_bound(open(a.input).read(), machine)
    if a.format == "yaml":
        sys.stdout.write(microperf.report_yaml(rep, machine))
    else:
        ns = rep.predicted_cycles / machine.clock_hz * 1e9
        print(f"{rep.kernel}: {rep.predicted_cycles:.0f} cycles ({ns / 1e3:.1f} us at {machine.clock_hz / 1e6:.0f} MHz), "
              f"bottleneck {rep.bottleneck}, {rep.total_flops:.3e} FLOP")
    return 0


if __name__ == "__main__":
    sys.exit(main())
