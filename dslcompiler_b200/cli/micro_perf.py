"""micro-perf: L0 static bound of a micro.kernel on a MachineModel
(``--machine``, ``--level``, ``--format``, positional input; the CLI of the
reference's simulator spec, section 10).  Only level 0 is implemented."""
from __future__ import annotations

import argparse
import os
import sys

from .. import compiler, microperf

DEFAULT_MACHINE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "machines",
                               "b200-sm100a.yaml")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="micro-perf")
    ap.add_argument("input")
    ap.add_argument("--machine", default=DEFAULT_MACHINE)
    ap.add_argument("--level", type=int, default=0, choices=[0])
    ap.add_argument("--format", choices=["yaml", "text"], default="yaml")
    ap.add_argument("--clock-hz", type=float, default=None,
                    help="predict at this SM clock (e.g. the clock measured under load) instead of the model's")
    ap.add_argument("--measured-us", type=float, default=None,
                    help="a measured kernel time to set against the prediction (adds measured_us and "
                         "efficiency = predicted / measured)")
    a = ap.parse_args(argv)
    try:
        machine = microperf.load_machine(a.machine)
    except microperf.MachineModelError as e:
        print(f"error: {a.machine}: {e}", file=sys.stderr)
        return 1
    if a.clock_hz is not None:
        if a.clock_hz <= 0:
            print("error: --clock-hz must be positive", file=sys.stderr)
            return 1
        # DRAM bandwidth is fixed in bytes per second, not per SM cycle: keep
        # it when the clock changes (on-chip spaces follow the clock).
        if "dram" in machine.memory:
            m = dict(machine.memory["dram"])
            m["bandwidth_bytes_per_cycle"] = float(m["bandwidth_bytes_per_cycle"]) * machine.clock_hz / a.clock_hz
            machine.memory = dict(machine.memory, dram=m)
        machine.clock_hz = a.clock_hz
    text = open(a.input).read()
    errs = compiler.verify_micro(text)
    if errs:
        for e in errs:
            print(f"error: {a.input}: {e}", file=sys.stderr)
        return 1
    rep = microperf.l0_bound(text, machine)
    ns = rep.predicted_cycles / machine.clock_hz * 1e9
    if a.format == "yaml":
        text = microperf.report_yaml(rep, machine)
        if a.measured_us is not None:
            text += f"measured_us: {a.measured_us}\nefficiency: {round(ns / 1e3 / a.measured_us, 3)}\n"
        sys.stdout.write(text)
    else:
        line = (f"{rep.kernel}: {rep.predicted_cycles:.0f} cycles ({ns / 1e3:.1f} us at {machine.clock_hz / 1e6:.0f} MHz), "
                f"bottleneck {rep.bottleneck}, {rep.total_flops:.3e} FLOP")
        if a.measured_us is not None:
            line += f"; measured {a.measured_us:.1f} us, efficiency {ns / 1e3 / a.measured_us:.3f}"
        print(line)
    return 0


if __name__ == "__main__":
    sys.exit(main())
