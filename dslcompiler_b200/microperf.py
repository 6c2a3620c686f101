"""MachineModel loader and the micro-perf L0 static bound.

Follows the reference's micro-IR simulator spec
(``docs/superpowers/specs/2026-08-11-micro-ir-avx2-simulator-implementation-spec.md``):
the MachineModel YAML schema and its validation rules (:81-266), the L0 bound
(:356-425: mma FLOPs times loop trips; copy / store bytes per memory space;
prediction = max(compute, memory) lower bounds) and the ``micro-perf`` report
(:545-602).  The spec's C++ loader is not implemented in the reference; this is
the B200 build's own.

GPU-specific rule: loads that the kernels serve from L2 (the operand tiles
re-read across CTAs) are charged to ``l2``; DRAM is charged the compulsory
bytes of the kernel's arguments (each read or written once) plus explicit
DRAM copies -- the measured behaviour of the sm_100a kernels (ncu: DRAM read
= algorithmic bytes).
"""
from __future__ import annotations

import math
import re
from dataclasses import dataclass, field

import yaml

KNOWN_DTYPES = {"f32": 4, "bf16": 2, "f16": 2, "i8": 1, "f8": 1}
KNOWN_LAYOUTS = {"row_major", "vectorized", "blocked", "swizzled_128b"}


class MachineModelError(ValueError):
    pass


@dataclass
class MachineModel:
    name: str
    clock_hz: float
    owners: dict
    matrix_engines: list
    vector_engines: list
    memory: dict
    dma: dict
    sync: dict
    worker_threads: int

    def engine(self, name_prefix: str) -> dict:
        for e in self.matrix_engines:
            if name_prefix.startswith(e["name"]):
                return e
        raise MachineModelError(f"no matrix engine for {name_prefix!r}")


def load_machine(path: str) -> MachineModel:
    with open(path) as f:
        d = yaml.safe_load(f)
    return validate_machine(d)


def validate_machine(d: dict) -> MachineModel:
    """The spec's rejection rules (:250-266)."""
    if not isinstance(d, dict) or "schema_version" not in d:
        raise MachineModelError("missing schema_version")
    if d["schema_version"] != 1:
        raise MachineModelError(f"unsupported schema version {d['schema_version']}")
    if not d.get("name"):
        raise MachineModelError("empty name")
    if not d.get("clock_hz") or d["clock_hz"] <= 0:
        raise MachineModelError("zero clock")
    comp = d.get("compute", {})
    owners = comp.get("owners", {})
    for n, o in owners.items():
        if int(o.get("count", 0)) <= 0:
            raise MachineModelError(f"zero engine count for owner {n}")
    mes = comp.get("matrix_engines", [])
    for e in mes:
        if int(e.get("count", 0)) <= 0:
            raise MachineModelError(f"zero engine count for {e.get('name')}")
        for s in e.get("tile_shapes", []):
            if len(s) != 3:
                raise MachineModelError("matrix tile shapes must have length 3")
        for dt in e.get("input_dtypes", []) + e.get("accumulator_dtypes", []):
            if dt not in KNOWN_DTYPES:
                raise MachineModelError(f"unknown dtype {dt}")
    ves = comp.get("vector_engines", [])
    for e in ves:
        if int(e.get("count", 0)) <= 0:
            raise MachineModelError(f"zero engine count for {e.get('name')}")
        for lay in e.get("supported_layouts", []):
            if lay not in KNOWN_LAYOUTS:
                raise MachineModelError(f"unsupported layout {lay}")
        for dt in e.get("lanes", {}):
            if dt not in KNOWN_DTYPES:
                raise MachineModelError(f"unknown dtype {dt}")
    mem = d.get("memory", {})
    for n, m in mem.items():
        if float(m.get("bandwidth_bytes_per_cycle", 0)) <= 0:
            raise MachineModelError(f"non-positive bandwidth for {n}")
        if int(m.get("capacity_bytes", 0)) <= 0:
            raise MachineModelError(f"zero capacity for {n}")
        for lay in m.get("supported_layouts", []):
            if lay not in KNOWN_LAYOUTS:
                raise MachineModelError(f"unsupported layout {lay}")
    for req in ("dram", "sram", "acc"):
        if req not in mem:
            raise MachineModelError(f"missing memory space {req}")
    return MachineModel(d["name"], float(d["clock_hz"]), owners, mes, ves, mem, d.get("dma", {}), d.get("sync", {}),
                        int(comp.get("worker_threads", {}).get("count", 1)))


# ------------------------------------------------------------------ micro IR
_LOOP_RE = re.compile(r"micro\.(?:spatial_for|for)\s+%\w+\s*=\s*(\d+)\s+to\s+(\d+)\s+step\s+(\d+)")
_MMA_RE = re.compile(r"micro\.mma\b.*?shape\s*=\s*\[(\d+),\s*(\d+),\s*(\d+)\].*?engine\s*=\s*\"([^\"]+)\"")
_COPY_RE = re.compile(r"micro\.(?:async_copy|tile_async_copy|load|tile_load)\b.*?src_memory\s*=\s*#micro\.memory<(\w+)>"
                      r".*?dst_memory\s*=\s*#micro\.memory<(\w+)>.*?:\s*tensor<([^>]*)>")
_STORE_RE = re.compile(r"micro\.(?:store|tile_store)\b.*?src_memory\s*=\s*#micro\.memory<(\w+)>"
                       r".*?dst_memory\s*=\s*#micro\.memory<(\w+)>.*?:\s*tensor<([^>]*)>")
_KERNEL_RE = re.compile(r"micro\.kernel\s+@(\w+)")
_SIG_RE = re.compile(r"%arg\d+:\s*tensor<([^>]*)>")


def _tensor_bytes(spec: str) -> int:
    parts = spec.split("x")
    n = 1
    for p in parts[:-1]:
        n *= int(p)
    return n * KNOWN_DTYPES[parts[-1].strip()]


@dataclass
class L0Report:
    kernel: str
    total_flops: int = 0
    bytes_by_memory: dict = field(default_factory=dict)
    compulsory_dram_bytes: int = 0
    compute_cycles: float = 0.0
    memory_cycles: dict = field(default_factory=dict)
    predicted_cycles: float = 0.0
    bottleneck: str = ""


def l0_bound(micro_text: str, machine: MachineModel) -> L0Report:
    """L0 static bound of the (single) micro.kernel in `micro_text`."""
    km = _KERNEL_RE.search(micro_text)
    rep = L0Report(kernel=km.group(1) if km else "<anonymous>")
    trips = []  # enclosing loop trip counts, innermost last
    flops_by_engine = {}
    for line in micro_text.splitlines():
        s = line.strip()
        if s.startswith("//"):
            rep.compulsory_dram_bytes += sum(_tensor_bytes(t) for t in _SIG_RE.findall(s))
            continue
        lm = _LOOP_RE.search(s)
        if lm:
            a, b, st = int(lm.group(1)), int(lm.group(2)), int(lm.group(3))
            trips.append(max(0, math.ceil((b - a) / st)))
            continue
        if s.endswith("{"):  # kernel, pipeline and other regions: no repetition
            trips.append(1)
            continue
        if s == "}":
            if trips:
                trips.pop()
            continue
        mult = math.prod(trips) if trips else 1
        mm = _MMA_RE.search(s)
        if mm:
            m, n, k = int(mm.group(1)), int(mm.group(2)), int(mm.group(3))
            f = 2 * m * n * k * mult
            flops_by_engine[mm.group(4)] = flops_by_engine.get(mm.group(4), 0) + f
            rep.total_flops += f
            continue
        for rx in (_COPY_RE, _STORE_RE):
            cm = rx.search(s)
            if cm:
                b = _tensor_bytes(cm.group(3)) * mult
                for space in (cm.group(1), cm.group(2)):
                    rep.bytes_by_memory[space] = rep.bytes_by_memory.get(space, 0) + b
                break
    compute = 0.0
    for eng, f in flops_by_engine.items():
        e = machine.engine(eng)
        compute += f / (int(e["count"]) * float(e["flops_per_cycle"]))
    rep.compute_cycles = compute
    dram = max(rep.compulsory_dram_bytes, rep.bytes_by_memory.get("dram", 0))
    traffic = dict(rep.bytes_by_memory)
    traffic["dram"] = dram
    for space, b in traffic.items():
        if space in machine.memory:
            rep.memory_cycles[space] = b / float(machine.memory[space]["bandwidth_bytes_per_cycle"])
    mem_bound = max(rep.memory_cycles.values()) if rep.memory_cycles else 0.0
    rep.predicted_cycles = max(compute, mem_bound)
    if compute >= mem_bound:
        rep.bottleneck = "matrix_engine"
    else:
        rep.bottleneck = max(rep.memory_cycles, key=rep.memory_cycles.get) + "_bandwidth"
    return rep


def report_yaml(rep: L0Report, machine: MachineModel) -> str:
    ns = rep.predicted_cycles / machine.clock_hz * 1e9
    d = {"schema_version": 1, "machine": machine.name, "kernel": rep.kernel, "level": 0,
         "predicted_cycles": int(math.ceil(rep.predicted_cycles)), "predicted_ns": round(ns, 1),
         "total_flops": rep.total_flops,
         "utilization": {"matrix": round(rep.compute_cycles / rep.predicted_cycles, 3) if rep.predicted_cycles else 0},
         "bandwidth": {k: round(v / rep.predicted_cycles, 3) if rep.predicted_cycles else 0
                       for k, v in rep.memory_cycles.items()},
         "bytes": dict(rep.bytes_by_memory, dram=max(rep.compulsory_dram_bytes, rep.bytes_by_memory.get("dram", 0))),
         "bottleneck": rep.bottleneck, "capacity_violations": []}
    return yaml.safe_dump(d, sort_keys=False)
