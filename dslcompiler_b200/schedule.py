"""Schedule database for the sm_100a kernels.

Same file format as the reference's ``schedules/schedule_db.json``
(``{"version": 1, "entries": [{"operation", "target", "shape": {"M_bucket",
"N", "K"}, "dtype", "math_mode", "schedule": {...}}]}``), read by
``lib/Transforms/Common/ScheduleLoader.cpp:31-98``.  Two differences, both
deliberate:

* the loader matches ``target`` and the exact ``N``/``K`` (the reference's
  loader reads N/K but never compares them and ignores ``target``,
  ``ScheduleLoader.cpp:59-76``), so an AVX2 entry can never be applied to the
  GPU;
* a B200 schedule holds a launch plan (``variant``, ``block_m``,
  ``block_n``, ``block_k``, ``stages``, ``split_k``, ``grid``) instead of the
  CPU's BM/BN/BK/VM/VN/threads; :func:`install` hands matching entries to the
  library's plan cache (``llk_plan_insert``) so launches use them.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

from . import capi

TARGET = "b200-sm100a"
DEFAULT_DB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "schedules", "schedule_db.json")
PLAN_FIELDS = ("variant", "block_m", "block_n", "block_k", "stages", "split_k", "grid", "threads", "smem_bytes", "sched")
VARIANT_NAMES = {v: k for k, v in capi.VARIANTS.items()}
OPS = {"fused_swiglu": capi.LLK_OP_FUSED_SWIGLU, "matmul": capi.LLK_OP_MATMUL}
DTYPES = {"bf16": capi.LLK_DTYPE_BF16, "f32": capi.LLK_DTYPE_FP32}


def classify_m(M: int) -> int:
    """M bucket: {1}, [2,4], [5,16], [17,64], >=65 (ScheduleLoader.cpp:19-29)."""
    if M == 1:
        return 0
    if M <= 4:
        return 1
    if M <= 16:
        return 2
    if M <= 64:
        return 3
    return 4


@dataclass
class ScheduleEntry:
    operation: str
    target: str
    M_bucket: int
    N: int
    K: int
    dtype: str = "bf16"
    math_mode: str = "strict"
    schedule: dict = field(default_factory=dict)
    measured_gflops: float | None = None

    def to_json(self) -> dict:
        d = {"operation": self.operation, "target": self.target,
             "shape": {"M_bucket": self.M_bucket, "N": self.N, "K": self.K},
             "dtype": self.dtype, "math_mode": self.math_mode, "schedule": dict(self.schedule)}
        if self.measured_gflops is not None:
            d["measured_gflops"] = self.measured_gflops
        return d


def read_db(path: str = DEFAULT_DB) -> list[ScheduleEntry]:
    """All well-formed entries of a schedule DB file; malformed ones are
    skipped (the reference's loader does the same, ScheduleLoader.cpp:55-71)."""
    with open(path) as f:
        root = json.load(f)
    out = []
    for e in root.get("entries", []) if isinstance(root, dict) else []:
        try:
            sh = e["shape"]
            out.append(ScheduleEntry(operation=e["operation"], target=e.get("target", ""),
                                     M_bucket=int(sh["M_bucket"]), N=int(sh["N"]), K=int(sh["K"]),
                                     dtype=e.get("dtype", "bf16"), math_mode=e.get("math_mode", ""),
                                     schedule=dict(e.get("schedule", {})),
                                     measured_gflops=e.get("measured_gflops")))
        except (KeyError, TypeError, ValueError):
            continue
    return out


def load(path: str, M_bucket: int, N: int, K: int, operation: str = "fused_swiglu",
         target: str = TARGET, dtype: str | None = None) -> list[ScheduleEntry]:
    """Entries for exactly this (operation, target, M bucket, N, K[, dtype]),
    best measured first."""
    hits = [e for e in read_db(path) if e.operation == operation and e.target == target
            and e.M_bucket == M_bucket and e.N == N and e.K == K and (dtype is None or e.dtype == dtype)]
    hits.sort(key=lambda e: -(e.measured_gflops or 0.0))
    return hits


def write_db(entries: list[ScheduleEntry], path: str, merge: bool = True) -> None:
    """Write entries; with merge, replace same-key entries of an existing file
    and keep the rest (other targets included)."""
    old = read_db(path) if merge and os.path.exists(path) else []

    def key(e):
        return (e.operation, e.target, e.M_bucket, e.N, e.K, e.dtype)

    new_keys = {key(e) for e in entries}
    keep = [e for e in old if key(e) not in new_keys]
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "w") as f:
        json.dump({"version": 1, "entries": [e.to_json() for e in keep + entries]}, f, indent=2)
        f.write("\n")


def entry_key(e: ScheduleEntry):
    """The library KernelKey a B200 entry applies to."""
    from .swiglu import KernelKey

    variant = e.schedule.get("variant", "tc")
    v = capi.VARIANTS[variant] if isinstance(variant, str) else int(variant)
    math = capi.MATH_MODES.get(e.math_mode, capi.LLK_MATH_STRICT) if e.operation == "fused_swiglu" else \
        capi.LLK_MATH_STRICT
    return KernelKey(operation=OPS[e.operation], output_type=DTYPES.get(e.dtype, capi.LLK_DTYPE_BF16),
                     M_bucket=e.M_bucket, N=e.N, K=e.K, thread_count=v, math_mode=math)


def entry_plan(e: ScheduleEntry) -> dict:
    p = {f: int(e.schedule.get(f, 0)) for f in PLAN_FIELDS if f != "variant"}
    variant = e.schedule.get("variant", "tc")
    p["variant"] = capi.VARIANTS[variant] if isinstance(variant, str) else int(variant)
    return p


def install(path: str = DEFAULT_DB, target: str = TARGET) -> int:
    """Installs every entry of `target` into the library's plan cache;
    returns how many."""
    n = 0
    for e in read_db(path):
        if e.target != target or e.operation not in OPS:
            continue
        entry_key(e).insert_plan(**entry_plan(e))
        n += 1
    return n
