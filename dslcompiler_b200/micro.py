"""micro.kernel dispatch and micro.search_space for the B200 target.

The reference's Micro-IR specs make ``micro.kernel`` the canonical execution
artifact of a lowered LLK op and ``micro.search_space`` the source of legal
schedule choices that ``llk-tune`` searches
(``docs/superpowers/specs/2026-08-11-llk-to-micro-lowering-implementation-spec.md:136-142,362-428``,
``docs/superpowers/specs/2026-08-11-micro-ir-dialect-implementation-spec.md:769-850``).
This module closes the loop for the sm_100a kernels:

* :func:`parse_micro_kernel` reads a ``micro.kernel`` (as printed by
  ``llk-compile --emit micro``) back into its dispatch record: the
  candidate kernel, the problem size and the launch-plan attributes;
* :func:`run_micro` installs that plan for the op's KernelKey through the C
  ABI (``llk_plan_insert``) and launches the named kernel through
  ``llk_swiglu_ex`` / ``llk_matmul`` -- a micro.kernel is a drop-in dispatch
  record, not a report;
* :func:`search_space` / :func:`emit_search_space` give the legal choices
  (``micro.param`` / ``micro.constraint`` / ``micro.objective``) and
  :func:`candidates` the launch plans they span after the legality rules,
  which is what ``llk-tune`` measures.

The attribute and op spellings follow the reference's micro dialect specs;
the parser reads them with whitespace, line breaks and attribute order free.
"""
from __future__ import annotations

import itertools
import re
from dataclasses import dataclass, field

from . import capi

TARGET = "b200-sm100a"
SM_COUNT = 148            # B200 SMs (2 dies x 74)
SMEM_OPTIN = 227 * 1024   # shared memory per CTA (opt-in)
TMEM_COLUMNS = 512        # 32-bit TMEM columns per SM (128 lanes each)

# Kernel names a micro.kernel's `candidate` may carry -> library variant.
CANDIDATES = {
    "tc2_kernel": "tc",        # CTA pairs, tcgen05 cta_group::2 (block_m 256)
    "tc_swiglu_kernel": "tc",  # one CTA per tile, cta_group::1 (block_m 128)
    "decode_kernel": "decode",  # small-M weight streaming (swap-AB)
    "simt_kernel": "simt",     # CUDA-core kernel for any stride / alignment
}


class MicroError(ValueError):
    """A micro.kernel / micro.search_space that cannot be dispatched."""


# ------------------------------------------------------------------ parsing
def _balanced(text: str, start: int, open_ch: str, close_ch: str) -> int:
    """Index just past the bracket that closes text[start] (== open_ch)."""
    depth = 0
    for i in range(start, len(text)):
        c = text[i]
        if c == open_ch:
            depth += 1
        elif c == close_ch:
            depth -= 1
            if depth == 0:
                return i + 1
    raise MicroError(f"unbalanced {open_ch}{close_ch} at offset {start}")


def _split_top(s: str, sep: str = ",") -> list[str]:
    """Split on `sep` outside (), [], {}, <> and quotes."""
    out, depth, cur, quote = [], 0, [], False
    for c in s:
        if c == '"':
            quote = not quote
        if not quote:
            if c in "([{<":
                depth += 1
            elif c in ")]}>":
                depth -= 1
            elif c == sep and depth == 0:
                out.append("".join(cur))
                cur = []
                continue
        cur.append(c)
    if "".join(cur).strip():
        out.append("".join(cur))
    return out


def parse_value(v: str):
    """An attribute value: integer, float, quoted string, [list] or the raw
    text (e.g. #micro.map<worker>)."""
    v = v.strip()
    if v.startswith('"') and v.endswith('"'):
        return v[1:-1]
    if v.startswith("[") and v.endswith("]"):
        return [parse_value(x) for x in _split_top(v[1:-1])]
    v_num = re.sub(r"\s*:\s*i\d+$", "", v)
    try:
        return int(v_num)
    except ValueError:
        pass
    try:
        return float(v_num)
    except ValueError:
        return v


def parse_attr_dict(body: str) -> dict:
    """`{a = 1, b = "x", c = [1, 2], d = #micro.map<worker>}` (braces
    included or not) -> dict."""
    body = body.strip()
    if body.startswith("{"):
        body = body[1:-1]
    out = {}
    for item in _split_top(body):
        if "=" not in item:
            continue
        k, v = item.split("=", 1)
        out[k.strip()] = parse_value(v)
    return out


def _strip_comments(text: str) -> str:
    return re.sub(r"//[^\n]*", "", text)


@dataclass
class MicroKernel:
    """Dispatch record of one micro.kernel."""
    name: str
    attrs: dict
    op: str                      # "fused_swiglu" | "matmul"
    candidate: str
    M: int
    N: int
    K: int
    block_m: int
    block_n: int
    block_k: int
    stages: int
    y_dtype: str
    math_mode: str
    plan: dict = field(default_factory=dict)

    @property
    def variant(self) -> str:
        return CANDIDATES[self.candidate]


def parse_micro_kernels(text: str) -> list[MicroKernel]:
    """Every micro.kernel in an MLIR text."""
    text = _strip_comments(text)
    out = []
    for m in re.finditer(r"micro\.kernel\s+@([\w.$-]+)", text):
        i = m.end()
        attrs = {}
        am = re.match(r"\s*attributes\s*", text[i:])
        if am:
            j = i + am.end()
            if text[j] != "{":
                raise MicroError("micro.kernel attributes must be a dictionary")
            k = _balanced(text, j, "{", "}")
            attrs = parse_attr_dict(text[j:k])
            i = k
        b = text.index("{", i)
        body = text[b:_balanced(text, b, "{", "}")]
        out.append(_kernel_record(m.group(1), attrs, body))
    return out


def parse_micro_kernel(text: str) -> MicroKernel:
    ks = parse_micro_kernels(text)
    if len(ks) != 1:
        raise MicroError(f"expected one micro.kernel, found {len(ks)}")
    return ks[0]


_FOR_RE = re.compile(r"micro\.(spatial_for|for)\s+%(\w+)\s*=\s*(-?\d+)\s+to\s+(-?\d+)\s+step\s+(\d+)")


def _kernel_record(name: str, attrs: dict, body: str) -> MicroKernel:
    for req in ("workload", "target", "candidate"):
        if req not in attrs:
            raise MicroError(f"micro.kernel @{name}: missing attribute '{req}'")
    if attrs["target"] != TARGET:
        raise MicroError(f"micro.kernel @{name}: target {attrs['target']!r} is not {TARGET!r}")
    cand = str(attrs["candidate"]).split("<")[0]
    if cand not in CANDIDATES:
        raise MicroError(f"micro.kernel @{name}: unknown candidate {attrs['candidate']!r}")
    op = attrs["workload"]
    if op not in ("fused_swiglu", "matmul"):
        raise MicroError(f"micro.kernel @{name}: unsupported workload {op!r}")
    loops = {m.group(2): (m.group(1), int(m.group(3)), int(m.group(4)), int(m.group(5))) for m in _FOR_RE.finditer(body)}
    st = re.search(r"micro\.pipeline\s+stages\s*=\s*(\d+)", body)
    stages = int(st.group(1)) if st else int(attrs.get("stages", 0))
    if "bk" not in loops:
        raise MicroError(f"micro.kernel @{name}: no reduction loop micro.for %bk")
    K, block_k = loops["bk"][2], loops["bk"][3]
    if cand == "decode_kernel":
        if "bn" not in loops:
            raise MicroError(f"micro.kernel @{name}: no spatial loop %bn")
        N, block_n = loops["bn"][2], loops["bn"][3]
        acc = re.search(r"%acc_wg\s*=\s*micro\.alloc\s+tensor<(\d+)x(\d+)xf32>", body)
        if not acc:
            raise MicroError(f"micro.kernel @{name}: no gate accumulator")
        block_m = int(acc.group(2))
        M = int(attrs.get("M", 0))
        if M <= 0:
            raise MicroError(f"micro.kernel @{name}: decode kernel needs the M attribute")
    else:
        if "bm" not in loops or "bn" not in loops:
            raise MicroError(f"micro.kernel @{name}: no spatial loops %bm / %bn")
        M, block_m = loops["bm"][2], loops["bm"][3]
        N, block_n = loops["bn"][2], loops["bn"][3]
    store = re.findall(r"micro\.store\s+[^:]*:\s*tensor<[^>]*x(\w+)>", body)
    y_dtype = store[-1] if store else ("bf16" if op == "fused_swiglu" else "f32")
    mm = re.search(r'micro\.vector\s+"silu"[^{]*\{([^}]*)\}', body)
    math_mode = str(parse_attr_dict(mm.group(1)).get("math_mode", "strict")) if mm else "strict"
    if math_mode not in capi.MATH_MODES:
        raise MicroError(f"micro.kernel @{name}: unknown math_mode {math_mode!r}")
    rec = MicroKernel(name, attrs, op, cand, M, N, K, block_m, block_n, block_k, stages, y_dtype, math_mode)
    rec.plan = _plan_of(rec)
    return rec


def _plan_of(k: MicroKernel) -> dict:
    """The llk_launch_plan fields the kernel's attributes and loops fix."""
    a = k.attrs
    plan = {"variant": capi.VARIANTS[k.variant], "block_m": k.block_m, "block_n": k.block_n, "block_k": k.block_k,
            "stages": k.stages, "grid": int(a.get("grid", 0)), "split_k": int(a.get("split_k", 0)),
            "sched": int(a.get("sched", 0)), "threads": int(a.get("threads", 192)),
            "smem_bytes": int(a.get("smem_bytes", 0))}
    return plan


# ----------------------------------------------------------------- dispatch
def kernel_key(k: MicroKernel):
    """The KernelKey the library files this kernel's plan under."""
    from .swiglu import KernelKey

    opcode = capi.LLK_OP_FUSED_SWIGLU if k.op == "fused_swiglu" else capi.LLK_OP_MATMUL
    out = capi.LLK_DTYPE_FP32 if k.y_dtype == "f32" else capi.LLK_DTYPE_BF16
    math = capi.MATH_MODES[k.math_mode] if k.op == "fused_swiglu" else capi.LLK_MATH_STRICT
    return KernelKey(operation=opcode, output_type=out, M_bucket=capi.lib().llk_classify_m(k.M), N=k.N, K=k.K,
                     thread_count=capi.VARIANTS[k.variant], math_mode=math)


def install(k: MicroKernel) -> None:
    """Install the kernel's launch plan for its key (llk_plan_insert): later
    calls of the op with this shape run exactly this kernel and plan."""
    kernel_key(k).insert_plan(**k.plan)


def run_micro(text, x, w0, w1=None, *, out=None, stream=None, device=None):
    """Dispatch a micro.kernel: parse it, install its plan for the op's key,
    and launch the kernel it names on the given operands.

    text: the micro.kernel (str) or a parsed :class:`MicroKernel`.
    fused_swiglu: x [M,K], w0 = Wg, w1 = Wu (bf16); matmul: x = A, w0 = B.
    The operand shapes must be the kernel's M/N/K.  Returns Y (or C)."""
    from .swiglu import fused_swiglu, matmul

    k = text if isinstance(text, MicroKernel) else parse_micro_kernel(text)
    M, K = x.shape[0], x.shape[1]
    N = w0.shape[1]
    if (M, N, K) != (k.M, k.N, k.K):
        raise MicroError(f"operands are M={M} N={N} K={K}; @{k.name} was lowered for M={k.M} N={k.N} K={k.K}")
    install(k)
    if k.op == "fused_swiglu":
        if w1 is None:
            raise MicroError("fused_swiglu needs Wg and Wu")
        return fused_swiglu(x, w0, w1, out=out, out_dtype=k.y_dtype, variant=k.variant, stream=stream,
                            device=device, math_mode=k.math_mode)
    return matmul(x, w0, out, variant=k.variant, stream=stream, device=device)


# ------------------------------------------------------------- search space
def _padded_m(M: int) -> int:
    return 16 if M <= 16 else 32 if M <= 32 else 64 if M <= 64 else 128


@dataclass
class SearchSpace:
    name: str
    workload: str
    M: int
    N: int
    K: int
    params: dict                 # name -> choices
    constraints: list            # (name, {attrs})
    objective: str = "latency"


def search_space(op: str, M: int, N: int, K: int) -> SearchSpace:
    """The B200 launch-plan choices for an op and shape (the micro.param
    choices) and the legality rules they must pass (micro.constraint)."""
    swiglu = op == "fused_swiglu"
    params = {
        "candidate": ["tc2_kernel", "tc_swiglu_kernel"] + (["decode_kernel"] if swiglu and M <= 128 else []),
        "BM": [256, 128],
        "BN": [128] if swiglu else [256],
        "BK": [64],
        "num_stages": [4, 6],
        "grid": [148, 144, 128, 112],
        "tail_split": [0, 1, 2, 4, -2, -3, -4, -5, -6, -8],
        "sched": [1, 0],
    }
    if swiglu and M <= 128:
        params["decode_BM"] = [_padded_m(M)]
        params["decode_stages"] = [3, 4, 6, 8]
        params["decode_cluster"] = [0, 2, 4, 8]
        params["decode_grid"] = [56, 74, 112, 148, 296]
    constraints = [
        ("sram_capacity", {"params": ["BM", "BN", "BK", "num_stages"], "memory": "#micro.memory<sram>",
                           "limit_bytes": SMEM_OPTIN}),
        ("acc_capacity", {"params": ["BM", "BN"], "memory": "#micro.memory<acc>", "limit_columns": TMEM_COLUMNS}),
        ("mma_compatible", {"params": ["BM", "BN", "BK"], "input": "#micro.dtype<bf16>",
                            "accumulator": "#micro.dtype<f32>"}),
        ("mapping_extent", {"params": ["grid", "BM"], "sm_count": SM_COUNT}),
        ("tail_supported", {"params": ["tail_split", "sched", "BM"]}),
        ("pipeline_live_tiles", {"params": ["num_stages"]}),
    ]
    return SearchSpace(f"{op}_M{M}_N{N}_K{K}_space", op, M, N, K, params, constraints)


def _tc_stage_bytes(bm: int) -> int:
    # per CTA: 128 rows of X x 64 k + that CTA's 128 weight columns x 64 k (bf16)
    return (128 * 64 + 128 * 64) * 2 if bm == 256 else (128 * 64 + 256 * 64) * 2


def legal(space: SearchSpace, c: dict) -> tuple[bool, str]:
    """Whether one choice of every param passes the constraints; the reason
    when it does not.  Mirrors the plans the kernels accept."""
    k_blocks = -(-space.K // 64)
    if c["candidate"] == "decode_kernel":
        mp, st = c["decode_BM"], c["decode_stages"]
        stage = 4 * 64 * 64 * 2 + ((mp * 64 * 2 + 1023) // 1024) * 1024
        if st * stage + 1024 + 256 > SMEM_OPTIN:
            return False, "sram_capacity"
        if 4 * mp > TMEM_COLUMNS:
            return False, "acc_capacity"
        s = c["decode_cluster"]
        tiles = -(-space.N // 128)
        if s:
            if s > k_blocks or tiles * s > 2 * SM_COUNT or st * stage < 2 * mp * 128 * 4:
                return False, "mapping_extent"
        elif c["decode_grid"] > tiles * k_blocks:
            return False, "mapping_extent"
        return True, ""
    bm = c["BM"]
    pair = c["candidate"] == "tc2_kernel"
    if pair != (bm == 256):
        return False, "mma_compatible"
    if pair and space.M <= 128:
        return False, "mapping_extent"
    smem = c["num_stages"] * _tc_stage_bytes(bm) + (32 * 1024 if pair else 0) + 2048
    if smem > SMEM_OPTIN:
        return False, "sram_capacity"
    if c["num_stages"] < 2:
        return False, "pipeline_live_tiles"
    if c["grid"] > SM_COUNT or (pair and c["grid"] % 2):
        return False, "mapping_extent"
    ts = c["tail_split"]
    if not pair and (ts not in (0, 1) or c["sched"] != 1):
        return False, "tail_supported"
    if ts < 0 and (-ts > k_blocks or c["sched"] != 1):
        return False, "tail_supported"
    if pair and c["num_stages"] != 6:
        return False, "sram_capacity"  # the pair kernel's ring is fixed at 6 stages
    if not pair and c["num_stages"] != 4:
        return False, "sram_capacity"  # the one-CTA kernel's ring is fixed at 4 stages
    return True, ""


def candidates(space: SearchSpace) -> list[dict]:
    """Every legal launch plan of the space, as llk_launch_plan dicts."""
    out, seen = [], set()
    p = space.params
    tc_keys = ["BM", "BN", "BK", "num_stages", "grid", "tail_split", "sched"]
    for cand in p["candidate"]:
        if cand == "decode_kernel":
            combos = itertools.product(p["decode_BM"], p["decode_stages"], p["decode_cluster"], p["decode_grid"])
            for mp, st, s, g in combos:
                c = {"candidate": cand, "decode_BM": mp, "decode_stages": st, "decode_cluster": s, "decode_grid": g}
                if s:
                    c["decode_grid"] = -(-space.N // 128) * s
                if not legal(space, c)[0]:
                    continue
                plan = {"variant": capi.VARIANTS["decode"], "block_m": mp, "block_n": 128, "block_k": 64,
                        "stages": st, "split_k": s if s else 0, "grid": c["decode_grid"], "threads": 192,
                        "smem_bytes": 0, "sched": 1 if s else 0}
                key = tuple(sorted(plan.items()))
                if key not in seen:
                    seen.add(key)
                    out.append(plan)
            continue
        for vals in itertools.product(*(p[k] for k in tc_keys)):
            c = dict(zip(tc_keys, vals), candidate=cand)
            if not legal(space, c)[0]:
                continue
            plan = {"variant": capi.VARIANTS["tc"], "block_m": c["BM"], "block_n": c["BN"], "block_k": c["BK"],
                    "stages": c["num_stages"], "split_k": c["tail_split"], "grid": c["grid"], "threads": 192,
                    "smem_bytes": 0, "sched": c["sched"]}
            key = tuple(sorted(plan.items()))
            if key not in seen:
                seen.add(key)
                out.append(plan)
    return out


def emit_search_space(space: SearchSpace) -> str:
    """micro.search_space text (micro-ir-dialect spec section 8)."""
    L = [f'micro.search_space @{space.name} attributes {{workload = "{space.workload}", target = "{TARGET}", '
         f"M = {space.M}, N = {space.N}, K = {space.K}}} {{"]
    for name, choices in space.params.items():
        ch = ", ".join(f'"{c}"' if isinstance(c, str) else str(c) for c in choices)
        L.append(f'  %{name} = micro.param "{name}" : {"!micro.string" if isinstance(choices[0], str) else "i64"} '
                 f"{{choices = [{ch}]}}")
    for name, attrs in space.constraints:
        items = []
        for k, v in attrs.items():
            if isinstance(v, list):
                items.append(f"{k} = [" + ", ".join(f'"{x}"' for x in v) + "]")
            elif isinstance(v, str) and v.startswith("#"):
                items.append(f"{k} = {v}")
            else:
                items.append(f"{k} = {v}")
        L.append(f'  micro.constraint "{name}" {{{", ".join(items)}}}')
    L.append(f'  micro.objective minimize "{space.objective}" {{secondary = ["maximize matrix_utilization", '
             f'"minimize dram_bytes"]}}')
    L.append("}")
    return "\n".join(L) + "\n"


def parse_search_space(text: str) -> SearchSpace:
    """A micro.search_space text back into a SearchSpace (params and
    constraints), e.g. to generate candidates from a stored space."""
    text = _strip_comments(text)
    m = re.search(r"micro\.search_space\s+@([\w.$-]+)\s*attributes\s*", text)
    if not m:
        raise MicroError("no micro.search_space")
    j = m.end()
    k = _balanced(text, j, "{", "}")
    attrs = parse_attr_dict(text[j:k])
    b = text.index("{", k)
    body = text[b:_balanced(text, b, "{", "}")]
    params = {}
    for pm in re.finditer(r'micro\.param\s+"(\w+)"\s*:\s*[^{]*\{([^}]*)\}', body):
        params[pm.group(1)] = parse_attr_dict(pm.group(2)).get("choices", [])
    if not params:
        raise MicroError("micro.search_space without micro.param")
    cons = [(cm.group(1), parse_attr_dict(cm.group(2)))
            for cm in re.finditer(r'micro\.constraint\s+"(\w+)"\s*\{([^}]*)\}', body)]
    return SearchSpace(m.group(1), attrs.get("workload", ""), int(attrs.get("M", 0)), int(attrs.get("N", 0)),
                       int(attrs.get("K", 0)), params, cons)
