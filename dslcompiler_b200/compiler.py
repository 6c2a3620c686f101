"""LLK -> micro lowering for the B200 target.

The reference lowers ``llk.fused_swiglu`` through Linalg to AVX2 code and
specifies (but never implements) an ``LLKToMicro`` lowering that produces a
``micro.kernel`` for the chosen schedule
(``docs/superpowers/specs/2026-08-11-llk-to-micro-lowering-implementation-spec.md:112-318``).
Here that lowering targets the sm_100a kernels: it reads the op from MLIR
text, applies the op verifier's rules (``lib/Dialect/LLK/LLKOps.cpp:42-83``;
``MicroOps.cpp:246-291`` for the emitted ``micro.mma``), resolves the launch
plan the library would use (KernelKey -> plan cache, optionally seeded from
the schedule DB), and prints the ``micro.kernel`` that describes exactly that
kernel: CTA-pair tiles, the TMA pipeline, the tcgen05 MMA shape and the fused
epilogue.  The micro kernel is the dispatch record -- ``target =
"b200-sm100a"`` and ``candidate`` name the CUDA kernel it runs -- and is what
``micro-perf`` consumes.

No MLIR installation is involved; the parser understands the ops' custom
assembly format (``include/LLK/Dialect/LLKOps.td:43-48, 239-244``).
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field

from . import capi

DYN = -1  # '?' dimension

_TENSOR_RE = re.compile(r"tensor<([^>]*)>")
_OP_NAME_RE = re.compile(r'(?P<res>%[\w.#]+(?::\d+)?)\s*=\s*(?P<q>"?)llk\.(?P<op>fused_swiglu|matmul)(?P=q)')


class VerifyError(ValueError):
    """The op fails the reference verifier's rules."""


@dataclass
class TensorType:
    shape: list
    dtype: str

    @staticmethod
    def parse(text: str) -> "TensorType":
        m = _TENSOR_RE.search(text)
        if not m:
            raise VerifyError(f"expected a tensor type, got {text!r}")
        parts = m.group(1).split("x")
        dims = [DYN if p.strip() == "?" else int(p) for p in parts[:-1]]
        return TensorType(dims, parts[-1].strip())

    def __str__(self):
        return "tensor<" + "x".join("?" if d == DYN else str(d) for d in self.shape) + "x" + self.dtype + ">"


@dataclass
class LLKOp:
    op: str                      # "fused_swiglu" or "matmul"
    operands: list               # operand SSA names
    types: list                  # TensorType per operand (ins then outs)
    result_type: TensorType
    attrs: dict = field(default_factory=dict)

    @property
    def x(self):
        return self.types[0]


def _balanced_end(text: str, start: int, open_ch: str, close_ch: str) -> int:
    depth = 0
    for i in range(start, len(text)):
        if text[i] == open_ch:
            depth += 1
        elif text[i] == close_ch:
            depth -= 1
            if depth == 0:
                return i + 1
    raise VerifyError(f"unbalanced {open_ch}{close_ch}")


def _types(text: str) -> list:
    return [TensorType.parse("tensor<" + t) for t in text.split("tensor<")[1:]]


def _attrs(body: str) -> dict:
    from .micro import parse_attr_dict

    return {k: str(v) for k, v in parse_attr_dict(body).items()}


def parse_llk(text: str) -> list[LLKOp]:
    """Every llk.fused_swiglu / llk.matmul op in an MLIR text, in the ops'
    custom assembly format (``include/LLK/Dialect/LLKOps.td:43-48``:
    ``%r = llk.op ins(%a, .. : T, ..) outs(%i : T) {attrs} -> T``) or the
    generic one (``%r = "llk.op"(%a, .., %i) {attrs} : (T, ..) -> T``), with
    any line breaks, spacing and comments."""
    text = re.sub(r"//[^\n]*", "", text)
    ops = []
    for m in _OP_NAME_RE.finditer(text):
        i = m.end()
        if m.group("q"):  # generic form
            j = text.index("(", i)
            k = _balanced_end(text, j, "(", ")")
            names = [s.strip() for s in text[j + 1:k - 1].split(",") if s.strip()]
            rest = text[k:]
            attrs = {}
            am = re.match(r"\s*\{", rest)
            if am:
                a0 = k + am.end() - 1
                a1 = _balanced_end(text, a0, "{", "}")
                attrs = _attrs(text[a0:a1])
                k = a1
            tm = re.match(r"\s*:\s*\(", text[k:])
            if not tm:
                raise VerifyError("generic llk op without a function type")
            t0 = k + tm.end() - 1
            t1 = _balanced_end(text, t0, "(", ")")
            types = _types(text[t0:t1])
            rm = re.match(r"\s*->\s*(tensor<[^>]*>)", text[t1:])
            if not rm:
                raise VerifyError("generic llk op without a result type")
            ops.append(LLKOp(m.group("op"), names, types, TensorType.parse(rm.group(1)), attrs))
            continue
        # custom form
        im = re.match(r"\s*ins\s*\(", text[i:])
        if not im:
            continue
        j = i + im.end() - 1
        k = _balanced_end(text, j, "(", ")")
        ins = text[j + 1:k - 1]
        om = re.match(r"\s*outs\s*\(", text[k:])
        if not om:
            raise VerifyError(f"llk.{m.group('op')} without outs(...)")
        j2 = k + om.end() - 1
        k2 = _balanced_end(text, j2, "(", ")")
        outs = text[j2 + 1:k2 - 1]
        attrs = {}
        am = re.match(r"\s*(attributes\s*)?\{", text[k2:])
        pos = k2
        if am:
            a0 = k2 + am.end() - 1
            a1 = _balanced_end(text, a0, "{", "}")
            attrs = _attrs(text[a0:a1])
            pos = a1
        rm = re.match(r"\s*->\s*(tensor<[^>]*>)", text[pos:])
        if not rm:
            raise VerifyError(f"llk.{m.group('op')} without a result type")
        in_names, in_types = ins.split(":", 1)
        out_names, out_types = outs.split(":", 1)
        names = [s.strip() for s in in_names.split(",")] + [s.strip() for s in out_names.split(",")]
        ops.append(LLKOp(m.group("op"), names, _types(in_types) + _types(out_types),
                         TensorType.parse(rm.group(1)), attrs))
    return ops


def op_math_mode(op: LLKOp) -> str:
    """The op's math_mode attribute (#llk.math_mode<strict> ..) as a name;
    strict when absent (the fused lowering's epilogue)."""
    v = op.attrs.get("math_mode", "")
    m = re.search(r"<\s*(\w+)\s*>", v)
    name = m.group(1) if m else (v.strip('"') or "strict")
    if name not in capi.MATH_MODES:
        raise VerifyError(f"unknown math_mode {name!r}")
    return name


def verify(op: LLKOp) -> None:
    """The reference's verifier rules (LLKOps.cpp:42-83 for fused_swiglu;
    the matmul contract lhs [M,K], rhs [K,N], acc [M,N])."""
    for t in op.types:
        if len(t.shape) != 2:
            raise VerifyError("operands must be 2D tensors")

    def mismatch(a, b):
        return a != DYN and b != DYN and a != b

    if op.op == "fused_swiglu":
        if len(op.types) != 4:
            raise VerifyError("llk.fused_swiglu takes X, Wg, Wu and one init")
        x, wg, wu, init = op.types
        if mismatch(x.shape[0], init.shape[0]):
            raise VerifyError(f"M dimension mismatch: X={x.shape[0]} vs init={init.shape[0]}")
        if mismatch(wg.shape[1], init.shape[1]):
            raise VerifyError(f"N dimension mismatch: Wg={wg.shape[1]} vs init={init.shape[1]}")
        if mismatch(x.shape[1], wg.shape[0]):
            raise VerifyError(f"K dimension mismatch between X={x.shape[1]} and Wg={wg.shape[0]}")
        if mismatch(x.shape[1], wu.shape[0]):
            raise VerifyError(f"K dimension mismatch between X={x.shape[1]} and Wu={wu.shape[0]}")
        if mismatch(wg.shape[1], wu.shape[1]):
            raise VerifyError(f"N dimension mismatch between Wg={wg.shape[1]} and Wu={wu.shape[1]}")
    else:
        if len(op.types) != 3:
            raise VerifyError("llk.matmul takes A, B and one init")
        a, b, c = op.types
        if mismatch(a.shape[1], b.shape[0]):
            raise VerifyError(f"K dimension mismatch between A={a.shape[1]} and B={b.shape[0]}")
        if mismatch(a.shape[0], c.shape[0]) or mismatch(b.shape[1], c.shape[1]):
            raise VerifyError("init shape must be [M, N]")
    for t in op.types[: 3 if op.op == "fused_swiglu" else 2]:
        if t.dtype != "bf16":
            raise VerifyError(f"the B200 kernels take bf16 inputs, got {t.dtype}")


def resolve_shape(op: LLKOp, M: int = 0, N: int = 0, K: int = 0) -> tuple[int, int, int]:
    """Static dims from the types; '?' dims from the --M/--N/--K values."""
    x, w = op.types[0], op.types[1]
    sm, sk, sn = x.shape[0], x.shape[1], w.shape[1]

    def pick(static, flag, name):
        if static != DYN:
            if flag and flag != static:
                raise VerifyError(f"--{name}={flag} contradicts the static dimension {static}")
            return static
        if flag <= 0:
            raise VerifyError(f"dimension {name} is dynamic: pass --{name}")
        return flag

    return pick(sm, M, "M"), pick(sn, N, "N"), pick(sk, K, "K")


@dataclass
class Lowered:
    name: str
    text: str
    plan: dict
    M: int
    N: int
    K: int
    op: str
    y_dtype: str


def _plan(op: str, M: int, N: int, K: int, y_dtype: str, variant: str = "auto", math_mode: str = "strict") -> dict:
    from .swiglu import KernelKey

    opcode = capi.LLK_OP_FUSED_SWIGLU if op == "fused_swiglu" else capi.LLK_OP_MATMUL
    out = capi.LLK_DTYPE_FP32 if y_dtype == "f32" else capi.LLK_DTYPE_BF16
    if variant == "auto":
        # the dispatcher's rule: decode kernel for <= 16 tokens of SwiGLU
        variant = "decode" if (op == "fused_swiglu" and M <= 16) else "tc"
    math = capi.MATH_MODES[math_mode] if op == "fused_swiglu" else capi.LLK_MATH_STRICT
    key = KernelKey(operation=opcode, output_type=out, M_bucket=capi.lib().llk_classify_m(M), N=N, K=K,
                    thread_count=capi.VARIANTS[variant], math_mode=math)
    return key.plan(M)


def _plan_attrs(plan: dict) -> str:
    """The launch-plan fields a micro.kernel carries (read back by
    micro.parse_micro_kernel to dispatch it)."""
    return (f"grid = {plan['grid']}, split_k = {plan['split_k']}, sched = {plan['sched']}, "
            f"threads = {plan['threads']}, smem_bytes = {plan['smem_bytes']}")


_DEF_RE = re.compile(r"^\s*(%\w+)(?:\s*,\s*%\w+)?\s*=\s*micro\.(\w+)\b(.*)$")
_ALLOC_TYPE_RE = re.compile(r"micro\.(?:alloc|tile_alloc)\s+tensor<([^>]*)>")
_TRAILING_TYPE_RE = re.compile(r":\s*tensor<([^>]*)>\s*$")
_MMA_LINE_RE = re.compile(r"micro\.mma\s+(%\w+)\s*,\s*(%\w+)\s*,\s*(%\w+)\s*\{(.*)\}")
_SHAPE_ATTR_RE = re.compile(r"shape\s*=\s*\[([^\]]*)\]")
_DTYPE_ATTR_RE = re.compile(r"(input|accumulator)\s*=\s*#micro\.dtype<(\w+)>")


def _tensor(spec: str):
    parts = spec.split("x")
    return [int(d) if d != "?" else -1 for d in parts[:-1]], parts[-1].strip()


def verify_micro(text: str) -> list[str]:
    """The micro.mma verifier rules (``lib/Dialect/Micro/MicroOps.cpp:246-291``)
    over micro IR text: each mma's operand types come from the ops that
    define them.  Returns the error messages (empty: valid)."""
    types = {}
    errors = []
    for n, line in enumerate(text.splitlines(), 1):
        m = _DEF_RE.match(line)
        if m:
            t = _ALLOC_TYPE_RE.search(line) or _TRAILING_TYPE_RE.search(line)
            if t:
                types[m.group(1)] = _tensor(t.group(1))
        mm = _MMA_LINE_RE.search(line)
        if not mm:
            continue

        def err(msg):
            errors.append(f"line {n}: 'micro.mma' op {msg}")

        operands = [types.get(v) for v in mm.group(1, 2, 3)]
        if any(o is None for o in operands):
            err("mma operands and result must be tile types")
            continue
        sh = _SHAPE_ATTR_RE.search(mm.group(4))
        shape = [int(v) for v in sh.group(1).split(",")] if sh and sh.group(1).strip() else []
        if len(shape) != 3:
            err("mma shape must have exactly 3 dimensions")
            continue
        if any(d <= 0 for d in shape):
            err("mma shape dimensions must be positive")
            continue
        M_, N_, K_ = shape
        (ls, lt), (rs, rt), (as_, at) = operands
        if len(ls) != 2 or len(rs) != 2 or len(as_) != 2:
            err("mma operands and result must be rank-2 tiles")
            continue

        def fits(expected, actual):
            return actual == -1 or expected == actual

        if not (fits(M_, ls[0]) and fits(K_, ls[1])):
            err("lhs tile shape must be [M, K]")
        elif not (fits(K_, rs[0]) and fits(N_, rs[1])):
            err("rhs tile shape must be [K, N]")
        elif not (fits(M_, as_[0]) and fits(N_, as_[1])):
            err("accumulator tile shape must be [M, N]")
        else:
            dts = dict(_DTYPE_ATTR_RE.findall(mm.group(4)))
            if lt != dts.get("input") or rt != dts.get("input"):
                err("input dtype must match operand element types")
            elif at != dts.get("accumulator"):
                err("accumulator dtype must match accumulator element type")
    return errors


def lower_to_micro(op: LLKOp, M: int, N: int, K: int, variant: str = "auto", schedule_id: str = "") -> Lowered:
    """The micro.kernel for the kernel and plan that will run this op."""
    y_dtype = op.result_type.dtype if op.result_type.dtype in ("bf16", "f32") else "bf16"
    math_mode = op_math_mode(op) if op.op == "fused_swiglu" else "strict"
    plan = _plan(op.op, M, N, K, y_dtype, variant, math_mode)
    v = plan["variant"]
    swiglu = op.op == "fused_swiglu"
    name = f"{op.op}_M{M}_N{N}_K{K}"
    sid = schedule_id or f"b200_builtin_v1_bucket{capi.lib().llk_classify_m(M)}"
    L = []
    if v == capi.VARIANTS["tc"]:
        bm, bn, bk, stages = plan["block_m"], plan["block_n"], plan["block_k"], plan["stages"]
        pair = bm == 256
        cand = ("tc2_kernel" if pair else "tc_swiglu_kernel") + f"<{'swiglu' if swiglu else 'matmul'}>"
        owner = "cta_pair" if pair else "worker"
        mma_n = 2 * bn if swiglu else bn
        engine = "tcgen05.cta_group::2" if pair else "tcgen05.cta_group::1"
        L.append(f'micro.kernel @{name} attributes {{workload = "{op.op}", target = "b200-sm100a", '
                 f'candidate = "{cand}", schedule_id = "{sid}", {_plan_attrs(plan)}}} {{')
        L.append(f"  micro.spatial_for %bm = 0 to {M} step {bm} map = #micro.map<{owner}> {{")
        L.append(f"    micro.spatial_for %bn = 0 to {N} step {bn} map = #micro.map<{owner}> {{")
        L.append(f"      %acc = micro.alloc tensor<{bm}x{mma_n}xf32> memory = #micro.memory<acc>")
        L.append(f"      micro.pipeline stages = {stages} {{")
        L.append(f"        micro.for %bk = 0 to {K} step {bk} {{")
        L.append(f"          %x_view = micro.tile_view %arg0[%bm, %bk] {{shape = [{bm}, {bk}], layout = #micro.layout<row_major>}}")
        L.append(f"          %x, %x_tok = micro.async_copy %x_view {{src_memory = #micro.memory<l2>, dst_memory = #micro.memory<sram>, owner = #micro.owner<dma>, layout = \"swizzled_128b\"}} : tensor<{bm}x{bk}xbf16>")
        toks = ["%x_tok"]
        wnames = ["wg", "wu"] if swiglu else ["b"]
        for i, w in enumerate(wnames):
            L.append(f"          %{w}_view = micro.tile_view %arg{i + 1}[%bk, %bn] {{shape = [{bk}, {bn}], layout = #micro.layout<row_major>}}")
            L.append(f"          %{w}, %{w}_tok = micro.async_copy %{w}_view {{src_memory = #micro.memory<l2>, dst_memory = #micro.memory<sram>, owner = #micro.owner<dma>, layout = \"swizzled_128b\"}} : tensor<{bk}x{bn}xbf16>")
            toks.append(f"%{w}_tok")
        L.append(f"          micro.wait {', '.join(toks)}")
        rhs = "%wg_wu" if swiglu else "%b"
        if swiglu:
            L.append(f"          %wg_wu = micro.concat %wg, %wu {{axis = 1}} : tensor<{bk}x{mma_n}xbf16>")
        L.append(f"          micro.mma %x, {rhs}, %acc {{shape = [{bm}, {mma_n}, {bk}], input = #micro.dtype<bf16>, "
                 f"accumulator = #micro.dtype<f32>, engine = \"{engine}\", owner = #micro.owner<matrix_engine>}}")
        L.append("        }")
        L.append("      }")
        if swiglu:
            L.append(f"      %gate = micro.slice %acc {{offsets = [0, 0], shape = [{bm}, {bn}]}}")
            L.append(f"      %up = micro.slice %acc {{offsets = [0, {bn}], shape = [{bm}, {bn}]}}")
            L.append(f'      %silu = micro.vector "silu" %gate {{math_mode = "{math_mode}"}}')
            L.append('      %out = micro.vector "mul" %silu, %up')
            L.append(f"      micro.store %out, %arg3 {{src_memory = #micro.memory<acc>, dst_memory = #micro.memory<dram>}} : tensor<{bm}x{bn}x{y_dtype}>")
        else:
            L.append(f"      micro.store %acc, %arg2 {{src_memory = #micro.memory<acc>, dst_memory = #micro.memory<dram>}} : tensor<{bm}x{bn}xf32>")
        L.append("    }")
        L.append("  }")
    else:  # decode kernel: weight-streaming, Y^T = W^T X^T, stream-K over (tile, k-block)
        # W^T and X^T are column-major views of the row-major W and X, so
        # each micro.mma is [M, K] x [K, N] -> [M, N] with M = 128 weight
        # columns and N = the padded token count; gate and up accumulate in
        # two accumulators (adjacent TMEM columns on the device).
        mp, bk = plan["block_m"], plan["block_k"]
        L.append(f'micro.kernel @{name} attributes {{workload = "{op.op}", target = "b200-sm100a", '
                 f'candidate = "decode_kernel", schedule_id = "{sid}", M = {M}, {_plan_attrs(plan)}}} {{')
        L.append(f"  micro.spatial_for %bn = 0 to {N} step 128 map = #micro.map<worker> {{")
        for w in ["wg", "wu"]:
            L.append(f"    %acc_{w} = micro.alloc tensor<128x{mp}xf32> memory = #micro.memory<acc>")
        L.append(f"    micro.pipeline stages = {plan['stages']} {{")
        L.append(f"      micro.for %bk = 0 to {K} step {bk} {{")
        for i, w in enumerate(["wg", "wu"]):
            L.append(f"        %{w}_view = micro.tile_view %arg{i + 1}[%bk, %bn] {{shape = [128, {bk}], layout = #micro.layout<col_major>}}")
            L.append(f"        %{w}, %{w}_tok = micro.async_copy %{w}_view {{src_memory = #micro.memory<dram>, dst_memory = #micro.memory<sram>, owner = #micro.owner<dma>, layout = \"swizzled_128b\"}} : tensor<128x{bk}xbf16>")
        L.append(f"        %x_view = micro.tile_view %arg0[0, %bk] {{shape = [{bk}, {mp}], layout = #micro.layout<col_major>}}")
        L.append(f"        %x, %x_tok = micro.async_copy %x_view {{src_memory = #micro.memory<l2>, dst_memory = #micro.memory<sram>, owner = #micro.owner<dma>}} : tensor<{bk}x{mp}xbf16>")
        L.append("        micro.wait %wg_tok, %wu_tok, %x_tok")
        for w in ["wg", "wu"]:
            L.append(f"        micro.mma %{w}, %x, %acc_{w} {{shape = [128, {mp}, {bk}], input = #micro.dtype<bf16>, "
                     f"accumulator = #micro.dtype<f32>, engine = \"tcgen05.cta_group::1\", owner = #micro.owner<matrix_engine>}}")
        L.append("      }")
        L.append("    }")
        L.append(f'    %silu = micro.vector "silu" %acc_wg {{math_mode = "{math_mode}"}}')
        L.append('    %out = micro.vector "mul" %silu, %acc_wu')
        L.append(f"    micro.store %out, %arg3 {{src_memory = #micro.memory<acc>, dst_memory = #micro.memory<dram>}} : tensor<{mp}x128x{y_dtype}>")
        L.append("  }")
    L.append("  micro.yield")
    L.append("}")
    # the argument types with every dimension resolved
    if swiglu:
        shapes = [(M, K, "bf16"), (K, N, "bf16"), (K, N, "bf16"), (M, N, y_dtype)]
    else:
        shapes = [(M, K, "bf16"), (K, N, "bf16"), (M, N, "f32")]
    args = [f"%arg{i}: tensor<{r}x{c}x{d}>" for i, (r, c, d) in enumerate(shapes)]
    header = f"// micro.kernel signature: ({', '.join(args)})  M={M} N={N} K={K}"
    return Lowered(name, header + "\n" + "\n".join(L) + "\n", plan, M, N, K, op.op, y_dtype)
