"""The compiler-side tools on CPU: LLK parsing + the reference verifier
rules, the LLK -> micro lowering, the MachineModel loader/validation, the
micro-perf L0 bound, the schedule DB loader and the CLI entry points."""
import json
import os
import subprocess
import sys

import pytest
import yaml

from dslcompiler_b200 import compiler, microperf, schedule
from tests.conftest import ROOT

MACHINE = os.path.join(ROOT, "dslcompiler_b200", "machines", "b200-sm100a.yaml")

SWIGLU = """
func.func @f(%x: tensor<{M}x{K}xbf16>, %wg: tensor<{K}x{N}xbf16>, %wu: tensor<{K}x{N2}xbf16>, %init: tensor<{M}x{N}xbf16>) -> tensor<{M}x{N}xbf16> {{
  %y = llk.fused_swiglu ins(%x, %wg, %wu : tensor<{M}x{K}xbf16>, tensor<{K}x{N}xbf16>, tensor<{K}x{N2}xbf16>)
      outs(%init : tensor<{M}x{N}xbf16>)
      {{accumulator_type = f32, activation = #llk.activation<silu>, math_mode = #llk.math_mode<bounded_fast>}}
      -> tensor<{M}x{N}xbf16>
  return %y : tensor<{M}x{N}xbf16>
}}
"""

DYN = """
  %y = llk.fused_swiglu ins(%x, %wg, %wu : tensor<?x?xbf16>, tensor<?x?xbf16>, tensor<?x?xbf16>)
      outs(%init : tensor<?x?xbf16>)
      {accumulator_type = f32, activation = #llk.activation<silu>, math_mode = #llk.math_mode<strict>}
      -> tensor<?x?xbf16>
"""

MATMUL = """
  %0 = llk.matmul ins(%a, %b : tensor<4096x4096xbf16>, tensor<4096x4096xbf16>)
      outs(%c : tensor<4096x4096xf32>) {accumulator_type = f32, math_mode = #llk.math_mode<strict>}
      -> tensor<4096x4096xf32>
"""


def test_parse_and_verify_static():
    ops = compiler.parse_llk(SWIGLU.format(M=2048, K=4096, N=11008, N2=11008))
    assert len(ops) == 1 and ops[0].op == "fused_swiglu"
    compiler.verify(ops[0])
    assert compiler.resolve_shape(ops[0]) == (2048, 11008, 4096)
    assert "math_mode" in ops[0].attrs


def test_verifier_rules_match_reference_messages():
    # LLKOps.cpp:69-81: "N dimension mismatch between Wg=... and Wu=..."
    op = compiler.parse_llk(SWIGLU.format(M=8, K=64, N=128, N2=96))[0]
    with pytest.raises(compiler.VerifyError, match="N dimension mismatch between Wg=128 and Wu=96"):
        compiler.verify(op)


def test_dynamic_dims_need_flags():
    op = compiler.parse_llk(DYN)[0]
    compiler.verify(op)
    with pytest.raises(compiler.VerifyError, match="dynamic"):
        compiler.resolve_shape(op)
    assert compiler.resolve_shape(op, 4, 14336, 4096) == (4, 14336, 4096)


@pytest.mark.parametrize("M,variant,candidate", [(2048, "auto", "tc2_kernel"), (64, "tc", "tc_swiglu_kernel"),
                                                  (4, "auto", "decode_kernel")])
def test_lowering_picks_the_dispatched_kernel(M, variant, candidate):
    op = compiler.parse_llk(DYN)[0]
    low = compiler.lower_to_micro(op, M, 14336, 4096, variant)
    assert f'candidate = "{candidate}' in low.text and 'target = "b200-sm100a"' in low.text
    assert low.text.count("{") == low.text.count("}")


def test_l0_bound_counts_work_exactly():
    machine = microperf.load_machine(MACHINE)
    op = compiler.parse_llk(SWIGLU.format(M=2048, K=4096, N=11008, N2=11008))[0]
    rep = microperf.l0_bound(compiler.lower_to_micro(op, 2048, 11008, 4096).text, machine)
    assert rep.total_flops == 4 * 2048 * 4096 * 11008
    assert rep.compulsory_dram_bytes == 2 * 2048 * 4096 + 4 * 4096 * 11008 + 2 * 2048 * 11008
    assert rep.bottleneck == "matrix_engine"
    # 3.694e11 FLOP / (148 SMs x 8192 FLOP/cycle)
    assert abs(rep.compute_cycles - 4 * 2048 * 4096 * 11008 / (148 * 8192)) < 1
    decode = compiler.lower_to_micro(compiler.parse_llk(DYN)[0], 1, 14336, 4096, "decode").text
    rep = microperf.l0_bound(decode, machine)
    assert rep.bottleneck == "dram_bandwidth"


def test_machine_model_validation_rules():
    d = yaml.safe_load(open(MACHINE))
    microperf.validate_machine(d)
    for mutate, msg in [(lambda d: d.pop("schema_version"), "schema_version"),
                        (lambda d: d.update(schema_version=2), "unsupported schema"),
                        (lambda d: d.update(clock_hz=0), "zero clock"),
                        (lambda d: d["memory"]["dram"].update(bandwidth_bytes_per_cycle=0), "bandwidth"),
                        (lambda d: d["compute"]["matrix_engines"][0].update(tile_shapes=[[1, 2]]), "length 3"),
                        (lambda d: d["compute"]["matrix_engines"][0].update(input_dtypes=["f64x"]), "unknown dtype"),
                        (lambda d: d["memory"].pop("acc"), "missing memory")]:
        bad = yaml.safe_load(open(MACHINE))
        mutate(bad)
        with pytest.raises(microperf.MachineModelError, match=msg):
            microperf.validate_machine(bad)


def test_schedule_db_is_target_and_shape_aware(tmp_path):
    p = tmp_path / "db.json"
    json.dump({"version": 1, "entries": [
        {"operation": "fused_swiglu", "target": "x86-avx2", "shape": {"M_bucket": 4, "N": 11008, "K": 4096},
         "dtype": "bf16", "math_mode": "bounded_fast", "schedule": {"BM": 32, "BN": 64, "BK": 64}},
        {"operation": "fused_swiglu", "target": "b200-sm100a", "shape": {"M_bucket": 4, "N": 11008, "K": 4096},
         "dtype": "bf16", "math_mode": "strict", "schedule": {"variant": "tc", "block_m": 256}, "measured_gflops": 5.0},
        {"operation": "fused_swiglu", "target": "b200-sm100a", "shape": {"M_bucket": 4, "N": 11008, "K": 4096},
         "dtype": "bf16", "math_mode": "strict", "schedule": {"variant": "tc", "block_m": 128}, "measured_gflops": 9.0},
        {"operation": "fused_swiglu", "target": "b200-sm100a", "shape": {"M_bucket": 4, "N": 4096, "K": 4096},
         "schedule": {}},
        {"broken": True}]}, open(p, "w"))
    hits = schedule.load(str(p), 4, 11008, 4096)
    assert [h.schedule["block_m"] for h in hits] == [128, 256]  # best measured first, AVX2 entry excluded
    assert schedule.load(str(p), 4, 11008, 2048) == []
    assert len(schedule.load(str(p), 4, 11008, 4096, target="x86-avx2")) == 1
    e = schedule.ScheduleEntry("fused_swiglu", "b200-sm100a", 4, 11008, 4096, schedule={"variant": "tc", "block_m": 256})
    schedule.write_db([e], str(p), merge=True)
    assert len(schedule.read_db(str(p))) == 3  # replaced the two same-key entries, kept the others


def test_shipped_schedule_db_entries_are_installable():
    n = schedule.install(schedule.DEFAULT_DB)
    assert n >= 1


def _run(args):
    return subprocess.run([sys.executable, "-m"] + args, capture_output=True, text=True, cwd=ROOT, timeout=120)


def test_llk_compile_cli(tmp_path):
    f = tmp_path / "in.mlir"
    f.write_text(SWIGLU.format(M=2048, K=4096, N=11008, N2=11008))
    r = _run(["dslcompiler_b200.cli.llk_compile", str(f), "--emit", "micro"])
    assert r.returncode == 0 and r.stdout.strip().endswith("Compilation successful")
    assert "micro.kernel @fused_swiglu_M2048_N11008_K4096" in r.stdout
    bad = tmp_path / "bad.mlir"
    bad.write_text(SWIGLU.format(M=8, K=64, N=128, N2=96))
    r = _run(["dslcompiler_b200.cli.llk_compile", str(bad)])
    assert r.returncode == 1 and "Compilation pipeline failed" in r.stderr
    empty = tmp_path / "e.mlir"
    empty.write_text("module {}")
    r = _run(["dslcompiler_b200.cli.llk_compile", str(empty)])
    assert r.returncode == 1 and "Failed to parse" in r.stderr
    m = tmp_path / "mm.mlir"
    m.write_text(MATMUL)
    out = tmp_path / "mm.micro.mlir"
    r = _run(["dslcompiler_b200.cli.llk_compile", str(m), "--emit", "micro", "-o", str(out)])
    assert r.returncode == 0
    r = _run(["dslcompiler_b200.cli.micro_perf", str(out), "--format", "yaml"])
    rep = yaml.safe_load(r.stdout)
    assert rep["total_flops"] == 2 * 4096 ** 3 and rep["machine"] == "b200-sm100a"


def test_llk_tune_dry_run_writes_schedule_entries(tmp_path):
    out = tmp_path / "tune.json"
    r = _run(["dslcompiler_b200.cli.llk_tune", "--M", "2048", "--N", "11008", "--K", "4096", "--dry-run", "-o", str(out)])
    assert r.returncode == 0 and "Wrote top-3 configs" in r.stdout
    ents = schedule.read_db(str(out))
    assert len(ents) == 3 and all(e.target == "b200-sm100a" and e.M_bucket == 4 for e in ents)


def test_cpu_baseline_bench_has_llk_bench_output():
    r = _run(["oracle.cpu_bench", "--M", "8", "--N", "256", "--K", "256", "--threads", "2",
              "--warmup-ms", "10", "--measure-ms", "50", "--reps", "2"])
    assert r.returncode == 0
    assert r.stdout.splitlines()[0].startswith("LLK Bench")
    assert "Best:" in r.stdout and "GFLOPS" in r.stdout


@pytest.mark.gpu
def test_llk_bench_and_tune_on_gpu(tmp_path):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    r = _run(["dslcompiler_b200.cli.llk_bench", "--M", "512", "--N", "2048", "--K", "1024", "--warmup-ms", "20",
              "--measure-ms", "50", "--reps", "2", "--json"])
    assert r.returncode == 0, r.stderr
    rec = json.loads(r.stdout.strip().splitlines()[-1])
    assert rec["gflops"] > 1000  # a real tensor-core kernel, not a stand-in loop
    out = tmp_path / "t.json"
    r = _run(["dslcompiler_b200.cli.llk_tune", "--M", "8", "--N", "2048", "--K", "1024", "--iters", "3", "-o", str(out)])
    assert r.returncode == 0, r.stderr
    ents = schedule.read_db(str(out))
    assert len(ents) == 3 and all(e.measured_gflops > 0 for e in ents)


def test_micro_perf_clock_override_and_measured(tmp_path):
    """--clock-hz rescales the matrix-engine bound and keeps DRAM's bytes per
    second; --measured-us reports predicted / measured."""
    out = tmp_path / "c4.micro.mlir"
    src = os.path.join(ROOT, "dslcompiler_b200", "examples", "llk", "c4_m1.mlir")
    assert _run(["dslcompiler_b200.cli.llk_compile", src, "--emit", "micro", "-o", str(out)]).returncode == 0
    a = yaml.safe_load(_run(["dslcompiler_b200.cli.micro_perf", str(out)]).stdout)
    b = yaml.safe_load(_run(["dslcompiler_b200.cli.micro_perf", str(out), "--clock-hz", "1e9",
                             "--measured-us", "40"]).stdout)
    assert a["bottleneck"] == "dram_bandwidth" == b["bottleneck"]
    assert abs(a["predicted_ns"] - b["predicted_ns"]) < 0.01 * a["predicted_ns"]  # DRAM time: clock-independent
    assert b["measured_us"] == 40 and abs(b["efficiency"] - b["predicted_ns"] / 40e3) < 1e-3
    c3 = tmp_path / "c3.micro.mlir"
    src = os.path.join(ROOT, "dslcompiler_b200", "examples", "llk", "c3.mlir")
    assert _run(["dslcompiler_b200.cli.llk_compile", src, "--emit", "micro", "-o", str(c3)]).returncode == 0
    f = yaml.safe_load(_run(["dslcompiler_b200.cli.micro_perf", str(c3)]).stdout)
    s = yaml.safe_load(_run(["dslcompiler_b200.cli.micro_perf", str(c3), "--clock-hz", "982500000"]).stdout)
    assert f["bottleneck"] == "matrix_engine" and abs(s["predicted_ns"] / f["predicted_ns"] - 2.0) < 0.01


@pytest.mark.parametrize("M,variant", [(2048, "auto"), (64, "auto"), (1, "auto"), (16, "decode"), (100, "tc")])
def test_lowered_micro_passes_the_mma_verifier(M, variant):
    ops = compiler.parse_llk(SWIGLU.format(M=M, K=4096, N=11008, N2=11008))
    low = compiler.lower_to_micro(ops[0], M, 11008, 4096, variant=variant)
    assert compiler.verify_micro(low.text) == []
    mm = compiler.parse_llk(MATMUL)
    assert compiler.verify_micro(compiler.lower_to_micro(mm[0], 4096, 4096, 4096).text) == []


def test_micro_mma_verifier_messages(tmp_path):
    """The rules and messages of MicroOps.cpp:246-291 for micro.mma."""
    base = ("%a, %t0 = micro.async_copy %v {{}} : tensor<{a}>\n"
            "%b, %t1 = micro.async_copy %w {{}} : tensor<{b}>\n"
            "%c = micro.alloc tensor<{c}> memory = #micro.memory<acc>\n"
            "micro.mma %a, %b, %c {{shape = [{s}], input = #micro.dtype<bf16>, accumulator = #micro.dtype<f32>}}\n")
    ok = dict(a="128x64xbf16", b="64x256xbf16", c="128x256xf32", s="128, 256, 64")
    assert compiler.verify_micro(base.format(**ok)) == []
    cases = {
        "mma shape must have exactly 3 dimensions": dict(ok, s="128, 256"),
        "mma shape dimensions must be positive": dict(ok, s="128, 0, 64"),
        "lhs tile shape must be [M, K]": dict(ok, a="64x128xbf16"),
        "rhs tile shape must be [K, N]": dict(ok, b="256x64xbf16"),
        "accumulator tile shape must be [M, N]": dict(ok, c="128x128xf32"),
        "input dtype must match operand element types": dict(ok, b="64x256xf16"),
        "accumulator dtype must match accumulator element type": dict(ok, c="128x256xbf16"),
        "mma operands and result must be rank-2 tiles": dict(ok, a="128x64x2xbf16"),
    }
    for msg, kw in cases.items():
        errs = compiler.verify_micro(base.format(**kw))
        assert len(errs) == 1 and errs[0].endswith(msg), (msg, errs)
    assert compiler.verify_micro("micro.mma %p, %q, %r {shape = [1, 1, 1]}")[0].endswith(
        "mma operands and result must be tile types")
    bad = tmp_path / "bad.micro.mlir"
    bad.write_text(base.format(**dict(ok, a="64x128xbf16")))
    r = _run(["dslcompiler_b200.cli.micro_perf", str(bad)])
    assert r.returncode == 1 and "lhs tile shape must be [M, K]" in r.stderr


# ------------------------------------------------ micro.kernel dispatch records
GENERIC = """
// the generic form of the same op, split over lines, attributes reordered
%y = "llk.fused_swiglu"(%x, %wg, %wu, %init)
     {math_mode = #llk.math_mode<unsafe_fast>, accumulator_type = f32}
     : (tensor<300x512xbf16>, tensor<512x640xbf16>, tensor<512x640xbf16>,
        tensor<300x640xf32>) -> tensor<300x640xf32>
"""


def test_parse_generic_form_and_math_mode():
    op = compiler.parse_llk(GENERIC)[0]
    compiler.verify(op)
    assert op.operands == ["%x", "%wg", "%wu", "%init"]
    assert compiler.resolve_shape(op) == (300, 640, 512)
    assert compiler.op_math_mode(op) == "unsafe_fast"
    assert compiler.op_math_mode(compiler.parse_llk(SWIGLU.format(M=8, K=64, N=128, N2=128))[0]) == "bounded_fast"


@pytest.mark.parametrize("M,K,N", [(2048, 4096, 11008), (300, 512, 640), (1, 4096, 14336)])
def test_micro_kernel_round_trip_to_dispatch_record(M, K, N):
    from dslcompiler_b200 import micro

    op = compiler.parse_llk(SWIGLU.format(M=M, K=K, N=N, N2=N))[0]
    low = compiler.lower_to_micro(op, M, N, K)
    assert compiler.verify_micro(low.text) == []
    k = micro.parse_micro_kernel(low.text)
    assert (k.M, k.N, k.K, k.op) == (M, N, K, "fused_swiglu")
    assert k.math_mode == "bounded_fast" and k.y_dtype == "bf16"
    assert k.plan == {f: low.plan[f] for f in k.plan}  # every launch-plan field survives the text
    assert k.variant == ("decode" if M <= 16 else "tc")
    # reformatting (line breaks, attribute order) does not change the record
    head, rest = low.text.split("attributes {", 1)
    attrs, body = rest.split("} {", 1)
    swapped = head + "attributes {\n  " + ",\n  ".join(reversed(attrs.split(", "))) + "\n} {" + body
    assert micro.parse_micro_kernel(swapped).plan == k.plan


def test_micro_kernel_refuses_foreign_targets():
    from dslcompiler_b200 import micro

    op = compiler.parse_llk(SWIGLU.format(M=256, K=512, N=384, N2=384))[0]
    text = compiler.lower_to_micro(op, 256, 384, 512).text
    with pytest.raises(micro.MicroError, match="target"):
        micro.parse_micro_kernel(text.replace('"b200-sm100a"', '"avx2"'))
    with pytest.raises(micro.MicroError, match="candidate"):
        micro.parse_micro_kernel(text.replace('candidate = "tc2_kernel<swiglu>"', 'candidate = "avx2_kernel"'))


def test_search_space_emit_parse_and_candidates(tmp_path):
    from dslcompiler_b200 import micro

    for op, M, N, K in [("fused_swiglu", 2048, 11008, 4096), ("fused_swiglu", 4, 1792, 4096),
                        ("matmul", 4096, 4096, 4096)]:
        sp = micro.search_space(op, M, N, K)
        text = micro.emit_search_space(sp)
        assert text.startswith(f"micro.search_space @{op}_M{M}_N{N}_K{K}_space")
        back = micro.parse_search_space(text)
        assert back.params == sp.params and [c[0] for c in back.constraints] == [c[0] for c in sp.constraints]
        cands = micro.candidates(back)
        pair = {"candidate": "tc2_kernel", "BM": 256, "BN": sp.params["BN"][0], "BK": 64, "num_stages": 6,
                "grid": 148, "tail_split": 0, "sched": 1}
        assert cands and micro.legal(sp, pair)[0] == (M > 128)
        # the K-split tail needs the static schedule; pairs need M > 128
        assert not any(c["split_k"] < 0 and c["sched"] == 0 for c in cands)
        if M <= 128:
            assert not any(c["block_m"] == 256 for c in cands)
    f = tmp_path / "in.mlir"
    f.write_text(SWIGLU.format(M=2048, K=4096, N=11008, N2=11008))
    r = _run(["dslcompiler_b200.cli.llk_compile", str(f), "--emit", "micro-search-space"])
    assert r.returncode == 0 and "micro.search_space @fused_swiglu_M2048_N11008_K4096_space" in r.stdout
    space = tmp_path / "space.mlir"
    space.write_text(r.stdout.replace("Compilation successful", ""))
    out = tmp_path / "tune.json"
    r = _run(["dslcompiler_b200.cli.llk_tune", "--M", "2048", "--N", "11008", "--K", "4096", "--dry-run",
              "--search-space", str(space), "-o", str(out)])
    assert r.returncode == 0 and "Wrote top-3 configs" in r.stdout, r.stderr
