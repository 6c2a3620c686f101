"""A micro.kernel as a drop-in dispatch record, and the math_mode keys.

llk-compile --emit micro lowers an LLK op to the micro.kernel of the kernel
and launch plan that serve it; run_micro parses that text back, installs the
plan for the op's KernelKey through the C ABI and launches the named kernel.
Checked against the CPU oracle for the configurations' shapes.  The math
mode of the op (strict / bounded_fast) selects different kernel
instantiations under different keys; both must match the oracle.
"""
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import dslcompiler_b200 as llk  # noqa: E402
import oracle  # noqa: E402
from dslcompiler_b200 import capi, compiler, micro  # noqa: E402
from dslcompiler_b200 import datagen as dg  # noqa: E402
from tests.conftest import ROOT  # noqa: E402

pytestmark = pytest.mark.gpu

TOL_F32 = 2e-3
TOL_BF16 = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


def as_f64(t):
    if t.dtype == torch.bfloat16:
        return dg.bf16_bits_to_f32(t.cpu().view(torch.int16).numpy().view(np.uint16)).astype(np.float64)
    return t.cpu().numpy().astype(np.float64)


def emit_micro(example, *extra):
    """llk-compile --emit micro on one of the shipped example ops."""
    path = f"{ROOT}/dslcompiler_b200/examples/llk/{example}.mlir"
    r = subprocess.run([sys.executable, "-m", "dslcompiler_b200.cli.llk_compile", path, "--emit", "micro", *extra],
                       capture_output=True, text=True, cwd=ROOT, timeout=120)
    assert r.returncode == 0, r.stderr
    return r.stdout.replace("Compilation successful", "")


@pytest.mark.parametrize("example,cfg", [("c3", "c3"), ("c4_m1", "c4_m1"), ("c4_m16", "c4_m16")])
def test_run_micro_from_llk_compile_matches_oracle(example, cfg):
    text = emit_micro(example)
    k = micro.parse_micro_kernel(text)
    c = dg.CONFIGS[cfg]
    assert (k.M, k.K, k.N) == (c["M"], c["K"], c["N"])
    x, wg, wu = dg.config_inputs(cfg)
    y = micro.run_micro(text, dev(x), dev(wg), dev(wu))
    torch.cuda.synchronize()
    llk.synchronize(0)
    assert y.dtype == torch.bfloat16 and tuple(y.shape) == (k.M, k.N)
    # the plan the micro.kernel names is the one installed for the key
    assert micro.kernel_key(k).plan(k.M) == k.plan
    rng = np.random.default_rng(3)
    rows = np.concatenate([rng.integers(0, k.M, 4000), np.full(k.N, k.M - 1)])
    cols = np.concatenate([rng.integers(0, k.N, 4000), np.arange(k.N)])
    ref = oracle.swiglu_fp64_points(x, wg, wu, rows, cols)
    yy = as_f64(y)
    assert float(np.abs(yy[rows, cols] - ref).max() / np.abs(ref).max()) <= TOL_BF16


def test_run_micro_matmul_and_edited_plan():
    """A micro.kernel whose plan attributes were edited (another tail split,
    fewer pairs) dispatches exactly that plan; the result still matches."""
    M = N = K = 1024
    op = compiler.parse_llk(f"""
      %c = llk.matmul ins(%a, %b : tensor<{M}x{K}xbf16>, tensor<{K}x{N}xbf16>)
          outs(%i : tensor<{M}x{N}xf32>) {{accumulator_type = f32, math_mode = #llk.math_mode<strict>}}
          -> tensor<{M}x{N}xf32>""")[0]
    text = compiler.lower_to_micro(op, M, N, K).text
    a, b = dg.matmul_inputs(M, K, N, seed=11)
    ref = oracle.matmul(a, b).astype(np.float64)
    base = micro.parse_micro_kernel(text)
    try:
        for edit in ({}, {"split_k": -3, "grid": 14, "sched": 1}, {"split_k": 2, "grid": 10, "sched": 0}):
            t = text
            for f, v in edit.items():
                t = t.replace(f"{f} = {base.plan[f]},", f"{f} = {v},", 1)
            k = micro.parse_micro_kernel(t)
            assert all(k.plan[f] == v for f, v in edit.items())
            c = micro.run_micro(t, dev(a), dev(b))
            torch.cuda.synchronize()
            llk.synchronize(0)
            assert micro.kernel_key(k).plan(M) == k.plan
            err = float(np.abs(as_f64(c) - ref).max() / np.abs(ref).max())
            assert err <= 1e-5, (edit, err)
    finally:
        micro.install(base)


@pytest.mark.parametrize("M,K,N,variant", [(512, 1024, 1000, "tc"), (2048, 1024, 1408, "tc"), (96, 512, 384, "tc"),
                                           (4, 4096, 1792, "decode"), (3, 256, 200, "simt")])
def test_math_modes_select_different_kernels_and_match_oracle(M, K, N, variant):
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0, 0.05, seed=M + N)
    ref = oracle.swiglu_fused(x, wg, wu, "f32").astype(np.float64)
    xd, gd, ud = dev(x), dev(wg), dev(wu)
    ys = {}
    for mode in ("strict", "bounded_fast"):
        ys[mode] = llk.fused_swiglu(xd, gd, ud, out_dtype="f32", variant=variant, math_mode=mode)
    torch.cuda.synchronize()
    llk.synchronize(0)
    for mode, y in ys.items():
        assert float(np.abs(as_f64(y) - ref).max() / np.abs(ref).max()) <= TOL_F32, mode
    # the two epilogues are different code: some elements differ in the last bits
    assert not torch.equal(ys["strict"], ys["bounded_fast"])
    # and the strict one is the closer to the oracle's strict f32 epilogue
    d_strict = float(np.abs(as_f64(ys["strict"]) - ref).max())
    d_fast = float(np.abs(as_f64(ys["bounded_fast"]) - ref).max())
    assert d_strict <= d_fast
    if variant != "simt":
        # both keys are in the plan cache, filed under their math mode
        for mode in ("strict", "bounded_fast"):
            key = llk.KernelKey(N=N, K=K, M_bucket=llk.classify_m(M), output_type=capi.LLK_DTYPE_FP32,
                                thread_count=capi.VARIANTS[variant], math_mode=capi.MATH_MODES[mode])
            assert key.find() is not None, mode


def test_strict_epilogue_reciprocal_equals_ieee_division():
    """The strict epilogue's own reciprocal (Markstein's method) gives the
    correctly rounded 1/b, i.e. the IEEE division 1.0f / b, for every finite
    float b >= 1 (the range of 1 + e^-g): all 2^30 of them, on the GPU."""
    import ctypes

    n = ctypes.c_uint64(123)
    assert capi.lib().llk_diag_reciprocal_check(0, 0x3F800000, 0x7F800000, ctypes.byref(n)) == capi.LLK_OK
    assert n.value == 0
