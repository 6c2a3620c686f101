"""llk.rope and llk.attention on the GPU (C ABI llk_rope / llk_attention)
against the CPU oracle: the reference's own FP64 references (golden
fixtures) and the f32 restatement of its lowering.

Tolerances: RoPE (f32 in, f32 out, element-wise) max |y - ref| <= 4e-6 *
max |ref| against the f32 lowering (cos / sin of the same f32 angle may
differ by a couple of ulp between libraries); attention max |o - ref| <=
1e-4 * max |ref| (f32 sums over up to a few thousand terms in another order).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import dslcompiler_b200 as llk  # noqa: E402
import oracle  # noqa: E402
from dslcompiler_b200 import capi  # noqa: E402
from dslcompiler_b200 import datagen as dg  # noqa: E402
from tests.conftest import load_golden  # noqa: E402

pytestmark = pytest.mark.gpu

TOL_ROPE = 4e-6
TOL_ATTN = 1e-4


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def rel(a, ref):
    return float(np.abs(np.asarray(a, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ------------------------------------------------------------------- RoPE
def test_rope_golden_fixtures(rope_golden_names):
    for name in rope_golden_names:
        g = load_golden(name)
        y = llk.rope(cuda(g["x"]), cuda(g["pos"]), theta=float(g["theta"])).cpu().numpy()
        ref32 = oracle.rope_f32(g["x"], g["pos"], float(g["theta"]))
        assert rel(y, ref32.astype(np.float64)) <= TOL_ROPE, name
        tol = 2e-6 + 2.0 * float(np.abs(g["pos"]).max()) * 2.0 ** -24
        assert np.abs(y - g["y_ref_f64"]).max() <= (tol + TOL_ROPE) * max(np.abs(g["y_ref_f64"]).max(), 1.0), name


@pytest.mark.parametrize("B,H,L,D,theta", [(2, 32, 2048, 128, 10000.0), (1, 8, 333, 64, 500000.0), (3, 2, 17, 6, 10.0),
                                           (1, 1, 5, 2, 10000.0), (4, 4, 64, 256, 10000.0), (1, 2, 40, 1026, 1e6)])
def test_rope_shapes_vs_lowering(B, H, L, D, theta):
    x = dg.normal_f32(B * 131 + D, (B, H, L, D))
    pos = np.random.default_rng(L).integers(0, 4096, L).astype(np.int64)
    y = llk.rope(cuda(x), cuda(pos), theta=theta).cpu().numpy()
    assert rel(y, oracle.rope_f32(x, pos, theta).astype(np.float64)) <= TOL_ROPE


def test_rope_in_place_host_arrays_and_fast_math():
    x = dg.normal_f32(5, (2, 4, 64, 128))
    pos = np.arange(64, dtype=np.int64)
    ref = oracle.rope_f32(x, pos, 10000.0).astype(np.float64)
    # host arrays: staged through the GPU, result back on the host
    y = llk.rope(x, pos)
    assert isinstance(y, np.ndarray) and rel(y, ref) <= TOL_ROPE
    # in place on the device
    xd = cuda(x)
    out = llk.rope(xd, cuda(pos), out=xd)
    assert out is xd and rel(xd.cpu().numpy(), ref) <= TOL_ROPE
    # the fast trig path: small angles only (__sinf / __cosf lose accuracy far from 0)
    yf = llk.rope(cuda(x), cuda(pos), math_mode="bounded_fast").cpu().numpy()
    assert rel(yf, ref) <= 1e-3


def test_rope_argument_errors():
    x = torch.zeros((1, 1, 4, 5), device="cuda")
    with pytest.raises(llk.LLKError) as e:  # odd D
        llk.rope(x, torch.zeros(4, dtype=torch.int64, device="cuda"))
    assert e.value.status == capi.LLK_ERR_SHAPE


# -------------------------------------------------------------- attention
def test_attention_golden_fixtures(attention_golden_names):
    for name in attention_golden_names:
        g = load_golden(name)
        o = llk.attention(cuda(g["q"]), cuda(g["k"]), cuda(g["v"]), scale=float(g["scale"]),
                          causal=bool(g["causal"])).cpu().numpy()
        assert rel(o, g["o_ref_f64"]) <= TOL_ATTN, name


@pytest.mark.parametrize("B,H,Lq,Lk,D,causal", [(1, 1, 128, 128, 128, True), (2, 8, 256, 256, 64, True),
                                                (1, 4, 100, 300, 64, False), (1, 2, 65, 130, 128, True),
                                                (2, 2, 300, 77, 32, True), (1, 1, 7, 9, 3, False),
                                                (1, 2, 50, 60, 80, False), (1, 1, 40, 40, 200, True),
                                                (1, 2, 1024, 1024, 128, True)])
def test_attention_shapes_vs_lowering(B, H, Lq, Lk, D, causal):
    q = dg.normal_f32(Lq + D, (B, H, Lq, D))
    k = dg.normal_f32(Lk + D + 1, (B, H, Lk, D))
    v = dg.normal_f32(Lk + D + 2, (B, H, Lk, D))
    scale = 1.0 / np.sqrt(D)
    o = llk.attention(cuda(q), cuda(k), cuda(v), scale=scale, causal=causal).cpu().numpy()
    ref = oracle.attention_f32(q, k, v, scale, causal).astype(np.float64)
    assert rel(o, ref) <= TOL_ATTN
    assert np.isfinite(o).all()


def test_attention_init_host_arrays_empty_keys_and_fast_math():
    B, H, Lq, Lk, D = 1, 2, 96, 96, 64
    q, k, v = (dg.normal_f32(s, (B, H, L, D)) for s, L in ((1, Lq), (2, Lk), (3, Lk)))
    init = dg.normal_f32(4, (B, H, Lq, D))
    ref = oracle.attention_f32(q, k, v, 0.125, True, init=init).astype(np.float64)
    # destination passing: the result is added to `out` (the op's init)
    o = llk.attention(cuda(q), cuda(k), cuda(v), scale=0.125, causal=True, out=cuda(init)).cpu().numpy()
    assert rel(o, ref) <= TOL_ATTN
    # host arrays
    oh = llk.attention(q, k, v, scale=0.125, causal=True, out=init.copy())
    assert isinstance(oh, np.ndarray) and rel(oh, ref) <= TOL_ATTN
    # no keys: O keeps its initial values
    empty = np.zeros((B, H, 0, D), np.float32)
    oe = llk.attention(cuda(q), cuda(empty), cuda(empty), out=cuda(init)).cpu().numpy()
    assert np.array_equal(oe, init)
    # fast exp
    of = llk.attention(cuda(q), cuda(k), cuda(v), scale=0.125, causal=True, out=cuda(init),
                       math_mode="bounded_fast").cpu().numpy()
    assert rel(of, ref) <= 1e-3
    # O may not alias an input
    qd = cuda(q)
    with pytest.raises(llk.LLKError) as e:
        llk.attention(qd, cuda(k), cuda(v), out=qd)
    assert e.value.status == capi.LLK_ERR_ARG
