"""llk_swiglu_decode_noalloc: the decode SwiGLU for callers that cannot
allocate device memory (their GPU memory belongs to another allocator, or
cudaMalloc's host round trips and implicit synchronisation are not allowed
on their path).  Its split-K scratch is a fixed device array inside the
library instead of a cudaMalloc'd workspace.

Called through the C ABI and checked against the existing entry point
(llk_swiglu_ex, decode variant) on two calls in a row -- the second call
finds the first call's leftovers in the shared array.  This file is named so
pytest collects it last; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import dslcompiler_b200 as llk  # noqa: E402
from dslcompiler_b200 import capi  # noqa: E402
from dslcompiler_b200 import datagen as dg  # noqa: E402

pytestmark = pytest.mark.gpu

TOL_F32 = 2e-3  # f32 Y: max|y - ref| <= 2e-3 * max|ref|, as in the other GPU tests
TOL_BF16 = 1e-2


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


def noalloc(x, wg, wu, y, status=None):
    tx, tg, tu, ty = (llk.tensor2d(t) for t in (x, wg, wu, y))
    g = capi.GpuContext()
    g.device = torch.cuda.current_device()
    g.stream = torch.cuda.current_stream().cuda_stream
    g.y_dtype = capi.LLK_DTYPE_FP32 if y.dtype == torch.float32 else capi.LLK_DTYPE_BF16
    g.variant = 0
    return capi.lib().llk_swiglu_decode_noalloc(ctypes.byref(tx), ctypes.byref(tg), ctypes.byref(tu),
                                                ctypes.byref(ty), status.data_ptr() if status is not None else None,
                                                ctypes.byref(g))


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


@pytest.mark.parametrize("M,K,N", [(16, 4096, 14336), (1, 4096, 14336), (5, 1024, 1000)])
def test_noalloc_matches_existing_entry_point_twice(M, K, N):
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0, 0.02, seed=100 + M)
    xd, gd, ud = dev(x), dev(wg), dev(wu)
    ref = llk.fused_swiglu(xd, gd, ud, out_dtype="f32", variant="decode")
    torch.cuda.synchronize()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    scale = ref.abs().max().item()
    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        assert noalloc(xd, gd, ud, y, status) == capi.LLK_OK
        torch.cuda.synchronize()
        assert status.item() == 0
        assert not torch.isnan(y).any()
        assert (y - ref).abs().max().item() <= TOL_F32 * scale


def test_noalloc_stream_k_shape_vs_oracle():
    """A shape whose column tiles are shared by several CTAs (8 tiles x 16
    k-blocks over every SM), so the partial-sum slots in the fixed array are
    used: checked against the CPU oracle directly, twice."""
    import oracle

    M, K, N = 5, 1024, 1000
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0, 0.02, seed=77)
    ref = oracle.swiglu_fused(x, wg, wu, "f32").astype(np.float64)
    xd, gd, ud = dev(x), dev(wg), dev(wu)
    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        assert noalloc(xd, gd, ud, y) == capi.LLK_OK
        torch.cuda.synchronize()
        err = np.abs(y.cpu().numpy().astype(np.float64) - ref).max() / np.abs(ref).max()
        assert err <= TOL_F32


def test_noalloc_bf16_output_and_limits():
    x, wg, wu = dg.swiglu_inputs(4, 512, 640, 1.0, 0.02, seed=3)
    xd, gd, ud = dev(x), dev(wg), dev(wu)
    ref = llk.fused_swiglu(xd, gd, ud, variant="decode")
    y = torch.empty((4, 640), dtype=torch.bfloat16, device="cuda")
    for _ in range(2):
        assert noalloc(xd, gd, ud, y) == capi.LLK_OK
        torch.cuda.synchronize()
        assert (y.float() - ref.float()).abs().max().item() <= TOL_BF16 * ref.float().abs().max().item()
    # wider than the fixed array's counters: refused with LLK_ERR_NOMEM before
    # any buffer is touched (the descriptors claim more columns than exist)
    tx, ty = llk.tensor2d(xd), llk.tensor2d(y)
    big = capi.LLK_DECODE_NOALLOC_MAX_N + 128
    tw = capi.Tensor2D(gd.data_ptr(), 512, big, big, 1)
    ty = capi.Tensor2D(y.data_ptr(), 4, big, big, 1)
    g = capi.GpuContext()
    g.device = torch.cuda.current_device()
    g.stream = torch.cuda.current_stream().cuda_stream
    rc = capi.lib().llk_swiglu_decode_noalloc(ctypes.byref(tx), ctypes.byref(tw), ctypes.byref(tw),
                                              ctypes.byref(ty), None, ctypes.byref(g))
    assert rc == capi.LLK_ERR_NOMEM
    # host buffers would need staging memory: refused
    xh = np.zeros((4, 512), np.uint16)
    assert noalloc(xh, gd, ud, y) == capi.LLK_ERR_ARG
    # a Y start not aligned to its element size: refused, not faulted
    raw = torch.empty((4 * 640 * 2 + 16,), dtype=torch.uint8, device="cuda")
    ty_bad = capi.Tensor2D(raw.data_ptr() + 1, 4, 640, 640, 1)
    g.y_dtype = capi.LLK_DTYPE_BF16
    tg, tu = llk.tensor2d(gd), llk.tensor2d(ud)
    rc = capi.lib().llk_swiglu_decode_noalloc(ctypes.byref(tx), ctypes.byref(tg), ctypes.byref(tu),
                                              ctypes.byref(ty_bad), None, ctypes.byref(g))
    assert rc == capi.LLK_ERR_ALIGN


def test_noalloc_leaves_current_device_alone():
    x, wg, wu = dg.swiglu_inputs(2, 256, 256, 1.0, 0.02, seed=9)
    xd, gd, ud = dev(x), dev(wg), dev(wu)
    y = torch.empty((2, 256), dtype=torch.float32, device="cuda")
    before = torch.cuda.current_device()
    assert noalloc(xd, gd, ud, y) == capi.LLK_OK
    torch.cuda.synchronize()
    assert torch.cuda.current_device() == before
