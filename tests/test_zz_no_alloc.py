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


def test_noalloc_bf16_output_and_limits():
    x, wg, wu = dg.swiglu_inputs(4, 512, 640, 1.0, 0.02, seed=3)
    xd, gd, ud = dev(x), dev(wg), dev(wu)
    ref = llk.fused_swiglu(xd, gd, ud, variant="decode")
    y = torch.empty((4, 640), dtype=torch.bfloat16, device="cuda")
    for _ in range(2):
        assert noalloc(xd, gd, ud, y) == capi.LLK_OK
        torch.cuda.synchronize()
        assert (y.float() - ref.float()).abs().max().item() <= TOL_BF16 * ref.float().abs().max().item()
    # a shape whose workspace exceeds the fixed array is refused, not allocated
    big_n = 128 * 40
    xb = torch.zeros((128, 64), dtype=torch.bfloat16, device="cuda")
    wb = torch.zeros((64, big_n), dtype=torch.bfloat16, device="cuda")
    yb = torch.empty((128, big_n), dtype=torch.bfloat16, device="cuda")
    assert noalloc(xb, wb, wb, yb) == capi.LLK_ERR_NOMEM
    # host buffers would need staging memory: refused
    xh = np.zeros((4, 512), np.uint16)
    assert noalloc(xh, gd, ud, y) == capi.LLK_ERR_ARG
