"""Parity of the CUDA path (called through the C ABI) with the CPU oracle.

Tolerances (from the benchmark's correctness bar):
  * f32 Y:  max|y - ref| <= 2e-3 * max|ref|
  * bf16 Y: max|y - ref| <= 1e-2 * max|ref|
ref is the FP64 SwiGLU of the same bf16 inputs (the reference's
swiglu_reference_fp64 semantics) or the fused f32 oracle.
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import dslcompiler_b200 as llk  # noqa: E402
import oracle  # noqa: E402
from dslcompiler_b200 import capi  # noqa: E402
from dslcompiler_b200 import datagen as dg  # noqa: E402
from tests.conftest import load_golden  # noqa: E402

pytestmark = pytest.mark.gpu

TOL_F32 = 2e-3
TOL_BF16 = 1e-2


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


def host(t):
    if t.dtype == torch.bfloat16:
        return dg.bf16_bits_to_f32(t.cpu().view(torch.int16).numpy().view(np.uint16)).astype(np.float64)
    return t.cpu().numpy().astype(np.float64)


def rel_err(y, ref):
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    llk.synchronize(0)
    yield
    llk.synchronize(0)


# ----------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("variant", ["auto", "simt"])
def test_golden_fixtures(golden_names, out, variant):
    for name in golden_names:
        g = load_golden(name)
        y = llk.fused_swiglu(dev(g["x"]), dev(g["wg"]), dev(g["wu"]), out_dtype=out, variant=variant)
        torch.cuda.synchronize()
        llk.synchronize(0)
        err = rel_err(host(y), g["y_ref_f64"])
        assert err <= (TOL_F32 if out == "f32" else TOL_BF16), (name, err)


def test_config1_tc_f32_full():
    g = load_golden("config1_64_512_256")
    y = llk.fused_swiglu(dev(g["x"]), dev(g["wg"]), dev(g["wu"]), out_dtype="f32", variant="tc")
    torch.cuda.synchronize()
    ref = oracle.swiglu_fused(g["x"], g["wg"], g["wu"], "f32").astype(np.float64)
    err = rel_err(host(y), ref)
    assert err <= TOL_F32
    assert err < 1e-5  # f32 accumulation of the same products: only summation order differs


def test_tc_requires_tma_alignment():
    g = load_golden("avx2_32_256_127")  # K = 127: X row pitch 254 B is not a multiple of 16
    with pytest.raises(llk.LLKError) as e:
        llk.fused_swiglu(dev(g["x"]), dev(g["wg"]), dev(g["wu"]), variant="tc")
    assert e.value.status == capi.LLK_ERR_UNSUPPORTED


# ----------------------------------------------------- shapes and edge cases
@pytest.mark.parametrize("M,K,N", [(1, 64, 128), (128, 64, 128), (129, 128, 256), (300, 200, 520), (64, 4096, 136),
                                   (256, 1024, 1024), (16, 512, 24), (2, 8, 8)])
@pytest.mark.parametrize("variant", ["tc", "auto"])
def test_swiglu_shapes_vs_oracle(M, K, N, variant):
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0 / math.sqrt(K), 1.0, seed=M + K + N)
    y = llk.fused_swiglu(dev(x), dev(wg), dev(wu), out_dtype="f32", variant=variant)
    torch.cuda.synchronize()
    llk.synchronize(0)
    ref = oracle.swiglu_fused(x, wg, wu, "f32").astype(np.float64)
    assert rel_err(host(y), ref) <= TOL_F32


def test_bf16_output_rounding_matches_oracle():
    x, wg, wu = dg.swiglu_inputs(200, 256, 384, 0.0625, 0.0625, seed=11)
    y = llk.fused_swiglu(dev(x), dev(wg), dev(wu), out_dtype="bf16", variant="tc")
    torch.cuda.synchronize()
    ref = oracle.swiglu_fused(x, wg, wu, "bf16")
    yb = y.cpu().view(torch.int16).numpy().view(np.uint16)
    # Same f32 products, different summation order: almost all elements round
    # to the same bf16; the rest differ by about one bf16 ulp (more only where
    # the sum cancels to near zero).
    assert (yb == ref).mean() > 0.99
    yv, rv = dg.bf16_bits_to_f32(yb).astype(np.float64), dg.bf16_bits_to_f32(ref).astype(np.float64)
    assert np.all(np.abs(yv - rv) <= 2.0 ** -7 * np.abs(rv) + 1e-5 * np.abs(rv).max())


def test_edge_known_answers_on_gpu():
    # edge_cases.cpp:47-150 on the device (values exactly representable in bf16)
    def run(x, wg, wu):
        y = llk.fused_swiglu(dev(dg.f32_to_bf16_bits(np.array(x, np.float32))),
                             dev(dg.f32_to_bf16_bits(np.array(wg, np.float32))),
                             dev(dg.f32_to_bf16_bits(np.array(wu, np.float32))), out_dtype="f32")
        torch.cuda.synchronize()
        return host(y)
    y = run([[2.0]], [[0.5]], [[0.25]])
    assert abs(y[0, 0] - (1.0 / (1.0 + math.exp(-1.0))) * 0.5) < 1e-5
    y = run([[10.0, -10.0]], np.eye(2), np.eye(2))
    assert y[0, 0] > 90.0 and abs(y[0, 1]) < 1.0
    y = run(np.zeros((2, 4)), np.zeros((4, 3)), np.zeros((4, 3)))
    assert np.all(y == 0.0)
    y = run(np.ones((3, 1)), np.full((1, 2), 0.5), np.full((1, 2), 0.25))
    assert np.all(y == y[0, 0])


def test_empty_and_k0():
    x = torch.zeros((0, 64), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((64, 128), dtype=torch.bfloat16, device="cuda")
    y = llk.fused_swiglu(x, w, w)
    assert y.shape == (0, 128)
    x0 = torch.zeros((4, 0), dtype=torch.bfloat16, device="cuda")
    w0 = torch.zeros((0, 16), dtype=torch.bfloat16, device="cuda")
    y = llk.fused_swiglu(x0, w0, w0, out_dtype="f32")
    torch.cuda.synchronize()
    assert torch.all(y == 0)


def test_strided_and_unaligned_views():
    x, wg, wu = dg.swiglu_inputs(70, 96, 200, 0.1, 0.1, seed=5)
    ref = oracle.swiglu_fused(x, wg, wu, "f32").astype(np.float64)
    # padded row pitch (TMA-describable)
    big = torch.zeros((70, 104), dtype=torch.bfloat16, device="cuda")
    big[:, :96] = dev(x)
    y = llk.fused_swiglu(big[:, :96], dev(wg), dev(wu), out_dtype="f32")
    torch.cuda.synchronize()
    assert rel_err(host(y), ref) <= TOL_F32
    # pointer offset by one element (not 16-byte aligned) -> SIMT kernel
    big2 = torch.zeros((70, 97), dtype=torch.bfloat16, device="cuda")
    big2[:, 1:] = dev(x)
    y = llk.fused_swiglu(big2[:, 1:], dev(wg), dev(wu), out_dtype="f32")
    torch.cuda.synchronize()
    assert rel_err(host(y), ref) <= TOL_F32
    # transposed weight view (inner stride != 1) -> SIMT kernel
    wgt = dev(np.ascontiguousarray(wg.T)).t()
    y = llk.fused_swiglu(dev(x), wgt, dev(wu), out_dtype="f32")
    torch.cuda.synchronize()
    assert rel_err(host(y), ref) <= TOL_F32


# ------------------------------------------------------------- host buffers
def bf16_close(y_bits, y_dev, tol=TOL_BF16):
    """bf16 host bit patterns vs a bf16 device tensor: max |a - b| <= tol * max |b|."""
    a = dg.bf16_bits_to_f32(np.ascontiguousarray(y_bits)).astype(np.float64)
    b = y_dev.float().cpu().numpy().astype(np.float64)
    return float(np.abs(a - b).max()) <= tol * float(np.abs(b).max())


def test_host_buffers_through_c_abi():
    g = load_golden("config1_64_512_256")
    y = np.zeros((64, 512), np.uint16)
    st = llk.swiglu_c_abi(g["x"], g["wg"], g["wu"], y)
    assert st == capi.LLK_OK
    assert rel_err(dg.bf16_bits_to_f32(y).astype(np.float64), g["y_ref_f64"]) <= TOL_BF16
    yd = llk.fused_swiglu(dev(g["x"]), dev(g["wg"]), dev(g["wu"]))
    torch.cuda.synchronize()
    assert np.array_equal(y, yd.cpu().view(torch.int16).numpy().view(np.uint16))


@pytest.mark.parametrize("M,K,N", [(300, 512, 1000), (2048, 256, 11008), (20, 64, 4096)])
def test_host_buffers_pipelined_chunks_match_device_path(M, K, N):
    """Host X/Wg/Wu/Y: weights and Y travel in column chunks overlapped with
    the kernel; the result equals the device-buffer call."""
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0, 0.02, seed=N)
    y = np.full((M, N + 3), 0xFFFF, np.uint16)[:, :N]  # strided host output
    st = llk.swiglu_c_abi(x, wg, wu, y)
    assert st == capi.LLK_OK
    yd = llk.fused_swiglu(dev(x), dev(wg), dev(wu), variant="tc")
    torch.cuda.synchronize()
    # a chunk is a smaller problem whose leftover tiles may be split along K
    # (another summation order): equal within the bf16 tolerance
    assert bf16_close(y, yd)


@pytest.mark.parametrize("M,K,N", [(1000, 512, 640), (2048, 256, 1408)])
def test_packed_weights_host_rows_pipelined(M, K, N):
    """Packed (device) weights with host X/Y: row blocks of X travel in,
    blocks of Y travel out, overlapped with the kernel."""
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0, 0.02, seed=M)
    pw = llk.PackedWeights(dev(wg), dev(wu))
    y = pw(x)
    yd = pw(dev(x))
    torch.cuda.synchronize()
    assert bf16_close(y, yd)  # row blocks: smaller problems, maybe another tail split
    pw.close()


def test_memref_kernelfn_shim():
    import ctypes
    g = load_golden("small_4_8_16")
    x, wg, wu = (np.ascontiguousarray(g[k]) for k in ("x", "wg", "wu"))
    y = np.zeros((4, 8), np.uint16)

    def mr(a):
        return capi.MemRef2D(a.ctypes.data, a.ctypes.data, 0, a.shape[0], a.shape[1], a.shape[1], 1)
    ms = [mr(x), mr(wg), mr(wu), mr(y), mr(y)]
    L = capi.lib()
    L.llk_swiglu_memref(*[ctypes.byref(m) for m in ms])
    assert L.llk_last_status() == capi.LLK_OK
    assert rel_err(dg.bf16_bits_to_f32(y).astype(np.float64), g["y_ref_f64"]) <= TOL_BF16


def test_packed_weights_match_unpacked():
    x, wg, wu = dg.swiglu_inputs(256, 512, 640, 0.05, 0.05, seed=21)
    pw = llk.PackedWeights(wg, wu)  # packed from host buffers
    assert pw.K == 512 and pw.N == 640
    y1 = pw(dev(x))
    y2 = llk.fused_swiglu(dev(x), dev(wg), dev(wu))
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    # host X / host Y through the packed weights
    yh = pw(x)
    assert bf16_close(yh, y2)
    # repack with new weights
    _, wg2, wu2 = dg.swiglu_inputs(256, 512, 640, 0.05, 0.05, seed=22)
    pw.repack(wg2, wu2)
    y3 = pw(dev(x))
    y4 = llk.fused_swiglu(dev(x), dev(wg2), dev(wu2))
    torch.cuda.synchronize()
    assert torch.equal(y3, y4)
    pw.close()


# ------------------------------------------------------------------ matmul
@pytest.mark.parametrize("M,K,N", [(128, 64, 256), (300, 200, 520), (1, 64, 64), (513, 1024, 768)])
def test_matmul_vs_oracle(M, K, N):
    a, b = dg.matmul_inputs(M, K, N, seed=M + N)
    c = llk.matmul(dev(a), dev(b))
    torch.cuda.synchronize()
    ref = oracle.matmul(a, b).astype(np.float64)
    assert rel_err(host(c), ref) <= TOL_F32
    assert rel_err(host(c), ref) < 1e-5


def test_matmul_accumulate():
    a, b = dg.matmul_inputs(200, 128, 300, seed=8)
    c0 = dg.normal_f32(9, (200, 300))
    c = torch.from_numpy(c0.copy()).cuda()
    llk.matmul(dev(a), dev(b), c, accumulate=True)
    torch.cuda.synchronize()
    ref = oracle.matmul(a, b, c0).astype(np.float64)
    assert rel_err(host(c), ref) < 1e-5


def test_matmul_config2_full():
    a, b = dg.config_inputs("c2")
    c = llk.matmul(dev(a), dev(b))
    torch.cuda.synchronize()
    ref = oracle.port_matmul(a, b).astype(np.float64)
    assert rel_err(host(c), ref) <= TOL_F32


# ------------------------------------------------------ full-size configs
def test_config3_sampled_fp64_and_torch():
    x, wg, wu = dg.config_inputs("c3")
    xd, gd, ud = dev(x), dev(wg), dev(wu)
    y = llk.fused_swiglu(xd, gd, ud)
    torch.cuda.synchronize()
    llk.synchronize(0)
    rng = np.random.default_rng(0)
    rows = np.concatenate([rng.integers(0, 2048, 4096), np.arange(2048)])
    cols = np.concatenate([rng.integers(0, 11008, 4096), rng.integers(0, 11008, 2048)])
    ref = oracle.swiglu_fp64_points(x, wg, wu, rows, cols)
    yy = host(y)
    err = float(np.abs(yy[rows, cols] - ref).max() / np.abs(ref).max())
    assert err <= TOL_BF16
    # full-tensor check against an fp32 torch restatement (size-independent bar)
    g = xd.float() @ gd.float()
    u = xd.float() @ ud.float()
    tref = (g / (1 + torch.exp(-g)) * u).double()
    terr = float((y.double() - tref).abs().max() / tref.abs().max())
    assert terr <= TOL_BF16
    assert not torch.isnan(y).any()


def _device_normal_bf16(shape, std, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda", dtype=torch.float32) * std).to(torch.bfloat16)


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def test_config5_sampled_fp64_rows_and_torch():
    """Config 5 (X[8192,8192], Wg/Wu[8192,28672], Y bf16; 1.6 GB of inputs,
    drawn on the device): 4096 random points plus two whole rows in FP64, 16
    whole rows against the fused f32 port, and the full tensor against an
    fp32 torch restatement, column block by column block."""
    M, K, N = 8192, 8192, 28672
    xd = _device_normal_bf16((M, K), 1.0, 501)
    gd = _device_normal_bf16((K, N), 0.015, 502)
    ud = _device_normal_bf16((K, N), 0.015, 503)
    y = llk.fused_swiglu(xd, gd, ud)
    torch.cuda.synchronize()
    llk.synchronize(0)
    assert not torch.isnan(y).any()
    x, wg, wu = _bits(xd), _bits(gd), _bits(ud)
    yy = host(y)
    rng = np.random.default_rng(5)
    rows = np.concatenate([rng.integers(0, M, 4096), np.full(N, 0), np.full(N, M - 1)])
    cols = np.concatenate([rng.integers(0, N, 4096), np.arange(N), np.arange(N)])
    ref = oracle.swiglu_fp64_points(x, wg, wu, rows, cols)
    assert float(np.abs(yy[rows, cols] - ref).max() / np.abs(ref).max()) <= TOL_BF16
    sample = np.sort(rng.choice(M, 16, replace=False))
    pref = oracle.port_swiglu(x[sample], wg, wu, "f32").astype(np.float64)
    assert rel_err(yy[sample], pref) <= TOL_BF16
    terr, tmax = 0.0, 0.0
    xf = xd.float()
    for c0 in range(0, N, 4096):
        g = xf @ gd[:, c0:c0 + 4096].float()
        u = xf @ ud[:, c0:c0 + 4096].float()
        t = g / (1 + torch.exp(-g)) * u
        terr = max(terr, float((y[:, c0:c0 + 4096].float() - t).abs().max()))
        tmax = max(tmax, float(t.abs().max()))
    assert terr / tmax <= TOL_BF16


@pytest.mark.parametrize("cfg", ["c4_m1", "c4_m4", "c4_m16"])
@pytest.mark.parametrize("variant", ["auto", "tc"])
def test_config4_decode_shapes(cfg, variant):
    x, wg, wu = dg.config_inputs(cfg)
    y = llk.fused_swiglu(dev(x), dev(wg), dev(wu), out_dtype="f32", variant=variant)
    torch.cuda.synchronize()
    llk.synchronize(0)
    ref = oracle.port_swiglu(x, wg, wu, "f32").astype(np.float64)
    assert rel_err(host(y), ref) <= TOL_F32


def test_determinism_two_calls():
    x, wg, wu = dg.swiglu_inputs(512, 1024, 2048, 1.0, 0.02, seed=77)
    a = llk.fused_swiglu(dev(x), dev(wg), dev(wu))
    b = llk.fused_swiglu(dev(x), dev(wg), dev(wu))
    torch.cuda.synchronize()
    assert torch.equal(a, b)


# ---------------------------------------------------------- failure paths
def test_bounded_wait_reports_timeout_and_context_survives():
    st = capi.lib().llk_diag_timeout_probe(0, 2_000_000)  # 2 ms limit, barrier never arrives
    assert st == capi.LLK_ERR_TIMEOUT
    # the status word was cleared and the context still runs kernels
    llk.synchronize(0)
    g = load_golden("small_4_8_16")
    y = llk.fused_swiglu(dev(g["x"]), dev(g["wg"]), dev(g["wu"]), out_dtype="f32")
    torch.cuda.synchronize()
    assert rel_err(host(y), g["y_ref_f64"]) <= TOL_F32


def test_probe_reports_b200():
    p = llk.probe(0)
    assert p["is_sm100a"] == 1 and p["sm_count"] >= 100


# ------------------------------------------------------------ decode kernel
@pytest.mark.parametrize("M,K,N", [(1, 4096, 14336), (4, 4096, 14336), (16, 4096, 14336), (3, 512, 200),
                                   (17, 1024, 1000), (64, 2048, 4096), (100, 256, 384), (128, 1024, 1536),
                                   (1, 64, 128), (7, 4104, 136),
                                   # 8-way column shards of config 4 (14 and 13 tiles over every SM:
                                   # ~10 contributors per tile)
                                   (1, 4096, 1792), (4, 4096, 1792), (16, 4096, 1792), (1, 4096, 1664),
                                   (4, 4096, 1664), (16, 4096, 1664), (2, 4096, 3584), (33, 8192, 256)])
def test_decode_vs_oracle(M, K, N):
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0, 0.02, seed=M * 7 + N)
    y = llk.fused_swiglu(dev(x), dev(wg), dev(wu), out_dtype="f32", variant="decode")
    torch.cuda.synchronize()
    llk.synchronize(0)
    ref = oracle.port_swiglu(x, wg, wu, "f32").astype(np.float64)
    assert rel_err(host(y), ref) <= TOL_F32


def test_decode_bf16_deterministic_and_matches_tc():
    x, wg, wu = dg.config_inputs("c4_m16")
    a = llk.fused_swiglu(dev(x), dev(wg), dev(wu), variant="decode")
    b = llk.fused_swiglu(dev(x), dev(wg), dev(wu), variant="decode")
    c = llk.fused_swiglu(dev(x), dev(wg), dev(wu), variant="tc")
    torch.cuda.synchronize()
    llk.synchronize(0)
    assert torch.equal(a, b)  # fixed-order split-K reduction: bitwise reproducible
    d = (a.float() - c.float()).abs().max().item() / c.float().abs().max().item()
    assert d <= TOL_BF16


def test_decode_caller_scratch():
    x, wg, wu = dg.swiglu_inputs(8, 1024, 2048, 1.0, 0.02, seed=5)
    ref = llk.fused_swiglu(dev(x), dev(wg), dev(wu), variant="decode")
    scratch = torch.full((8 << 20,), 7, dtype=torch.uint8, device="cuda")  # garbage-filled
    y = llk.fused_swiglu(dev(x), dev(wg), dev(wu), variant="decode", scratch=scratch)
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    small = torch.zeros((64,), dtype=torch.uint8, device="cuda")
    with pytest.raises(llk.LLKError) as e:
        llk.fused_swiglu(dev(x), dev(wg), dev(wu), variant="decode", scratch=small)
    assert e.value.status == capi.LLK_ERR_NOMEM


@pytest.mark.parametrize("M,K,N", [(4, 1024, 200), (16, 4096, 14336), (300, 512, 136), (1, 64, 64)])
@pytest.mark.parametrize("variant", ["auto", "tc", "decode", "simt"])
def test_packed_slab_layout_matches_row_major(M, K, N, variant):
    if variant == "decode" and M > 128:
        pytest.skip("decode kernel serves M <= 128")
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0, 0.02, seed=N + M)
    pw = llk.PackedWeights(dev(wg), dev(wu))  # packed from device buffers
    assert pw.nbytes == 2 * K * ((N + 63) // 64) * 128
    a = pw(dev(x), out_dtype="f32", variant=variant)
    b = llk.fused_swiglu(dev(x), dev(wg), dev(wu), out_dtype="f32", variant=variant)
    torch.cuda.synchronize()
    llk.synchronize(0)
    assert torch.equal(a, b)  # same kernel, same accumulation order: identical
    pw.close()


@pytest.mark.parametrize("M,N", [(2048, 1408), (2048, 1280), (2048, 2816), (2048, 5504), (4096, 1408)])
def test_column_shard_shapes_k_split_tail(M, N):
    """Config-3 column shards at 2 / 4 / 8 GPUs (and a taller X): few tiles
    per pair, so the built-in plan cuts the leftover tiles along K.  FP64
    points plus whole rows and columns against the oracle, f32 Y; two calls
    give identical results."""
    K = 4096
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0, 0.02, seed=N + 7)
    xd, gd, ud = dev(x), dev(wg), dev(wu)
    y = llk.fused_swiglu(xd, gd, ud, out_dtype="f32")
    y2 = llk.fused_swiglu(xd, gd, ud, out_dtype="f32")
    torch.cuda.synchronize()
    llk.synchronize(0)
    assert torch.equal(y, y2)
    yy = host(y)
    rng = np.random.default_rng(N)
    rows = np.concatenate([rng.integers(0, M, 3000), np.full(N, M - 1), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 3000), np.arange(N), np.full(M, N - 1)])
    ref = oracle.swiglu_fp64_points(x, wg, wu, rows, cols)
    assert float(np.abs(yy[rows, cols] - ref).max() / np.abs(ref).max()) <= TOL_F32


@pytest.mark.parametrize("M,K,N,op", [(300, 512, 520, "swiglu"), (2048, 1024, 1024, "swiglu"), (513, 256, 768, "matmul"),
                                      (1000, 256, 1400, "matmul"), (700, 320, 1408, "swiglu")])
def test_cta_pair_and_single_cta_kernels_agree(M, K, N, op):
    """M > 128 runs on CTA pairs (256-row MMAs); a plan override with
    block_m = 128 pins the one-CTA kernel.  Both must match the oracle."""
    if op == "swiglu":
        x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0 / math.sqrt(K), 1.0, seed=M + 1)
        ref = oracle.swiglu_fused(x, wg, wu, "f32").astype(np.float64)
        run = lambda: llk.fused_swiglu(dev(x), dev(wg), dev(wu), out_dtype="f32", variant="tc")  # noqa: E731
        key = llk.KernelKey(N=N, K=K, M_bucket=llk.classify_m(M), output_type=capi.LLK_DTYPE_FP32)
    else:
        x, wg = dg.matmul_inputs(M, K, N, seed=M + 2)
        ref = oracle.matmul(x, wg).astype(np.float64)
        run = lambda: llk.matmul(dev(x), dev(wg), variant="tc")  # noqa: E731
        key = llk.KernelKey(operation=capi.LLK_OP_MATMUL, N=N, K=K, M_bucket=llk.classify_m(M),
                            output_type=capi.LLK_DTYPE_FP32)
    base = key.plan(M)
    assert base["block_m"] == 256
    y_auto = run()  # the built-in choice (may cut the tail along K)
    torch.cuda.synchronize()
    llk.synchronize(0)
    assert rel_err(host(y_auto), ref) < 1e-5
    key.insert_plan(**dict(base, split_k=1))
    try:
        y_pair = run()  # whole tiles only: the bitwise reference of the column splits
        torch.cuda.synchronize()
        llk.synchronize(0)
    finally:
        key.insert_plan(**base)
    assert rel_err(host(y_pair), ref) < 1e-5
    # leftover tiles cut along K into 2..8 parts (static schedule): partial
    # sums through L2, summed in part order -- deterministic, within tolerance
    for ks in (2, 3, 5, 8):
        key.insert_plan(**dict(base, split_k=-ks, grid=2 * 7, sched=1))
        try:
            y_k = run()
            y_k2 = run()
            torch.cuda.synchronize()
            llk.synchronize(0)
        finally:
            key.insert_plan(**base)
        assert torch.equal(y_k, y_k2), ks
        assert rel_err(host(y_k), ref) < 1e-5, ks
    # leftover tiles cut into 1, 2 or 4 column parts (MMA N 256 / 128 / 64)
    for split, sched in ((1, 0), (2, 0), (4, 0), (1, 1), (4, 1)):
        # 7 pairs: every shape leaves a tail; sched 0 = dynamic, 1 = static
        key.insert_plan(**dict(base, split_k=split, grid=2 * 7, sched=sched))
        try:
            y_split = run()
            torch.cuda.synchronize()
            llk.synchronize(0)
        finally:
            key.insert_plan(**base)
        assert torch.equal(y_split, y_pair), (split, sched)  # same per-element accumulation order
    single = dict(base, block_m=128, grid=148, stages=4)
    key.insert_plan(**single)
    try:
        y_one = run()
        torch.cuda.synchronize()
        llk.synchronize(0)
    finally:
        key.insert_plan(**base)
    assert rel_err(host(y_one), ref) < 1e-5


@pytest.mark.parametrize("M,K,N,op", [(2816, 8192, 1000, "swiglu"), (2600, 16384, 640, "swiglu"),
                                      (2600, 16384, 704, "matmul")])
def test_pair_kernel_row_bands(M, K, N, op):
    """Large K makes the CTA-pair kernel run its tiles in bands of row blocks
    (8 blocks at K = 8192, 4 at K = 16384; the last band narrower): the result
    must match FP64 points and the one-CTA kernel (no bands)."""
    if op == "swiglu":
        x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0 / math.sqrt(K), 1.0, seed=K + 3)
        run = lambda: llk.fused_swiglu(dev(x), dev(wg), dev(wu), out_dtype="f32", variant="tc")  # noqa: E731
        key = llk.KernelKey(N=N, K=K, M_bucket=llk.classify_m(M), output_type=capi.LLK_DTYPE_FP32)
    else:
        x, wg = dg.matmul_inputs(M, K, N, seed=K + 4)
        run = lambda: llk.matmul(dev(x), dev(wg), variant="tc")  # noqa: E731
        key = llk.KernelKey(operation=capi.LLK_OP_MATMUL, N=N, K=K, M_bucket=llk.classify_m(M),
                            output_type=capi.LLK_DTYPE_FP32)
    base = key.plan(M)
    assert base["block_m"] == 256
    y_pair = run()
    torch.cuda.synchronize()
    llk.synchronize(0)
    key.insert_plan(**dict(base, block_m=128, grid=148, stages=4))
    try:
        y_one = run()
        torch.cuda.synchronize()
        llk.synchronize(0)
    finally:
        key.insert_plan(**base)
    yp, yo = host(y_pair), host(y_one)
    assert rel_err(yp, yo) < 1e-4  # the pair kernel may cut its tail along K: another summation order
    rng = np.random.default_rng(K)
    rows = np.concatenate([rng.integers(0, M, 3000), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 3000), rng.integers(0, N, M)])
    if op == "swiglu":
        ref = oracle.swiglu_fp64_points(x, wg, wu, rows, cols)
    else:
        xa = dg.bf16_bits_to_f32(x).astype(np.float64)
        wa = dg.bf16_bits_to_f32(wg).astype(np.float64)
        ref = np.einsum("ik,ki->i", xa[rows], wa[:, cols])
    assert float(np.abs(yp[rows, cols] - ref).max() / np.abs(ref).max()) <= TOL_F32


def test_packed_weights_l4_cache():
    """PackedWeights.cached: a miss packs and inserts, a hit returns the same
    device copy (no second pack), results equal the unpacked path, and the
    copy outlives the first handle until the cache evicts it."""
    M, K, N = 300, 512, 640
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0 / math.sqrt(K), 1.0, seed=9)
    xd, gd, ud = dev(x), dev(wg), dev(wu)
    llk.cache_level_clear(4)
    a = llk.PackedWeights.cached(gd, ud)
    b = llk.PackedWeights.cached(gd, ud)
    s = llk.cache_level_stats(4)
    assert s["misses"] == 1 and s["hits"] == 1 and s["size"] == 1
    assert a.layout()["wg"] == b.layout()["wg"] and a.layout()["box_n"] == 64
    ref = llk.fused_swiglu(xd, gd, ud, out_dtype="f32")
    a.close()  # the cache's reference keeps the device copy
    y = b(xd, out_dtype="f32")
    torch.cuda.synchronize()
    llk.synchronize(0)
    assert torch.equal(y, ref)
    llk.cache_level_set_max_entries(4, 0)
    assert llk.cache_level_stats(4)["size"] == 0
    y2 = b(xd, out_dtype="f32")  # b still holds its reference
    torch.cuda.synchronize()
    assert torch.equal(y2, ref)
    b.close()
    llk.cache_level_set_max_entries(4, 64)
    llk.cache_level_clear(4)


def test_fused_call_allocates_no_intermediate():
    """The fused kernel keeps gate and up in TMEM: after the first call (the
    library's workspace and plan), further calls of config-3 size allocate no
    device memory at all -- in particular no [M, N] intermediate (the
    reference checks the same of its fused IR, test/Execution/
    swiglu_fused_memory.cpp:152-183)."""
    M, K, N = 2048, 4096, 11008
    x = torch.randn(M, K, device="cuda").bfloat16()
    wg = (torch.randn(K, N, device="cuda") * 0.02).bfloat16()
    wu = (torch.randn(K, N, device="cuda") * 0.02).bfloat16()
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):
        llk.fused_swiglu(x, wg, wu, out=y)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(20):
        llk.fused_swiglu(x, wg, wu, out=y)
    torch.cuda.synchronize()
    llk.synchronize(0)
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0 - free1)
