"""The CPU oracle pinned against the reference's own outputs and known answers.

The fixtures in tests/golden were produced by the reference's
test/Execution/swiglu_reference.cpp compiled from its source
(tests/golden/make_golden.py).  The restatement must reproduce them
bit-for-bit where it follows the same loops.
"""
import math

import numpy as np
import pytest

import oracle
from dslcompiler_b200 import datagen as dg
from tests.conftest import load_golden


def test_golden_fixtures_present(golden_names):
    assert len(golden_names) >= 8


def test_naive_f32_bit_exact_vs_reference(golden_names):
    for name in golden_names:
        g = load_golden(name)
        x, wg, wu = (dg.bf16_bits_to_f32(g[k]) for k in ("x", "wg", "wu"))
        y = oracle.swiglu_naive_f32(x, wg, wu)
        assert np.array_equal(y.view(np.uint32), g["y_ref_f32"].view(np.uint32)), name


def test_fp64_matches_reference(golden_names):
    for name in golden_names:
        g = load_golden(name)
        x, wg, wu = (dg.bf16_bits_to_f32(g[k]).astype(np.float64) for k in ("x", "wg", "wu"))
        y = oracle.swiglu_fp64(x, wg, wu)
        np.testing.assert_allclose(y, g["y_ref_f64"], rtol=1e-13, atol=1e-15, err_msg=name)


def test_fused_semantics_within_tolerance_of_reference(golden_names):
    # The fused (production) epilogue g*(1/(1+e^-g))*u differs from the test
    # oracle's g/(1+e^-g)*u only in rounding.
    for name in golden_names:
        g = load_golden(name)
        y = oracle.swiglu_fused(g["x"], g["wg"], g["wu"], "f32")
        ref = g["y_ref_f64"]
        scale = max(np.abs(ref).max(), 1e-30)
        assert np.abs(y - ref).max() / scale < 1e-5, name
        yb = dg.bf16_bits_to_f32(oracle.swiglu_fused(g["x"], g["wg"], g["wu"], "bf16"))
        assert np.abs(yb - ref).max() / scale < 1e-2, name


def test_points_fp64_matches_full():
    g = load_golden("config1_64_512_256")
    rows = np.array([0, 5, 63, 17]); cols = np.array([0, 511, 100, 257])
    pts = oracle.swiglu_fp64_points(g["x"], g["wg"], g["wu"], rows, cols)
    np.testing.assert_allclose(pts, g["y_ref_f64"][rows, cols], rtol=1e-12)


def test_known_values():
    # swiglu_reference.cpp:156-175: X=1, Wg=2, Wu=3 -> 2/(1+e^-2) * 3
    y = oracle.swiglu_fp64(np.array([[1.0]]), np.array([[2.0]]), np.array([[3.0]]))
    assert abs(y[0, 0] - (2.0 / (1.0 + math.exp(-2.0))) * 3.0) < 1e-12
    y32 = oracle.swiglu_naive_f32(np.array([[1.0]]), np.array([[2.0]]), np.array([[3.0]]))
    assert abs(float(y32[0, 0]) - float(y[0, 0])) < 1e-4


def test_edge_cases_known_answers():
    # edge_cases.cpp:47-150
    y = oracle.swiglu_fp64(np.array([[2.0]]), np.array([[0.5]]), np.array([[0.3]]))
    assert abs(y[0, 0] - (1.0 / (1.0 + math.exp(-1.0))) * 0.6) < 1e-12
    y = oracle.swiglu_fp64(np.ones((3, 1)), np.full((1, 2), 0.5), np.full((1, 2), 0.3))
    assert np.all(y == y[0, 0])
    y = oracle.swiglu_fp64(np.zeros((0, 4)), np.full((4, 8), 0.5), np.full((4, 8), 0.3))
    assert y.shape == (0, 8)
    x = np.array([[10.0, -10.0]]); w = np.eye(2)
    y = oracle.swiglu_fp64(x, w, w)
    assert y[0, 0] > 90.0 and abs(y[0, 1]) < 1.0
    y = oracle.swiglu_fp64(np.zeros((2, 4)), np.zeros((4, 3)), np.zeros((4, 3)))
    assert np.all(y == 0.0)


def test_bf16_round_trip():
    # swiglu_reference.cpp:145-154
    for v in (-3.14, -1.0, 0.0, 1.0, 3.14, 42.0):
        r = float(oracle.bf16_to_f32(oracle.f32_to_bf16(np.array([v], np.float32)))[0])
        assert abs(r - v) <= 1e-2 * max(1.0, abs(v))


def test_datagen_rounding_matches_oracle():
    a = dg.normal_f32(5, (1000,), 0.0, 3.0)
    assert np.array_equal(dg.f32_to_bf16_bits(a), oracle.f32_to_bf16(a))


def test_datagen_deterministic_and_distributed():
    a = dg.normal_f32(42, (200000,), 0.0, 1.0)
    b = dg.normal_f32(42, (200000,), 0.0, 1.0)
    assert np.array_equal(a, b)
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1.0) < 0.01
    u = dg.uniform_f32(1, (100000,), -1.0, 1.0)
    assert u.min() >= -1.0 and u.max() < 1.0 and abs(u.mean()) < 0.01
    # chunk boundaries do not change the stream
    n = (1 << 24) + 5
    big = dg.normal_f32(9, (n,), 0.0, 1.0)
    assert np.array_equal(big[:1000], dg.normal_f32(9, (1000,), 0.0, 1.0))


def test_packing_bit_identical():
    # packed_vs_unpacked.cpp:77-106: BKxBN tile packing is a pure relayout
    rng = np.random.default_rng(0)
    M, N, K, BK, BN = 8, 64, 64, 32, 32
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.standard_normal((K, N)).astype(np.float32)
    p = oracle.pack_weights_tiled(w, BK, BN)
    nb = N // BN
    unpacked = np.empty_like(w)
    for k in range(K):
        for n in range(N):
            unpacked[k, n] = p[((k // BK) * nb + n // BN) * BK * BN + (k % BK) * BN + n % BN]
    assert np.array_equal(unpacked, w)
    assert p.size == K * N  # NoIntermediatesLeaked: same element count


def test_kblock_packing_layout():
    # runtime/PackedWeights.cpp:5-33: K rows padded to a multiple of BK
    w = dg.f32_to_bf16_bits(dg.normal_f32(3, (70, 24)))
    p = oracle.pack_weights_kblock(w, 64)
    assert p.shape == (128, 24)
    assert np.array_equal(p[:70], w) and np.all(p[70:] == 0)


@pytest.mark.parametrize("M,bucket", [(1, 0), (2, 1), (4, 1), (5, 2), (8, 2), (16, 2), (17, 3), (32, 3), (64, 3),
                                      (65, 4), (128, 4), (512, 4)])
def test_classify_m_table(M, bucket):
    # specialization_dispatch.cpp:31-61
    assert oracle.classify_m(M) == bucket


def test_port_matches_oracle():
    x, wg, wu = dg.swiglu_inputs(37, 200, 150, 0.1, 0.1, seed=3)
    ref = oracle.swiglu_fused(x, wg, wu, "f32")
    y = oracle.port_swiglu(x, wg, wu, "f32", threads=4)
    assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()
    a, b = dg.matmul_inputs(33, 70, 90, seed=4)
    np.testing.assert_allclose(oracle.port_matmul(a, b, threads=3), oracle.matmul(a, b), rtol=1e-4, atol=1e-4)
