"""The llk.rope / llk.attention CPU oracle pinned against the reference's own
FP64 references (tests/golden/rope_*.npz, attention_*.npz, produced by
test/Execution/rope_correctness.cpp and attention_correctness.cpp compiled
from their sources: tests/golden/make_golden_rope_attention.py) and their
known answers."""
import numpy as np

import oracle
from tests.conftest import load_golden


def test_fixtures_present(rope_golden_names, attention_golden_names):
    assert len(rope_golden_names) >= 5 and len(attention_golden_names) >= 5


def test_rope_fp64_bit_exact_vs_reference(rope_golden_names):
    for name in rope_golden_names:
        g = load_golden(name)
        y = oracle.rope_fp64(g["x"].astype(np.float64), g["pos"], float(g["theta"]))
        assert np.array_equal(y, g["y_ref_f64"]), name


def test_rope_f32_lowering_within_f32_rounding_of_reference(rope_golden_names):
    for name in rope_golden_names:
        g = load_golden(name)
        y = oracle.rope_f32(g["x"], g["pos"], float(g["theta"]))
        ref = g["y_ref_f64"]
        # the lowering rounds the angle to f32 before cos / sin: up to half an
        # ulp of the largest angle (pos * theta^0 = pos), plus f32 rounding
        tol = 2e-6 + 2.0 * float(np.abs(g["pos"]).max()) * 2.0 ** -24
        assert np.abs(y - ref).max() <= tol * max(np.abs(ref).max(), 1.0), name


def test_rope_known_answers():
    # position 0 is the identity for any theta (rope_correctness.cpp:81-95)
    x = np.arange(1, 65, dtype=np.float32).reshape(1, 1, 1, 64)
    for theta in (1.0, 10000.0):
        assert np.array_equal(oracle.rope_f32(x, np.zeros(1, np.int64), theta), x)
    # pairs rotate by pos * theta^(-2i/D): pair 0 turns by exactly pos radians
    x = np.zeros((1, 1, 1, 4), np.float32)
    x[..., 0] = 1.0
    y = oracle.rope_f32(x, np.array([1], np.int64), 10000.0)
    assert np.allclose(y[0, 0, 0, :2], [np.cos(1.0), np.sin(1.0)], atol=1e-7)


def test_attention_fp64_bit_exact_vs_reference(attention_golden_names):
    for name in attention_golden_names:
        g = load_golden(name)
        o = oracle.attention_fp64(g["q"], g["k"], g["v"], float(g["scale"]), bool(g["causal"]))
        assert np.array_equal(o, g["o_ref_f64"]), name


def test_attention_f32_lowering_within_tolerance_of_reference(attention_golden_names):
    for name in attention_golden_names:
        g = load_golden(name)
        o = oracle.attention_f32(g["q"], g["k"], g["v"], float(g["scale"]), bool(g["causal"]))
        ref = g["o_ref_f64"]
        assert np.abs(o - ref).max() <= 1e-5 * max(np.abs(ref).max(), 1e-30), name


def test_attention_known_answers_and_init():
    # causal: token 0 attends only to itself, token 1 uniformly to 0 and 1
    # (attention_correctness.cpp:110-140)
    g = load_golden("attention_known_1_1_4_4_4_causal")
    o = oracle.attention_f32(g["q"], g["k"], g["v"], float(g["scale"]), True)
    assert np.allclose(o[0, 0, 0], 2.0) and np.allclose(o[0, 0, 1], 1.0)
    # destination passing: the result adds to the init operand
    init = np.full(o.shape, 0.5, np.float32)
    o2 = oracle.attention_f32(g["q"], g["k"], g["v"], float(g["scale"]), True, init=init)
    assert np.allclose(o2, o + 0.5)
