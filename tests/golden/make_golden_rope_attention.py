"""Generates tests/golden/rope_*.npz and attention_*.npz by running the
DSLCompiler reference's OWN FP64 RoPE and attention references
(test/Execution/rope_correctness.cpp:14-35, attention_correctness.cpp:15-60,
compiled from their sources by ``make -C oracle ref`` into
oracle/_ref/ref_rope_attention_driver) on seeded inputs.

Run here, where the reference tree exists:

    make -C oracle ref REF=<DSLCompiler tree> && python tests/golden/make_golden_rope_attention.py

Inputs are f32 values (seeded, dslcompiler_b200.datagen) given to the
reference as f64; each fixture stores them with the reference's f64 output.
Shapes are those of the reference's tests and lowering tests:
  * RoPE (1,1,8,64) theta 1e4, (2,4,32,128) theta 5e4     rope_correctness.cpp:40, 62
  * RoPE (1,1,1,64), positions 0, theta 1, x = 1..64      rope_correctness.cpp:81-95 (identity)
  * RoPE (2,4,32,64) and (1,1,128,64)                     test/Transforms/rope_broadcast.mlir:9,
                                                          test/Conversion/rope_lowering.mlir:4
  * attention (1,1,8,8,64) causal, (2,4,16,16,64)          attention_correctness.cpp:65, 88
  * attention (1,1,4,4,4) causal, the known-answer inputs  attention_correctness.cpp:110-140
  * attention (1,1,32,32,64) causal, (1,1,128,128,128)     test/Transforms/causal_mask.mlir:5,
                                                          test/Transforms/online_softmax.mlir:4
"""
from __future__ import annotations

import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from dslcompiler_b200 import datagen as dg  # noqa: E402

DRIVER = os.path.join(ROOT, "oracle", "_ref", "ref_rope_attention_driver")


def ref_rope(x, pos, theta):
    B, H, L, D = x.shape
    with tempfile.TemporaryDirectory() as d:
        px, pp, py = (os.path.join(d, n) for n in ("x", "pos", "y"))
        x.astype(np.float64).tofile(px)
        pos.astype(np.int64).tofile(pp)
        subprocess.run([DRIVER, "rope", str(B), str(H), str(L), str(D), repr(float(theta)), px, pp, py], check=True)
        return np.fromfile(py, np.float64).reshape(x.shape)


def ref_attention(q, k, v, scale, causal):
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    with tempfile.TemporaryDirectory() as d:
        pq, pk, pv, po = (os.path.join(d, n) for n in ("q", "k", "v", "o"))
        for a, p in ((q, pq), (k, pk), (v, pv)):
            a.astype(np.float64).tofile(p)
        subprocess.run([DRIVER, "attention", str(B), str(H), str(Lq), str(Lk), str(D), repr(float(scale)),
                        str(int(causal)), pq, pk, pv, po], check=True)
        return np.fromfile(po, np.float64).reshape(q.shape)


def main():
    if not os.path.exists(DRIVER):
        sys.exit("oracle/_ref/ref_rope_attention_driver missing: run `make -C oracle ref REF=<DSLCompiler tree>`")
    ropes = [("rope_1_1_8_64", (1, 1, 8, 64), 1e4, "arange"), ("rope_2_4_32_128", (2, 4, 32, 128), 5e4, "arange"),
             ("rope_identity_1_1_1_64", (1, 1, 1, 64), 1.0, "zero"), ("rope_2_4_32_64", (2, 4, 32, 64), 1e4, "arange"),
             ("rope_1_1_128_64", (1, 1, 128, 64), 1e4, "random")]
    for i, (name, shape, theta, posmode) in enumerate(ropes):
        B, H, L, D = shape
        if name.startswith("rope_identity"):
            x = np.arange(1, D + 1, dtype=np.float32).reshape(shape)
        else:
            x = dg.normal_f32(2000 + i, shape)
        pos = {"arange": np.arange(L, dtype=np.int64), "zero": np.zeros(L, np.int64),
               "random": np.random.default_rng(i).integers(0, 8192, L).astype(np.int64)}[posmode]
        y = ref_rope(x, pos, theta)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), x=x, pos=pos, theta=np.float64(theta), y_ref_f64=y)
        print(f"{name}: max|y|={np.abs(y).max():.4g}")
    atts = [("attention_1_1_8_8_64_causal", (1, 1, 8, 8, 64), True, 0.02),
            ("attention_2_4_16_16_64", (2, 4, 16, 16, 64), False, 0.02),
            ("attention_known_1_1_4_4_4_causal", (1, 1, 4, 4, 4), True, None),
            ("attention_1_1_32_32_64_causal", (1, 1, 32, 32, 64), True, 1.0),
            ("attention_1_1_128_128_128_causal", (1, 1, 128, 128, 128), True, 1.0)]
    for i, (name, (B, H, Lq, Lk, D), causal, std) in enumerate(atts):
        if std is None:  # attention_correctness.cpp:110-140
            q = np.zeros((B, H, Lq, D), np.float32)
            q[..., 0, :] = 1.0
            k = np.ones((B, H, Lk, D), np.float32)
            v = np.zeros((B, H, Lk, D), np.float32)
            v[..., 0, :] = 2.0
        else:
            q = dg.normal_f32(3000 + 3 * i, (B, H, Lq, D), 0.0, std)
            k = dg.normal_f32(3001 + 3 * i, (B, H, Lk, D), 0.0, std)
            v = dg.normal_f32(3002 + 3 * i, (B, H, Lk, D), 0.0, std)
        scale = 1.0 / np.sqrt(D)
        o = ref_attention(q, k, v, scale, causal)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), q=q, k=k, v=v, scale=np.float64(scale),
                            causal=np.bool_(causal), o_ref_f64=o)
        print(f"{name}: max|o|={np.abs(o).max():.4g}")


if __name__ == "__main__":
    main()
