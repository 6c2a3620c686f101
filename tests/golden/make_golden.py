"""Generates tests/golden/*.npz by running the DSLCompiler reference's OWN
SwiGLU oracle (test/Execution/swiglu_reference.cpp, compiled from its source
by ``make -C oracle ref`` into oracle/_ref/ref_driver) on seeded inputs.

Run here, where the reference tree exists:

    make -C oracle ref REF=<DSLCompiler tree> && python tests/golden/make_golden.py

Each fixture holds bf16 inputs (uint16 bit patterns, drawn with
dslcompiler_b200.datagen and rounded RNE), and the reference's outputs on
those exact values: ``y_ref_f32`` from its naive FP32 ``swiglu_reference``
and ``y_ref_f64`` from ``swiglu_reference_fp64``.  Nothing at test time
needs the reference tree.

Shapes (M, N, K) are the ones the reference's tests use:
  * SmallShapes (1,4,2), (2,3,4), (4,8,16)     swiglu_reference.cpp:111-115
  * E2EWithAbiWrapper (4,8,3)                   swiglu_scalar.cpp:355
  * SwiGLUVectorAVX2 (32,128,256), (16,512,512), (32,256,127)
                                                swiglu_vector_avx2.cpp:214-218
  * benchmark config 1: M=64, K=256, N=512 with N(0,1)/sqrt(K) inputs
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

REF_DRIVER = os.path.join(ROOT, "oracle", "_ref", "ref_driver")

CASES = [
    ("small_1_4_2", 1, 4, 2, 1.0),
    ("small_2_3_4", 2, 3, 4, 1.0),
    ("small_4_8_16", 4, 8, 16, 1.0),
    ("e2e_4_8_3", 4, 8, 3, 1.0),
    ("avx2_32_128_256", 32, 128, 256, 1.0 / 16.0),
    ("avx2_16_512_512", 16, 512, 512, 1.0 / np.sqrt(512.0)),
    ("avx2_32_256_127", 32, 256, 127, 1.0 / np.sqrt(127.0)),
    ("config1_64_512_256", 64, 512, 256, 1.0 / 16.0),
]


def run_reference(x, wg, wu):
    M, K = x.shape
    N = wg.shape[1]
    with tempfile.TemporaryDirectory() as d:
        paths = {n: os.path.join(d, n) for n in ("x", "wg", "wu", "y32", "y64")}
        dg.bf16_bits_to_f32(x).tofile(paths["x"])
        dg.bf16_bits_to_f32(wg).tofile(paths["wg"])
        dg.bf16_bits_to_f32(wu).tofile(paths["wu"])
        subprocess.run([REF_DRIVER, "swiglu", str(M), str(N), str(K), paths["x"], paths["wg"], paths["wu"],
                        paths["y32"], paths["y64"]], check=True)
        y32 = np.fromfile(paths["y32"], np.float32).reshape(M, N)
        y64 = np.fromfile(paths["y64"], np.float64).reshape(M, N)
    return y32, y64


def main():
    if not os.path.exists(REF_DRIVER):
        sys.exit("oracle/_ref/ref_driver missing: run `make -C oracle ref REF=<DSLCompiler tree>` where the reference tree exists")
    for i, (name, M, N, K, std) in enumerate(CASES):
        x, wg, wu = dg.swiglu_inputs(M, K, N, std, std, seed=1000 + i)
        y32, y64 = run_reference(x, wg, wu)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), x=x, wg=wg, wu=wu, y_ref_f32=y32, y_ref_f64=y64,
                            shape=np.array([M, N, K]))
        print(f"{name}: M={M} N={N} K={K} max|y|={np.abs(y64).max():.4g}")


if __name__ == "__main__":
    main()
