"""Builds the in-tree shared library ``dslcompiler_b200/lib/libllk_b200.so``.

Every CUDA source is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked with the static
CUDA runtime, so the library does not depend on which libcudart the host
process (e.g. torch) has loaded; device pointers and streams are shared
through the driver's primary context.

    python -m dslcompiler_b200.build [--force] [--jobs N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT_DIR = os.path.join(PKG, "lib")
OBJ_DIR = os.path.join(ROOT, "_build", "obj")
LIB = os.path.join(OUT_DIR, "libllk_b200.so")

SOURCES = ["swiglu_tc.cu", "swiglu_tc2.cu", "swiglu_decode.cu", "swiglu_simt.cu", "llk_runtime.cu", "swiglu_decode_noalloc.cu", "shard_gather.cu",
           "rope_attention.cu"]
HEADERS = ["sm100_ptx.cuh", "tc_kernels.h", "decode_kernels.h", "workspace.h",
           "attention_kernels.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
          "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the B200 library cannot be built")


def _newest_input() -> float:
    paths = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    paths.append(os.path.join(ROOT, "include", "llk_b200.h"))
    paths.append(os.path.abspath(__file__))
    return max(os.path.getmtime(p) for p in paths)


def up_to_date() -> bool:
    return os.path.exists(LIB) and os.path.getmtime(LIB) >= _newest_input()


def _compile(src: str) -> str:
    obj = os.path.join(OBJ_DIR, os.path.splitext(src)[0] + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
    subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=jobs or min(len(SOURCES), os.cpu_count() or 1)) as ex:
        objs = list(ex.map(_compile, SOURCES))
    tmp = LIB + ".tmp"
    # Export only the C ABI (llk_*); everything else stays local.
    vs = os.path.join(OBJ_DIR, "exports.map")
    with open(vs, "w") as f:
        f.write("{ global: llk_*; local: *; };\n")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-Xlinker", "--version-script=" + vs, "-o", tmp, *objs]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    if verbose:
        print("built", LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    a = ap.parse_args(argv)
    build(force=a.force, jobs=a.jobs, verbose=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
