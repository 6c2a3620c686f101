"""CPU oracle for DSLCompiler's fused SwiGLU / micro.mma path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm import this package, and only as
the checker or the timed CPU baseline -- never as the thing measured on the
GPU or shipped.  The product (``dslcompiler_b200``) never imports it.

It wraps ``_build/liboracle.so`` built from:
  * ``swiglu_oracle.c`` -- scalar restatement of the reference arithmetic
    (``test/Execution/swiglu_reference.cpp:38-99``,
    ``lib/Transforms/FuseDoubleContraction.cpp:119-199``), bit-exact against
    the reference compiled from its own sources (``_ref/ref_driver``);
  * ``swiglu_port.c`` -- threaded fused-schedule restatement used as the CPU
    baseline (``lib/Transforms/TileAndVectorize.cpp:53-57`` tiling);
  * ``rope_attention_oracle.c`` -- the llk.rope / llk.attention lowerings
    (``lib/Conversion/LLKToLinalg/LLKToLinalg.cpp:162-608``) in f32 and the
    reference tests' FP64 references.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
REF_DRIVER = os.path.join(HERE, "_ref", "ref_driver")

_lib = None


def build(force: bool = False) -> str:
    """Compile liboracle.so with gcc (no reference sources needed)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.oracle_swiglu_naive_f32.argtypes = [p, p, p, p, i64, i64, i64]
        L.oracle_swiglu_fp64.argtypes = [p, p, p, p, i64, i64, i64]
        L.oracle_swiglu_fp64_points.argtypes = [p, i64, p, p, i64, i64, p, p, i64, p]
        L.oracle_swiglu_fused.argtypes = [p, i64, p, p, i64, i64, i64, i64, p, p, i64]
        L.oracle_matmul.argtypes = [p, i64, p, i64, p, i64, i64, i64, i64, i32]
        L.oracle_pack_weights_kblock.argtypes = [p, i64, i64, i64, i64, p]
        L.oracle_pack_weights_tiled.argtypes = [p, i64, i64, i64, i64, p]
        L.oracle_classify_m.argtypes = [i64]
        L.oracle_classify_m.restype = i32
        L.oracle_f32_to_bf16_array.argtypes = [p, p, i64]
        L.oracle_bf16_to_f32_array.argtypes = [p, p, i64]
        L.port_swiglu.argtypes = [p, i64, p, p, i64, i64, i64, i64, p, p, i64, i32]
        L.port_matmul.argtypes = [p, i64, p, i64, p, i64, i64, i64, i64, i32]
        L.oracle_rope_f32.argtypes = [p, p, p, i64, i64, i64, i64, ctypes.c_double]
        L.oracle_rope_fp64.argtypes = [p, p, p, i64, i64, i64, i64, ctypes.c_double]
        L.oracle_attention_f32.argtypes = [p, p, p, p, i64, i64, i64, i64, i64, ctypes.c_float, i32]
        L.oracle_attention_fp64.argtypes = [p, p, p, p, i64, i64, i64, i64, i64, ctypes.c_double, i32]
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def f32_to_bf16(a) -> np.ndarray:
    """f32 -> bf16 bit patterns (uint16), round-to-nearest-even."""
    a = _c(a, np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().oracle_f32_to_bf16_array(_ptr(a), _ptr(out), a.size)
    return out


def bf16_to_f32(a) -> np.ndarray:
    a = _c(a, np.uint16)
    out = np.empty(a.shape, np.float32)
    lib().oracle_bf16_to_f32_array(_ptr(a), _ptr(out), a.size)
    return out


def swiglu_naive_f32(x, wg, wu) -> np.ndarray:
    """The reference test oracle's FP32 SwiGLU (swiglu_reference.cpp:38-71)."""
    x, wg, wu = _c(x, np.float32), _c(wg, np.float32), _c(wu, np.float32)
    M, K = x.shape
    N = wg.shape[1]
    y = np.empty((M, N), np.float32)
    lib().oracle_swiglu_naive_f32(_ptr(x), _ptr(wg), _ptr(wu), _ptr(y), M, N, K)
    return y


def swiglu_fp64(x, wg, wu) -> np.ndarray:
    """FP64 ground truth (swiglu_reference.cpp:77-99)."""
    x, wg, wu = _c(x, np.float64), _c(wg, np.float64), _c(wu, np.float64)
    M, K = x.shape
    N = wg.shape[1]
    y = np.empty((M, N), np.float64)
    lib().oracle_swiglu_fp64(_ptr(x), _ptr(wg), _ptr(wu), _ptr(y), M, N, K)
    return y


def swiglu_fused(x_bf16, wg_bf16, wu_bf16, out: str = "f32") -> np.ndarray:
    """Fused production semantics on bf16 inputs.  out: 'f32' or 'bf16'
    (bf16 returns uint16 bit patterns)."""
    x, wg, wu = _c(x_bf16, np.uint16), _c(wg_bf16, np.uint16), _c(wu_bf16, np.uint16)
    M, K = x.shape
    N = wg.shape[1]
    if out == "f32":
        y = np.empty((M, N), np.float32)
        lib().oracle_swiglu_fused(_ptr(x), K, _ptr(wg), _ptr(wu), N, M, N, K, _ptr(y), None, N)
    else:
        y = np.empty((M, N), np.uint16)
        lib().oracle_swiglu_fused(_ptr(x), K, _ptr(wg), _ptr(wu), N, M, N, K, None, _ptr(y), N)
    return y


def swiglu_fp64_points(x_bf16, wg_bf16, wu_bf16, rows, cols) -> np.ndarray:
    """FP64 SwiGLU of bf16 inputs at the listed (row, col) points only."""
    x, wg, wu = _c(x_bf16, np.uint16), _c(wg_bf16, np.uint16), _c(wu_bf16, np.uint16)
    rows, cols = _c(rows, np.int64), _c(cols, np.int64)
    K = x.shape[1]
    out = np.empty(rows.shape[0], np.float64)
    lib().oracle_swiglu_fp64_points(_ptr(x), K, _ptr(wg), _ptr(wu), wg.shape[1], K,
                                    _ptr(rows), _ptr(cols), rows.shape[0], _ptr(out))
    return out


def matmul(a_bf16, b_bf16, c_init=None) -> np.ndarray:
    """micro.mma semantics: C (f32) = [C_init +] A*B, bf16 operands."""
    a, b = _c(a_bf16, np.uint16), _c(b_bf16, np.uint16)
    M, K = a.shape
    N = b.shape[1]
    c = np.zeros((M, N), np.float32) if c_init is None else _c(c_init, np.float32).copy()
    lib().oracle_matmul(_ptr(a), K, _ptr(b), N, _ptr(c), N, M, N, K, int(c_init is not None))
    return c


def port_swiglu(x_bf16, wg_bf16, wu_bf16, out: str = "f32", threads: int | None = None):
    """Threaded fused-schedule CPU port (the CPU baseline)."""
    x, wg, wu = _c(x_bf16, np.uint16), _c(wg_bf16, np.uint16), _c(wu_bf16, np.uint16)
    M, K = x.shape
    N = wg.shape[1]
    threads = threads or os.cpu_count() or 1
    if out == "f32":
        y = np.empty((M, N), np.float32)
        lib().port_swiglu(_ptr(x), K, _ptr(wg), _ptr(wu), N, M, N, K, _ptr(y), None, N, threads)
    else:
        y = np.empty((M, N), np.uint16)
        lib().port_swiglu(_ptr(x), K, _ptr(wg), _ptr(wu), N, M, N, K, None, _ptr(y), N, threads)
    return y


def port_matmul(a_bf16, b_bf16, threads: int | None = None):
    a, b = _c(a_bf16, np.uint16), _c(b_bf16, np.uint16)
    M, K = a.shape
    N = b.shape[1]
    c = np.empty((M, N), np.float32)
    lib().port_matmul(_ptr(a), K, _ptr(b), N, _ptr(c), N, M, N, K, threads or os.cpu_count() or 1)
    return c


def pack_weights_kblock(w_bf16, BK: int) -> np.ndarray:
    """runtime/PackedWeights.cpp:5-33 layout (K padded to a multiple of BK)."""
    w = _c(w_bf16, np.uint16)
    K, N = w.shape
    kb = (K + BK - 1) // BK
    out = np.empty((kb * BK, N), np.uint16)
    lib().oracle_pack_weights_kblock(_ptr(w), K, N, N, BK, _ptr(out))
    return out


def pack_weights_tiled(w_f32, BK: int, BN: int) -> np.ndarray:
    """test/Execution/packed_vs_unpacked.cpp:31-51 layout."""
    w = _c(w_f32, np.float32)
    K, N = w.shape
    kb, nb = (K + BK - 1) // BK, (N + BN - 1) // BN
    out = np.empty(kb * nb * BK * BN, np.float32)
    lib().oracle_pack_weights_tiled(_ptr(w), K, N, BK, BN, _ptr(out))
    return out


def classify_m(M: int) -> int:
    return lib().oracle_classify_m(M)


def ref_driver_available() -> bool:
    return os.path.exists(REF_DRIVER)


def rope_f32(x, pos, theta: float = 10000.0) -> np.ndarray:
    """llk.rope as lowered by the reference (f32 result)."""
    x = _c(x, np.float32)
    pos = _c(pos, np.int64)
    B, H, L, D = x.shape
    y = np.empty_like(x)
    lib().oracle_rope_f32(_ptr(x), _ptr(pos), _ptr(y), B, H, L, D, float(theta))
    return y


def rope_fp64(x, pos, theta: float = 10000.0) -> np.ndarray:
    """FP64 RoPE of the reference's tests (rope_correctness.cpp:14-35)."""
    x = _c(x, np.float64)
    pos = _c(pos, np.int64)
    B, H, L, D = x.shape
    y = np.empty_like(x)
    lib().oracle_rope_fp64(_ptr(x), _ptr(pos), _ptr(y), B, H, L, D, float(theta))
    return y


def attention_f32(q, k, v, scale: float, causal: bool, init=None) -> np.ndarray:
    """llk.attention as lowered by the reference: init + softmax(scale QK^T) V (f32)."""
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    o = np.zeros_like(q) if init is None else _c(init, np.float32).copy()
    lib().oracle_attention_f32(_ptr(q), _ptr(k), _ptr(v), _ptr(o), B, H, Lq, Lk, D, float(scale), int(bool(causal)))
    return o


def attention_fp64(q, k, v, scale: float, causal: bool) -> np.ndarray:
    """FP64 attention of the reference's tests (attention_correctness.cpp:15-60)."""
    q, k, v = _c(q, np.float64), _c(k, np.float64), _c(v, np.float64)
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    o = np.zeros_like(q)
    lib().oracle_attention_fp64(_ptr(q), _ptr(k), _ptr(v), _ptr(o), B, H, Lq, Lk, D, float(scale), int(bool(causal)))
    return o
