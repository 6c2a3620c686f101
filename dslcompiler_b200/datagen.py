"""Seeded synthetic inputs for the SwiGLU / matmul configurations.

The reference draws its test data from ``std::mt19937(42)`` and
``std::normal_distribution<float>`` (e.g. ``test/Execution/swiglu_reference.cpp:120-121``),
whose stream is implementation-defined (libstdc++ and libc++ differ).  This
module uses a portable counter-based generator instead: splitmix64 outputs
turned into normals by Box-Muller (cos branch then sin branch per pair) or
into uniforms by the top 53 bits.  Values are drawn in f32 and rounded to
bf16 (round-to-nearest-even) -- the same rounding as the reference's
``f32_to_bf16`` (``swiglu_reference.cpp:26-32``).

Everything is vectorised numpy so a Llama-70B-sized weight (235 M values)
is drawn in seconds.
"""
from __future__ import annotations

import numpy as np

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_CHUNK = 1 << 24


def _splitmix64(seed: int, start: int, n: int) -> np.ndarray:
    """Outputs start..start+n-1 of the splitmix64 stream seeded with `seed`."""
    with np.errstate(over="ignore"):
        i = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        z = np.uint64(seed) + i * _GAMMA
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def _u01(v: np.ndarray) -> np.ndarray:
    return ((v >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def normal_f32(seed: int, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    out = np.empty(n, np.float32)
    npairs = (n + 1) // 2
    for p0 in range(0, npairs, _CHUNK):
        p1 = min(npairs, p0 + _CHUNK)
        v = _splitmix64(seed, 2 * p0, 2 * (p1 - p0))
        u1, u2 = _u01(v[0::2]), _u01(v[1::2])
        r = np.sqrt(-2.0 * np.log(u1))
        t = 6.283185307179586 * u2
        pair = np.empty(2 * (p1 - p0), np.float64)
        pair[0::2] = mean + std * r * np.cos(t)
        pair[1::2] = mean + std * r * np.sin(t)
        lo, hi = 2 * p0, min(n, 2 * p1)
        out[lo:hi] = pair[: hi - lo]
    return out.reshape(shape)


def uniform_f32(seed: int, shape, lo: float, hi: float) -> np.ndarray:
    n = int(np.prod(shape))
    out = np.empty(n, np.float32)
    for s0 in range(0, n, _CHUNK):
        s1 = min(n, s0 + _CHUNK)
        u = (_splitmix64(seed, s0, s1 - s0) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
        out[s0:s1] = lo + (hi - lo) * u
    return out.reshape(shape)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round f32 to bf16 (nearest-even) and return the uint16 bit patterns."""
    b = np.ascontiguousarray(a, np.float32).view(np.uint32)
    with np.errstate(over="ignore"):
        r = b + np.uint32(0x8000) + ((b >> np.uint32(16)) & np.uint32(1))
    return (r >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


# The five configurations of the benchmark, as (name, description) -> inputs.
# Distributions follow the configuration table: C1 N(0,1)/sqrt(K); C2
# U(-1,1); C3/C4 X N(0,1), W N(0,0.02); C5 X N(0,1), W N(0,0.015).
CONFIGS = {
    "c1": dict(kind="swiglu", M=64, K=256, N=512, x_std=1.0 / 16.0, w_std=1.0 / 16.0, y="f32"),
    "c2": dict(kind="matmul", M=4096, K=4096, N=4096, y="f32"),
    "c3": dict(kind="swiglu", M=2048, K=4096, N=11008, x_std=1.0, w_std=0.02, y="bf16"),
    "c4_m1": dict(kind="swiglu", M=1, K=4096, N=14336, x_std=1.0, w_std=0.02, y="bf16"),
    "c4_m4": dict(kind="swiglu", M=4, K=4096, N=14336, x_std=1.0, w_std=0.02, y="bf16"),
    "c4_m16": dict(kind="swiglu", M=16, K=4096, N=14336, x_std=1.0, w_std=0.02, y="bf16"),
    "c5": dict(kind="swiglu", M=8192, K=8192, N=28672, x_std=1.0, w_std=0.015, y="bf16"),
}


def swiglu_inputs(M: int, K: int, N: int, x_std: float, w_std: float, seed: int = 42):
    """bf16 bit patterns for X[M,K], Wg[K,N], Wu[K,N] from three sub-streams."""
    x = f32_to_bf16_bits(normal_f32(seed * 3 + 0, (M, K), 0.0, x_std))
    wg = f32_to_bf16_bits(normal_f32(seed * 3 + 1, (K, N), 0.0, w_std))
    wu = f32_to_bf16_bits(normal_f32(seed * 3 + 2, (K, N), 0.0, w_std))
    return x, wg, wu


def matmul_inputs(M: int, K: int, N: int, seed: int = 42):
    a = f32_to_bf16_bits(uniform_f32(seed * 3 + 0, (M, K), -1.0, 1.0))
    b = f32_to_bf16_bits(uniform_f32(seed * 3 + 1, (K, N), -1.0, 1.0))
    return a, b


def config_inputs(name: str, seed: int = 42):
    c = CONFIGS[name]
    if c["kind"] == "matmul":
        return matmul_inputs(c["M"], c["K"], c["N"], seed)
    return swiglu_inputs(c["M"], c["K"], c["N"], c["x_std"], c["w_std"], seed)
