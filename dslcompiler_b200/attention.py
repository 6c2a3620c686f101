"""llk.rope and llk.attention on the B200 (the reference's other LLK ops,
``include/LLK/Dialect/LLKOps.td:69-131``), through the C ABI ``llk_rope`` /
``llk_attention``.

Tensors are f32 ([B, H, L, D]; position ids i64 [L]), torch CUDA tensors or
numpy arrays (host arrays are staged through the GPU).  No CPU path.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from . import capi
from .capi import check, lib
from .swiglu import _device_of, _is_torch, _stream_of, gpu_context

try:
    import torch
except Exception:  # pragma: no cover
    torch = None


def _ptr(t):
    if t is None:
        return None
    if _is_torch(t):
        if not t.is_contiguous():
            raise ValueError("llk.rope / llk.attention take contiguous tensors")
        return t.data_ptr()
    if not t.flags["C_CONTIGUOUS"]:
        raise ValueError("llk.rope / llk.attention take contiguous arrays")
    return t.ctypes.data


def _check(t, dtype_torch, dtype_np, what):
    if _is_torch(t):
        if t.dtype != dtype_torch:
            raise TypeError(f"{what} must be {dtype_torch}")
    elif not isinstance(t, np.ndarray) or t.dtype != dtype_np:
        raise TypeError(f"{what} must be a {np.dtype(dtype_np).name} array")


def _like(t, shape=None):
    if _is_torch(t):
        return torch.empty(shape or t.shape, dtype=t.dtype, device=t.device)
    return np.empty(shape or t.shape, t.dtype)


def rope(x, position_ids, *, theta: float = 10000.0, out=None, math_mode: str = "strict", stream=None,
         device=None):
    """y = RoPE(x): x [B, H, L, D] f32, position_ids [L] i64 (the op's
    operands, LLKOps.td:69-96).  ``out`` may be ``x`` (in place)."""
    _check(x, getattr(torch, "float32", None), np.float32, "x")
    _check(position_ids, getattr(torch, "int64", None), np.int64, "position_ids")
    if x.ndim != 4:
        raise ValueError("x must be [B, H, L, D]")
    B, H, L, D = x.shape
    if tuple(position_ids.shape) != (L,):
        raise ValueError(f"position_ids must be [{L}]")
    if out is None:
        out = _like(x)
    g = gpu_context(_device_of(x, device), _stream_of(x, stream), math_mode=math_mode)
    check(lib().llk_rope(_ptr(x), _ptr(position_ids), _ptr(out), B, H, L, D, float(theta), ctypes.byref(g)),
          "llk_rope")
    return out


def attention(q, k, v, *, scale: float | None = None, causal: bool = False, out=None, math_mode: str = "strict",
              stream=None, device=None):
    """O = init + softmax(scale * Q K^T [+ causal mask]) V for q [B, H, Lq, D],
    k / v [B, H, Lk, D] f32 (LLKOps.td:99-131).  ``out`` is the op's init
    operand: the result is added to it (zeros when not given).  scale
    defaults to 1/sqrt(D)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _check(t, getattr(torch, "float32", None), np.float32, n)
        if t.ndim != 4:
            raise ValueError(f"{n} must be [B, H, L, D]")
    B, H, Lq, D = q.shape
    if k.shape[:2] != (B, H) or k.shape[3] != D or tuple(v.shape) != tuple(k.shape):
        raise ValueError("k and v must be [B, H, Lk, D] with q's B, H and D")
    Lk = k.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.zeros(q.shape, dtype=q.dtype, device=q.device) if _is_torch(q) else np.zeros(q.shape, np.float32)
    g = gpu_context(_device_of(q, device), _stream_of(q, stream), math_mode=math_mode)
    check(lib().llk_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, Lq, Lk, D, float(scale), int(bool(causal)),
                              ctypes.byref(g)), "llk_attention")
    return out


__all__ = ["rope", "attention", "capi"]
