"""Python face of the C ABI: the llk.fused_swiglu and micro.mma operations.

The functions mirror the reference's operator contract
(``include/LLK/Dialect/LLKOps.td:13-67`` for ``llk.fused_swiglu``: X[M,K],
Wg/Wu[K,N] bf16 -> Y[M,N], f32 accumulation; ``MicroOps.td:196-222`` for
``micro.mma``: acc += lhs x rhs) and its error behaviour (the verifier rules of
``lib/Dialect/LLK/LLKOps.cpp:42-83`` surface as ``LLKError`` with
``LLK_ERR_SHAPE``).

Every call goes through ``libllk_b200.so``; tensors on a CUDA device are
processed asynchronously on the current torch stream, host tensors / numpy
arrays are staged through the device synchronously, as the reference's CPU
kernel call is synchronous.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import capi
from .capi import GpuContext, KernelContext, Tensor2D, check, lib

try:  # torch is the device-memory / stream plumbing; the product works without it for host arrays
    import torch
except Exception:  # pragma: no cover
    torch = None


def _is_torch(t) -> bool:
    return torch is not None and isinstance(t, torch.Tensor)


def tensor2d(t) -> Tensor2D:
    """Tensor2D view of a 2-D torch tensor or numpy array (strides in elements)."""
    if _is_torch(t):
        if t.dim() != 2:
            raise ValueError("expected a 2-D tensor")
        return Tensor2D(t.data_ptr(), *t.shape, *t.stride())
    a = t
    if not isinstance(a, np.ndarray) or a.ndim != 2:
        raise ValueError("expected a 2-D torch tensor or numpy array")
    es = a.itemsize
    return Tensor2D(a.ctypes.data, a.shape[0], a.shape[1], a.strides[0] // es, a.strides[1] // es)


def _stream_of(t, stream):
    if stream is not None:
        return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
    if _is_torch(t) and t.is_cuda:
        return _current_raw_stream(t.device.index)
    return None


def _current_raw_stream(index):
    """cudaStream_t of torch's current stream on device `index` (None = the
    current device), without building a torch.cuda.Stream object."""
    if index is None:
        index = torch.cuda.current_device()
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    return raw(index) if raw is not None else torch.cuda.current_stream(index).cuda_stream


def _device_of(t, device):
    if device is not None:
        return int(device)
    if _is_torch(t) and t.is_cuda:
        return t.device.index if t.device.index is not None else torch.cuda.current_device()
    return -1


def gpu_context(device=-1, stream=None, y_dtype=capi.LLK_DTYPE_BF16, variant="auto",
                math_mode="strict") -> GpuContext:
    g = GpuContext()
    g.device = device
    g.stream = stream
    g.y_dtype = y_dtype
    if variant not in capi.VARIANTS:
        raise ValueError(f"variant must be one of {sorted(capi.VARIANTS)}")
    g.variant = capi.VARIANTS[variant]
    if math_mode not in capi.MATH_MODES:
        raise ValueError(f"math_mode must be one of {sorted(capi.MATH_MODES)}")
    g.math_mode = capi.MATH_MODES[math_mode]
    return g


def _check_bf16(*ts):
    for t in ts:
        if _is_torch(t):
            if t.dtype != torch.bfloat16:
                raise TypeError("llk.fused_swiglu operands must be bf16")
        elif isinstance(t, np.ndarray):
            if t.dtype != np.uint16:
                raise TypeError("numpy operands must hold bf16 bit patterns (uint16)")


def _new_out(like, rows, cols, f32: bool):
    if _is_torch(like):
        dt = torch.float32 if f32 else torch.bfloat16
        return torch.empty((rows, cols), dtype=dt, device=like.device)
    return np.empty((rows, cols), np.float32 if f32 else np.uint16)


def fused_swiglu(x, wg, wu, *, out=None, out_dtype: str = "bf16", variant: str = "auto", stream=None,
                 device=None, scratch=None, math_mode: str = "strict"):
    """Y = SiLU(X Wg) * (X Wu) on the B200.  out_dtype: 'bf16' (the op
    contract) or 'f32'.  math_mode: 'strict' (accurate exp, IEEE division:
    the fused lowering's epilogue), 'bounded_fast' or 'unsafe_fast' (the
    hardware's approximate exp and division).  Returns Y (``out`` when given)."""
    _check_bf16(x, wg, wu)
    f32 = out_dtype in ("f32", "fp32", "float32")
    if out is None:
        out = _new_out(x, x.shape[0], wg.shape[1], f32)
    tx, tg, tu, ty = tensor2d(x), tensor2d(wg), tensor2d(wu), tensor2d(out)
    ctx = None  # no scratch: the library's own workspace
    if scratch is not None:
        ctx = KernelContext(scratch.data_ptr(), scratch.numel() * scratch.element_size())
    g = gpu_context(_device_of(x, device), _stream_of(x, stream),
                    capi.LLK_DTYPE_FP32 if f32 else capi.LLK_DTYPE_BF16, variant, math_mode)
    rc = lib().llk_swiglu_ex(tx, tg, tu, ty, ctx, g)
    if rc:
        check(rc, "llk_swiglu_ex")
    return out


def matmul(a, b, c=None, *, accumulate: bool = False, variant: str = "auto", stream=None, device=None):
    """micro.mma: C (f32) = [C +] A B with bf16 A[M,K], B[K,N]."""
    _check_bf16(a, b)
    if c is None:
        if accumulate:
            raise ValueError("accumulate=True needs c")
        c = _new_out(a, a.shape[0], b.shape[1], True)
    ta, tb, tc = tensor2d(a), tensor2d(b), tensor2d(c)
    g = gpu_context(_device_of(a, device), _stream_of(a, stream), capi.LLK_DTYPE_FP32, variant)
    check(lib().llk_matmul(ctypes.byref(ta), ctypes.byref(tb), ctypes.byref(tc), int(accumulate), None,
                           ctypes.byref(g)), "llk_matmul")
    return c


def swiglu_c_abi(x, wg, wu, y) -> int:
    """The documented public symbol ``llk_swiglu`` (bf16 Y), returning
    ``llk_last_status()``."""
    tx, tg, tu, ty = tensor2d(x), tensor2d(wg), tensor2d(wu), tensor2d(y)
    L = lib()
    L.llk_swiglu(ctypes.byref(tx), ctypes.byref(tg), ctypes.byref(tu), ctypes.byref(ty), None)
    return L.llk_last_status()


def synchronize(device: int = -1, stream=None) -> None:
    """Wait for the stream and raise LLKError(LLK_ERR_TIMEOUT) if a kernel
    of this library gave up a bounded wait since the last check."""
    check(lib().llk_synchronize(device, stream), "llk_synchronize")


class PackedWeights:
    """Device-resident Wg/Wu laid out for the kernels' TMA boxes: the
    runtime PackedWeights (``runtime/PackedWeights.cpp:5-37``) plus the
    L4 weight cache role (``JitCache.h:143-146``) -- packed once, reused by
    every call until :meth:`repack`."""

    def __init__(self, wg, wu, *, device=None, stream=None):
        _check_bf16(wg, wu)
        self._h = ctypes.c_void_p()
        tg, tu = tensor2d(wg), tensor2d(wu)
        dev = _device_of(wg, device)
        g = gpu_context(dev, _stream_of(wg, stream))
        check(lib().llk_pack_weights(ctypes.byref(tg), ctypes.byref(tu), ctypes.byref(g), ctypes.byref(self._h)),
              "llk_pack_weights")
        K, N, B = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        check(lib().llk_packed_weights_info(self._h, ctypes.byref(K), ctypes.byref(N), ctypes.byref(B)))
        self.K, self.N, self.nbytes = K.value, N.value, B.value

    @classmethod
    def cached(cls, wg, wu, *, device=None, stream=None) -> "PackedWeights":
        """The packed pair for (wg, wu) from the library's L4 cache, keyed by
        WeightKey (the weights' pointers, shapes and strides); packed and
        inserted on a miss.  The cache keeps its own reference, so the
        device copy outlives this object until evicted (see
        :func:`cache_level_set_max_entries`).  A caller that changes the
        weights in place must :meth:`repack` -- the key does not see the
        contents."""
        key = weight_key(wg, wu)
        h = ctypes.c_void_p()
        st = lib().llk_lookup_packed_weights(ctypes.byref(key), ctypes.byref(h))
        if st == capi.LLK_OK:
            self = cls.__new__(cls)
            self._h = h
            K, N, B = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
            check(lib().llk_packed_weights_info(self._h, ctypes.byref(K), ctypes.byref(N), ctypes.byref(B)))
            self.K, self.N, self.nbytes = K.value, N.value, B.value
            return self
        if st != capi.LLK_ERR_NOT_FOUND:
            check(st, "llk_lookup_packed_weights")
        self = cls(wg, wu, device=device, stream=stream)
        check(lib().llk_insert_packed_weights(ctypes.byref(key), self._h), "llk_insert_packed_weights")
        return self

    def layout(self) -> dict:
        """Device pointers and box geometry of the packed pair."""
        L = capi.PackedLayout()
        check(lib().llk_packed_weights_layout(self._h, ctypes.byref(L)), "llk_packed_weights_layout")
        return {f: getattr(L, f) for f, _ in capi.PackedLayout._fields_}

    def repack(self, wg, wu, stream=None):
        tg, tu = tensor2d(wg), tensor2d(wu)
        g = gpu_context(-1, _stream_of(wg, stream))
        check(lib().llk_repack(self._h, ctypes.byref(tg), ctypes.byref(tu), ctypes.byref(g)), "llk_repack")

    def __call__(self, x, *, out=None, out_dtype: str = "bf16", variant: str = "auto", stream=None,
                 math_mode: str = "strict"):
        _check_bf16(x)
        f32 = out_dtype in ("f32", "fp32", "float32")
        if out is None:
            out = _new_out(x, x.shape[0], self.N, f32)
        tx, ty = tensor2d(x), tensor2d(out)
        g = gpu_context(-1, _stream_of(x, stream), capi.LLK_DTYPE_FP32 if f32 else capi.LLK_DTYPE_BF16, variant,
                        math_mode)
        check(lib().llk_swiglu_packed(ctypes.byref(tx), self._h, ctypes.byref(ty), None, ctypes.byref(g)),
              "llk_swiglu_packed")
        return out

    def close(self):
        if self._h:
            lib().llk_packed_weights_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def weight_key(wg, wu) -> capi.WeightKeyC:
    """WeightKey of a (Wg, Wu) pair (llk_weight_key_for)."""
    k = capi.WeightKeyC()
    tg, tu = tensor2d(wg), tensor2d(wu)
    check(lib().llk_weight_key_for(ctypes.byref(tg), ctypes.byref(tu), ctypes.byref(k)), "llk_weight_key_for")
    return k


def cache_level_stats(level: int) -> dict:
    """hits / misses / evictions / size of cache level 1-4 (JitCache.h
    numbering: 3 = launch plans, 4 = packed weights)."""
    h, m, e, n = (ctypes.c_uint64() for _ in range(4))
    check(lib().llk_cache_level_stats(level, ctypes.byref(h), ctypes.byref(m), ctypes.byref(e), ctypes.byref(n)),
          "llk_cache_level_stats")
    return {"hits": h.value, "misses": m.value, "evictions": e.value, "size": n.value}


def cache_level_set_max_entries(level: int, n: int) -> None:
    check(lib().llk_cache_level_set_max_entries(level, n), "llk_cache_level_set_max_entries")


def cache_level_clear(level: int) -> None:
    check(lib().llk_cache_level_clear(level), "llk_cache_level_clear")


def probe(device: int = -1) -> dict:
    """CUDA target probe (analogue of lib/Target/X86/TargetAVX2.cpp:33-92)."""
    t = capi.CudaTarget()
    check(lib().llk_cuda_probe(device, ctypes.byref(t)), "llk_cuda_probe")
    return {f: (getattr(t, f).decode() if f == "name" else getattr(t, f)) for f, _ in capi.CudaTarget._fields_}


def classify_m(M: int) -> int:
    """M bucket (lib/Transforms/Common/ScheduleLoader.cpp:19-29)."""
    return lib().llk_classify_m(M)


def shard_columns(N: int, n_shards: int, index: int) -> tuple[int, int]:
    b, e = ctypes.c_int64(), ctypes.c_int64()
    check(lib().llk_shard_columns(N, n_shards, index, ctypes.byref(b), ctypes.byref(e)), "llk_shard_columns")
    return b.value, e.value


@dataclass
class KernelKey:
    """KernelKey (include/LLK/Runtime/KernelKey.h:45-58) with isa = SM100A."""
    operation: int = capi.LLK_OP_FUSED_SWIGLU
    input_type: int = capi.LLK_DTYPE_BF16
    output_type: int = capi.LLK_DTYPE_BF16
    M_bucket: int = 0
    N: int = 0
    K: int = 0
    weight_layout: int = 0
    isa: int = capi.LLK_ISA_SM100A
    math_mode: int = 0
    thread_count: int = capi.VARIANTS["tc"]
    compiler_version: int = field(default_factory=lambda: lib().llk_version())
    schedule_version: int = 1

    def to_c(self) -> capi.KernelKeyC:
        k = capi.KernelKeyC()
        ctypes.memset(ctypes.byref(k), 0, ctypes.sizeof(k))
        for f, _ in capi.KernelKeyC._fields_:
            setattr(k, f, getattr(self, f))
        return k

    def hash(self) -> int:
        k = self.to_c()
        return lib().llk_kernel_key_hash(ctypes.byref(k))

    def insert_plan(self, **plan) -> None:
        """Install a launch plan for this key (a tuned schedule)."""
        k = self.to_c()
        p = capi.LaunchPlan()
        for f, _ in capi.LaunchPlan._fields_:
            setattr(p, f, int(plan.get(f, 0)))
        check(lib().llk_plan_insert(ctypes.byref(k), ctypes.byref(p)), "llk_plan_insert")

    def find(self) -> dict | None:
        """The cached plan, or None (lookupObjectCode: builds nothing)."""
        k = self.to_c()
        p = capi.LaunchPlan()
        st = lib().llk_plan_find(ctypes.byref(k), ctypes.byref(p))
        if st == capi.LLK_ERR_NOT_FOUND:
            return None
        check(st, "llk_plan_find")
        return {f: getattr(p, f) for f, _ in capi.LaunchPlan._fields_}

    def plan(self, M: int) -> dict:
        k = self.to_c()
        p = capi.LaunchPlan()
        check(lib().llk_plan_lookup(ctypes.byref(k), M, ctypes.byref(p)), "llk_plan_lookup")
        return {f: getattr(p, f) for f, _ in capi.LaunchPlan._fields_}


def cache_stats() -> dict:
    h, m, e = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
    lib().llk_cache_stats(ctypes.byref(h), ctypes.byref(m), ctypes.byref(e))
    return {"hits": h.value, "misses": m.value, "evictions": e.value, "size": lib().llk_cache_size()}


def cache_clear() -> None:
    lib().llk_cache_clear()


def cache_set_max_entries(n: int) -> None:
    lib().llk_cache_set_max_entries(n)
