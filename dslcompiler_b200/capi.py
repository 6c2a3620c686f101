"""ctypes binding of the C ABI in ``include/llk_b200.h``.

Loads the in-tree ``lib/libllk_b200.so``.  There is no fallback: if the
library is missing or cannot be loaded, :func:`lib` raises, so no caller can
silently end up on a CPU or eager-PyTorch path.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libllk_b200.so")

# enum llk_status_code
LLK_OK = 0
LLK_ERR_SHAPE = 1
LLK_ERR_ALIGN = 2
LLK_ERR_CUDA = 3
LLK_ERR_NCCL = 4
LLK_ERR_TIMEOUT = 5
LLK_ERR_ARG = 6
LLK_ERR_DEVICE = 7
LLK_ERR_UNSUPPORTED = 8
LLK_ERR_NOMEM = 9
LLK_ERR_NOT_FOUND = 10
LLK_IPC_HANDLE_BYTES = 64

# include/llk_b200.h: the no-allocation decode entry point's limits
LLK_DECODE_NOALLOC_SCRATCH_BYTES = 16 << 20
LLK_DECODE_NOALLOC_MAX_N = 65536 * 128

# enum llk_dtype (KernelKey.h DType)
LLK_DTYPE_BF16 = 0
LLK_DTYPE_FP16 = 1
LLK_DTYPE_FP32 = 2

# enum llk_math_mode (KernelKey.h MathMode; the op's math_mode attribute)
LLK_MATH_STRICT = 0
LLK_MATH_BOUNDED_FAST = 1
LLK_MATH_UNSAFE_FAST = 2
MATH_MODES = {"strict": LLK_MATH_STRICT, "bounded_fast": LLK_MATH_BOUNDED_FAST, "unsafe_fast": LLK_MATH_UNSAFE_FAST}

# enum llk_variant
VARIANTS = {"auto": 0, "tc": 1, "decode": 2, "simt": 3}

LLK_OP_FUSED_SWIGLU = 0
LLK_OP_MATMUL = 3
LLK_ISA_SM100A = 16


class Tensor2D(ctypes.Structure):
    """include/LLK/Runtime/JitCache.h:30-36."""
    _fields_ = [("data", ctypes.c_void_p), ("dim0", ctypes.c_int64), ("dim1", ctypes.c_int64),
                ("stride0", ctypes.c_int64), ("stride1", ctypes.c_int64)]


class MemRef2D(ctypes.Structure):
    """include/LLK/Runtime/JitCache.h:42-50."""
    _fields_ = [("allocated", ctypes.c_void_p), ("aligned", ctypes.c_void_p), ("offset", ctypes.c_int64),
                ("size0", ctypes.c_int64), ("size1", ctypes.c_int64), ("stride0", ctypes.c_int64),
                ("stride1", ctypes.c_int64)]


class KernelContext(ctypes.Structure):
    """include/LLK/Runtime/JitCache.h:59-62."""
    _fields_ = [("scratch", ctypes.c_void_p), ("scratch_size", ctypes.c_size_t)]


class GpuContext(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("stream", ctypes.c_void_p), ("y_dtype", ctypes.c_int),
                ("variant", ctypes.c_int), ("math_mode", ctypes.c_int), ("reserved", ctypes.c_int * 3)]


class CudaTarget(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("cc_major", ctypes.c_int), ("cc_minor", ctypes.c_int),
                ("sm_count", ctypes.c_int), ("max_smem_per_block_optin", ctypes.c_int),
                ("global_mem_bytes", ctypes.c_int64), ("l2_bytes", ctypes.c_int), ("clock_khz", ctypes.c_int),
                ("name", ctypes.c_char * 96), ("is_sm100a", ctypes.c_int)]


class KernelKeyC(ctypes.Structure):
    """KernelKey (include/LLK/Runtime/KernelKey.h:45-58), natural C layout."""
    _fields_ = [("operation", ctypes.c_uint8), ("input_type", ctypes.c_uint8), ("output_type", ctypes.c_uint8),
                ("M_bucket", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
                ("weight_layout", ctypes.c_uint8), ("isa", ctypes.c_uint8), ("math_mode", ctypes.c_uint8),
                ("thread_count", ctypes.c_uint16), ("compiler_version", ctypes.c_uint64),
                ("schedule_version", ctypes.c_uint64)]


class WeightKeyC(ctypes.Structure):
    """WeightKey (include/LLK/Runtime/KernelKey.h:112-124)."""
    _fields_ = [("weight_ptr", ctypes.c_void_p), ("shape_hash", ctypes.c_uint64), ("BK", ctypes.c_int64),
                ("BN", ctypes.c_int64)]


class PackedLayout(ctypes.Structure):
    _fields_ = [("wg", ctypes.c_void_p), ("wu", ctypes.c_void_p), ("device", ctypes.c_int), ("box_n", ctypes.c_int),
                ("box_k", ctypes.c_int), ("slab_stride_bytes", ctypes.c_int64)]


class LaunchPlan(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("variant", "block_m", "block_n", "block_k", "stages", "split_k", "grid",
                                            "threads", "smem_bytes", "sched")]


# Every exported symbol with its prototype: (restype, argtypes).
_P = ctypes.POINTER
_vp, _i, _i64, _u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint64
PROTOTYPES = {
    "llk_swiglu": (None, [_P(Tensor2D), _P(Tensor2D), _P(Tensor2D), _P(Tensor2D), _P(KernelContext)]),
    "llk_swiglu_ex": (_i, [_P(Tensor2D), _P(Tensor2D), _P(Tensor2D), _P(Tensor2D), _P(KernelContext),
                           _P(GpuContext)]),
    "llk_swiglu_memref": (None, [_P(MemRef2D)] * 5),
    "llk_matmul": (_i, [_P(Tensor2D), _P(Tensor2D), _P(Tensor2D), _i, _P(KernelContext), _P(GpuContext)]),
    "llk_rope": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_double, _P(GpuContext)]),
    "llk_attention": (_i, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _i, _P(GpuContext)]),
    "llk_last_status": (_i, []),
    "llk_status_string": (ctypes.c_char_p, [_i]),
    "llk_synchronize": (_i, [_i, _vp]),
    "llk_diag_timeout_probe": (_i, [_i, _i64]),
    "llk_diag_reciprocal_check": (_i, [_i, ctypes.c_uint32, ctypes.c_uint32, _P(_u64)]),
    "llk_diag_pair_schedule": (_i, [_i, _i64, _i64, _i64, _i, _i, _i, _P(ctypes.c_int32), _i, _P(_i), _P(_i), _P(_i),
                                    _P(_i)]),
    "llk_swiglu_decode_noalloc": (_i, [_P(Tensor2D), _P(Tensor2D), _P(Tensor2D), _P(Tensor2D), _vp,
                                      _P(GpuContext)]),
    "llk_pack_weights": (_i, [_P(Tensor2D), _P(Tensor2D), _P(GpuContext), _P(_vp)]),
    "llk_repack": (_i, [_vp, _P(Tensor2D), _P(Tensor2D), _P(GpuContext)]),
    "llk_packed_weights_free": (None, [_vp]),
    "llk_packed_weights_info": (_i, [_vp, _P(_i64), _P(_i64), _P(_i64)]),
    "llk_swiglu_packed": (_i, [_P(Tensor2D), _vp, _P(Tensor2D), _P(KernelContext), _P(GpuContext)]),
    "llk_packed_weights_layout": (_i, [_vp, _P(PackedLayout)]),
    "llk_weight_key_for": (_i, [_P(Tensor2D), _P(Tensor2D), _P(WeightKeyC)]),
    "llk_lookup_packed_weights": (_i, [_P(WeightKeyC), _P(_vp)]),
    "llk_insert_packed_weights": (_i, [_P(WeightKeyC), _vp]),
    "llk_shard_columns": (_i, [_i64, _i, _i, _P(_i64), _P(_i64)]),
    "llk_gather_columns": (_i, [_vp, _i, _i64, _i64, _P(_i64), _vp, _i64, _i, _P(GpuContext)]),
    "llk_cuda_probe": (_i, [_i, _P(CudaTarget)]),
    "llk_peer_group_create": (_i, [_i, _i, _i64, _P(GpuContext), _P(_vp), ctypes.c_char_p]),
    "llk_peer_group_connect": (_i, [_vp, ctypes.c_char_p]),
    "llk_peer_group_y": (_i, [_vp, _P(_vp), _P(_i64)]),
    "llk_peer_group_destroy": (None, [_vp]),
    "llk_swiglu_column_parallel": (_i, [_P(Tensor2D), _P(Tensor2D), _P(Tensor2D), _vp, _i64, _vp, _P(GpuContext)]),
    "llk_kernel_key_hash": (_u64, [_P(KernelKeyC)]),
    "llk_plan_lookup": (_i, [_P(KernelKeyC), _i64, _P(LaunchPlan)]),
    "llk_plan_insert": (_i, [_P(KernelKeyC), _P(LaunchPlan)]),
    "llk_plan_find": (_i, [_P(KernelKeyC), _P(LaunchPlan)]),
    "llk_cache_level_stats": (_i, [_i, _P(_u64), _P(_u64), _P(_u64), _P(_u64)]),
    "llk_cache_level_set_max_entries": (_i, [_i, _u64]),
    "llk_cache_level_clear": (_i, [_i]),
    "llk_cache_stats": (None, [_P(_u64), _P(_u64), _P(_u64)]),
    "llk_cache_set_max_entries": (None, [_u64]),
    "llk_cache_clear": (None, []),
    "llk_cache_size": (_u64, []),
    "llk_classify_m": (_i, [_i64]),
    "llk_version": (_u64, []),
}

_lib = None
_lock = threading.Lock()


class LLKError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = status_string(status) if _lib is not None else str(status)
        super().__init__(f"{what}: {msg} (status {status})" if what else f"{msg} (status {status})")


def lib() -> ctypes.CDLL:
    """The loaded C-ABI library.  Raises if it was not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m dslcompiler_b200.build` "
                        "(there is no CPU fallback)")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in PROTOTYPES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def status_string(status: int) -> str:
    return lib().llk_status_string(status).decode()


def check(status: int, what: str = "") -> None:
    if status != LLK_OK:
        raise LLKError(status, what)
