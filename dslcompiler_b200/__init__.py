"""dslcompiler_b200 -- B200 (sm_100a) backend for DSLCompiler's fused SwiGLU
and micro.mma matmul path.

    import dslcompiler_b200 as llk
    y = llk.fused_swiglu(x, wg, wu)          # bf16 torch tensors on cuda
    c = llk.matmul(a, b)                      # f32 C = A B
    pw = llk.PackedWeights(wg, wu); y = pw(x)
    y = llk.rope(x, pos); o = llk.attention(q, k, v, causal=True)   # f32 ops

All compute runs in the hand-written CUDA kernels of ``lib/libllk_b200.so``
(built by ``python -m dslcompiler_b200.build``); there is no CPU fallback.
"""
from .attention import attention, rope  # noqa: F401
from .capi import LLKError, lib  # noqa: F401
from .swiglu import (  # noqa: F401
    KernelKey,
    PackedWeights,
    cache_clear,
    cache_level_clear,
    cache_level_set_max_entries,
    cache_level_stats,
    cache_set_max_entries,
    cache_stats,
    classify_m,
    fused_swiglu,
    matmul,
    probe,
    shard_columns,
    swiglu_c_abi,
    synchronize,
    tensor2d,
    weight_key,
)

__version__ = "0.1.0"
