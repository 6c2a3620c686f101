"""Column-parallel SwiGLU across the GPUs of one node.

The op shards naturally along N: rank r owns the 128-column tiles
``llk_shard_columns(N, world, r)`` deals out (11008 -> 11,11,11,11,11,11,10,10
tiles at 8 ranks), holds Wg[:, b:e] and Wu[:, b:e] and a replica of X, and
computes Y[:, b:e] with no communication.  Only when the caller wants the full
Y does it all-gather the shards (NCCL through torch.distributed) and relay them
out with the ``llk_gather_columns`` kernel.  One process per GPU.

The reference has no multi-device path; this module is the B200 build's.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import capi
from .capi import check, lib
from .swiglu import PackedWeights, fused_swiglu, gpu_context, shard_columns

try:
    import torch
    import torch.distributed as dist
except Exception:  # pragma: no cover
    torch = None
    dist = None


def shard_bounds(N: int, world: int) -> list[tuple[int, int]]:
    """[begin, end) columns of every rank."""
    return [shard_columns(N, world, r) for r in range(world)]


class ColumnShardedSwiGLU:
    """This rank's share of a column-sharded SwiGLU layer.

    wg, wu: the FULL [K, N] weights (host or device) -- each rank keeps only
    its columns -- or, with ``already_sharded=True``, this rank's [K, e-b]
    columns.  ``pack`` stores the shard as device-resident packed weights.
    """

    def __init__(self, wg, wu, *, rank: int | None = None, world: int | None = None, group=None,
                 already_sharded: bool = False, N: int | None = None, pack: bool = True, device=None):
        self.group = group
        self.rank = rank if rank is not None else (dist.get_rank(group) if dist and dist.is_initialized() else 0)
        self.world = world if world is not None else (
            dist.get_world_size(group) if dist and dist.is_initialized() else 1)
        self.N = N if N is not None else (wg.shape[1] if not already_sharded else None)
        if self.N is None:
            raise ValueError("N (the full width) is required with already_sharded=True")
        self.bounds = shard_bounds(self.N, self.world)
        self.begin, self.end = self.bounds[self.rank]
        self.width = max(e - b for b, e in self.bounds)
        if not already_sharded:
            wg = wg[:, self.begin:self.end]
            wu = wu[:, self.begin:self.end]
        self.K = wg.shape[0]
        self.device = device
        self._packed = None
        if pack and self.end > self.begin:
            self._packed = PackedWeights(_contig(wg), _contig(wu), device=device)
            self.wg = self.wu = None
        else:
            self.wg, self.wu = wg, wu

    def local(self, x, *, out=None, out_dtype: str = "bf16"):
        """Y[:, begin:end] of this rank (no communication)."""
        if self._packed is not None:
            return self._packed(x, out=out, out_dtype=out_dtype)
        return fused_swiglu(x, self.wg, self.wu, out=out, out_dtype=out_dtype)

    def full(self, x, *, out_dtype: str = "bf16", compute=None):
        """The whole Y[M, N] on every rank: local shard, all-gather, relayout.
        ``compute`` replaces the local kernel (CPU ranks in tests)."""
        M = x.shape[0]
        dt = torch.float32 if out_dtype in ("f32", "fp32", "float32") else torch.bfloat16
        buf = torch.zeros((M, self.width), dtype=dt, device=x.device)
        w = self.end - self.begin
        if w > 0:
            if compute is not None:
                buf[:, :w] = compute(x)
            else:
                self.local(x, out=buf[:, :w], out_dtype=out_dtype)
        gathered = torch.empty((self.world, M, self.width), dtype=dt, device=x.device)
        if self.world > 1:
            try:
                dist.all_gather_into_tensor(gathered, buf, group=self.group)
            except (RuntimeError, NotImplementedError):  # backends without the fused form
                dist.all_gather(list(gathered.unbind(0)), buf, group=self.group)
        else:
            gathered[0].copy_(buf)
        y = torch.empty((M, self.N), dtype=dt, device=x.device)
        gather_columns(gathered, self.bounds, y)
        return y


class _DeviceArray:
    """A raw device buffer seen through __cuda_array_interface__ (so torch
    can view the library-owned group Y without copying)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerGroupSwiGLU:
    """Column-parallel SwiGLU whose all-gather is fused into the kernel
    (``llk_swiglu_column_parallel``): rank r computes its columns and the
    epilogue stores them into every rank's Y over NVLink, so each call
    leaves the whole Y[M, N] on every GPU with no collective launched.

    wg, wu: this rank's [K, e-b] columns (``already_sharded=True``) or the
    full [K, N] weights.  ``max_rows`` sizes the group Y buffer.  ``group``:
    the torch.distributed group over which the IPC handles are exchanged
    (any backend; gloo works).  One process per GPU, all ranks on one node.
    """

    def __init__(self, wg, wu, N: int, max_rows: int, *, out_dtype: str = "bf16", group=None,
                 already_sharded: bool = False, pack: bool = True, device: int | None = None,
                 math_mode: str = "strict"):
        self.group = group
        self.math_mode = math_mode
        self.rank = dist.get_rank(group) if dist and dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist and dist.is_initialized() else 1
        self.N, self.max_rows = N, max_rows
        self.f32 = out_dtype in ("f32", "fp32", "float32")
        self.begin, self.end = shard_columns(N, self.world, self.rank)
        if not already_sharded:
            wg = wg[:, self.begin:self.end]
            wu = wu[:, self.begin:self.end]
        self.device = device if device is not None else torch.cuda.current_device()
        self._packed = PackedWeights(_contig(wg), _contig(wu), device=self.device) if pack else None
        self.wg, self.wu = (None, None) if pack else (wg, wu)
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(capi.LLK_IPC_HANDLE_BYTES)
        g = gpu_context(self.device, None)
        el = 4 if self.f32 else 2
        check(lib().llk_peer_group_create(self.world, self.rank, max_rows * N * el, ctypes.byref(g), ctypes.byref(h),
                                          buf), "llk_peer_group_create")
        self._h = h
        mine = bytes(buf.raw)
        try:
            if self.world > 1:
                allh = [None] * self.world
                dist.all_gather_object(allh, mine, group=group)
            else:
                allh = [mine]
            check(lib().llk_peer_group_connect(self._h, b"".join(allh)), "llk_peer_group_connect")
        except Exception:
            lib().llk_peer_group_destroy(self._h)
            self._h = None
            raise

    def y(self, M: int):
        """The Y [M, N] of the last call on this rank, as a torch tensor
        viewing the library buffer (the group alternates two buffers: the
        view stays valid until the call after next)."""
        yp, yb = ctypes.c_void_p(), ctypes.c_int64()
        check(lib().llk_peer_group_y(self._h, ctypes.byref(yp), ctypes.byref(yb)), "llk_peer_group_y")
        arr = _DeviceArray(yp.value or 0, (M, self.N), "<f4" if self.f32 else "<i2")
        t = torch.as_tensor(arr, device=torch.device("cuda", self.device))
        return t if self.f32 else t.view(torch.bfloat16)

    def __call__(self, x, *, stream=None):
        """Y = SwiGLU(x, Wg, Wu) [M, N] on every rank (x replicated)."""
        from .swiglu import tensor2d
        M = x.shape[0]
        if M > self.max_rows:
            raise ValueError(f"M = {M} exceeds the group's max_rows = {self.max_rows}")
        st = stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream
        g = gpu_context(self.device, st, capi.LLK_DTYPE_FP32 if self.f32 else capi.LLK_DTYPE_BF16,
                        math_mode=self.math_mode)
        tx = tensor2d(x)
        if self._packed is not None:
            rc = lib().llk_swiglu_column_parallel(ctypes.byref(tx), None, None, self._packed._h, self.N, self._h,
                                                  ctypes.byref(g))
        else:
            tg, tu = tensor2d(self.wg), tensor2d(self.wu)
            rc = lib().llk_swiglu_column_parallel(ctypes.byref(tx), ctypes.byref(tg), ctypes.byref(tu), None, self.N,
                                                  self._h, ctypes.byref(g))
        check(rc, "llk_swiglu_column_parallel")
        return self.y(M)

    def close(self):
        """Frees the group on every rank: collective (all ranks call it), so
        no peer is still storing into this rank's buffers when they go."""
        if getattr(self, "_h", None):
            torch.cuda.synchronize(self.device)
            if self.world > 1 and dist is not None and dist.is_initialized():
                dist.barrier(group=self.group)
            lib().llk_peer_group_destroy(self._h)
            self._h = None
        if self._packed is not None:
            self._packed.close()
            self._packed = None


def gather_columns(gathered, bounds, y):
    """[world, M, width] shard-major -> row-major y[M, N].  CUDA tensors go
    through the library's kernel; CPU tensors (gloo test ranks) are copied
    slice by slice."""
    if gathered.is_cuda:
        begins = (ctypes.c_int64 * (len(bounds) + 1))(*([b for b, _ in bounds] + [bounds[-1][1]]))
        g = gpu_context(gathered.device.index, torch.cuda.current_stream(gathered.device).cuda_stream)
        check(lib().llk_gather_columns(gathered.data_ptr(), len(bounds), gathered.shape[1], gathered.shape[2], begins,
                                       y.data_ptr(), y.stride(0), gathered.element_size(), ctypes.byref(g)),
              "llk_gather_columns")
        return y
    for s, (b, e) in enumerate(bounds):
        y[:, b:e] = gathered[s, :, : e - b]
    return y


def _contig(w):
    if torch is not None and isinstance(w, torch.Tensor):
        return w.contiguous()
    return np.ascontiguousarray(w)


__all__ = ["ColumnShardedSwiGLU", "PeerGroupSwiGLU", "gather_columns", "shard_bounds", "capi"]
