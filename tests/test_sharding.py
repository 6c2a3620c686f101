"""Column sharding across ranks: host logic on CPU with gloo ranks
(world sizes 2 and 3, uneven and empty shards), and the device relayout on a
GPU (shards emulated on one device)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dslcompiler_b200 import datagen as dg
from dslcompiler_b200.sharding import ColumnShardedSwiGLU, gather_columns, shard_bounds


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ref_swiglu(x, wg, wu):
    g = x.float() @ wg.float()
    u = x.float() @ wu.float()
    return g / (1 + torch.exp(-g)) * u


def _rank_main(rank, world, port, M, K, N, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0, 0.05, seed=7)
        xt, gt, ut = (torch.from_numpy(a.view(np.int16)).view(torch.bfloat16) for a in (x, wg, wu))
        layer = ColumnShardedSwiGLU(gt, ut, pack=False)
        b, e = layer.begin, layer.end
        y = layer.full(xt, out_dtype="f32", compute=lambda xx: _ref_swiglu(xx, layer.wg, layer.wu))
        ref = _ref_swiglu(xt, gt, ut)
        q.put((rank, b, e, float((y - ref).abs().max()), tuple(y.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,M,K,N", [(2, 16, 64, 300), (3, 8, 32, 130), (2, 5, 48, 1024)])
def test_gloo_column_sharding_full_output(world, M, K, N):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, M, K, N, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    spans = [(b, e) for _, b, e, _, _ in res]
    assert spans == shard_bounds(N, world)
    assert spans[0][0] == 0 and spans[-1][1] == N
    for _, _, _, err, shape in res:
        assert shape == (M, N) and err == 0.0  # exact: same fp32 arithmetic per column


def test_shard_bounds_tile_granular():
    b = shard_bounds(11008, 8)
    assert all(s % 128 == 0 for s, _ in b)
    assert [e - s for s, e in b] == [1408] * 6 + [1280] * 2


def test_cpu_gather_relayout():
    bounds = [(0, 128), (128, 200), (200, 200)]
    width = 128
    g = torch.arange(3 * 4 * width, dtype=torch.float32).reshape(3, 4, width)
    y = torch.full((4, 200), -1.0)
    gather_columns(g, bounds, y)
    assert torch.equal(y[:, :128], g[0])
    assert torch.equal(y[:, 128:200], g[1, :, :72])


@pytest.mark.gpu
def test_gpu_sharded_layers_reassemble_full_output():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import dslcompiler_b200 as llk
    M, K, N, world = 256, 512, 1000, 4
    x, wg, wu = dg.swiglu_inputs(M, K, N, 1.0, 0.05, seed=3)
    dev = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()  # noqa: E731
    xd, gd, ud = dev(x), dev(wg), dev(wu)
    full = llk.fused_swiglu(xd, gd, ud, out_dtype="f32")
    layers = [ColumnShardedSwiGLU(gd, ud, rank=r, world=world) for r in range(world)]
    width = layers[0].width
    gathered = torch.zeros((world, M, width), dtype=torch.float32, device="cuda")
    for r, L in enumerate(layers):
        w = L.end - L.begin
        if w:
            L.local(xd, out=gathered[r, :, :w], out_dtype="f32")
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    gather_columns(gathered, shard_bounds(N, world), y)
    torch.cuda.synchronize()
    llk.synchronize(0)
    # same kernel per column block: identical to the unsharded call
    assert torch.allclose(y, full, rtol=0, atol=1e-6 * full.abs().max().item())
