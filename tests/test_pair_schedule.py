"""The CTA-pair kernel's work split, enumerated on the host through
llk_diag_pair_schedule (the launch's own planner and the item mapping the
kernel runs; no GPU needed).

Whatever the split -- whole-tile waves, leftover tiles cut along N into 2 or
4 column parts, or along K into s parts whose partial sums are exchanged --
every (row tile, column, k-block) of the problem must be computed exactly
once, the K parts of a tile must cover its k-blocks in part order, and the
static schedule must give no pair more than one K part, always as its last
item (the K-split epilogue reuses the pipeline ring once the pair's loads
are done).
"""
import ctypes

import numpy as np
import pytest

from dslcompiler_b200 import capi

PAIRS_B200 = 74


def schedule(swiglu, M, N, K, pairs=PAIRS_B200, tail_split=0, dynamic=0):
    L = capi.lib()
    n_items, n_pairs, ks, ts = (ctypes.c_int() for _ in range(4))
    st = L.llk_diag_pair_schedule(swiglu, M, N, K, pairs, tail_split, dynamic, None, 0, ctypes.byref(n_items),
                                  ctypes.byref(n_pairs), ctypes.byref(ks), ctypes.byref(ts))
    assert st == capi.LLK_OK
    buf = (ctypes.c_int32 * (9 * n_items.value))()
    st = L.llk_diag_pair_schedule(swiglu, M, N, K, pairs, tail_split, dynamic, buf, n_items.value,
                                  ctypes.byref(n_items), ctypes.byref(n_pairs), ctypes.byref(ks), ctypes.byref(ts))
    assert st == capi.LLK_OK
    items = np.frombuffer(buf, dtype=np.int32).reshape(-1, 9).copy()
    return items, n_pairs.value, ks.value, ts.value


def check_cover(items, swiglu, M, N, K):
    tile_n = 128 if swiglu else 256
    m_tiles, n_tiles, kb = -(-M // 256), -(-N // tile_n), -(-K // 64)
    count = np.zeros((m_tiles, n_tiles, tile_n, kb), np.int32)
    for pair, mt, nt, c0, wn, kb0, kb1, part, nparts in items:
        assert 0 <= mt < m_tiles and 0 <= nt < n_tiles
        assert 0 <= c0 and c0 + wn <= tile_n and wn > 0
        assert 0 <= kb0 < kb1 <= kb
        assert 0 <= part < nparts
        count[mt, nt, c0:c0 + wn, kb0:kb1] += 1
    assert (count == 1).all(), "a (tile, column, k-block) computed zero or several times"


SHAPES = [
    (1, 2048, 4096, 11008),   # config 3, one GPU
    (1, 2048, 4096, 5504),    # its column shards at 2 / 4 / 8 GPUs
    (1, 2048, 4096, 2816),
    (1, 2048, 4096, 2688),
    (1, 2048, 4096, 1408),
    (1, 2048, 4096, 1280),
    (1, 8192, 8192, 28672),   # config 5
    (0, 4096, 4096, 4096),    # config 2 (matmul)
    (1, 64, 256, 512),        # config 1
    (1, 300, 512, 1000),      # ragged
    (0, 257, 4096, 100),
]


@pytest.mark.parametrize("swiglu,M,K,N", SHAPES)
def test_every_tile_column_and_kblock_exactly_once(swiglu, M, K, N):
    items, n_pairs, ks, ts = schedule(swiglu, M, N, K)
    check_cover(items, swiglu, M, N, K)
    assert 1 <= n_pairs <= PAIRS_B200
    per_pair = np.bincount(items[:, 0], minlength=n_pairs)
    assert (per_pair >= 1).all(), "a launched pair without work"
    if ks:
        assert ts == 1
        kparts = items[items[:, 8] > 1]
        # one K part per pair at most, and it is that pair's last item
        assert len(np.unique(kparts[:, 0])) == len(kparts)
        last = {int(p): i for i, p in enumerate(items[:, 0])}
        for i in np.nonzero(items[:, 8] > 1)[0]:
            assert last[int(items[i, 0])] == i
        # the parts of each tile cover its k-blocks in part order
        kb = -(-K // 64)
        for (mt, nt), grp in _group(kparts):
            grp = grp[np.argsort(grp[:, 7])]
            assert grp[0, 5] == 0 and grp[-1, 6] == kb
            assert (grp[1:, 5] == grp[:-1, 6]).all()


def _group(items):
    keys = {}
    for row in items:
        keys.setdefault((int(row[1]), int(row[2])), []).append(row)
    return [(k, np.array(v)) for k, v in keys.items()]


def test_config3_and_8gpu_shard_use_the_k_split():
    """The measured choices: config 3 (688 tiles = 9 waves + 22) cuts its
    leftover tiles along K in 3, the 1408-column shard (88 = 1 wave + 14) in 5."""
    assert schedule(1, 2048, 11008, 4096)[2] == 3
    assert schedule(1, 2048, 1408, 4096)[2] == 5
    assert schedule(0, 4096, 4096, 4096)[2] == 2


@pytest.mark.parametrize("tail_split", [1, 2, 4, -2, -3, -8])
@pytest.mark.parametrize("pairs", [74, 37, 10])
def test_forced_splits_and_grid_sizes(tail_split, pairs):
    for swiglu, M, K, N in [(1, 2048, 4096, 11008), (1, 2048, 4096, 1408), (0, 1024, 1024, 1024)]:
        items, n_pairs, ks, ts = schedule(swiglu, M, N, K, pairs=pairs, tail_split=tail_split)
        check_cover(items, swiglu, M, N, K)
        assert n_pairs <= pairs
        if tail_split > 0:
            assert ks == 0 and ts == tail_split
        else:
            # a K split that fits is taken as asked; one that does not (more
            # parts than pairs, or than k-blocks) falls back to the launch's
            # own choice
            tile_n = 128 if swiglu else 256
            tiles = -(-M // 256) * -(-N // tile_n)
            left = tiles % pairs
            fits = 0 < left and left * -tail_split <= pairs and -tail_split <= -(-K // 64)
            if fits:
                assert ks == -tail_split


def test_dynamic_schedule_never_splits_along_k():
    items, n_pairs, ks, ts = schedule(1, 2048, 11008, 4096, dynamic=1)
    assert ks == 0 and (items[:, 0] == -1).all()
    check_cover(items, 1, 2048, 11008, 4096)


def test_bad_arguments():
    n = ctypes.c_int()
    L = capi.lib()
    assert L.llk_diag_pair_schedule(1, 0, 128, 64, 74, 0, 0, None, 0, ctypes.byref(n), ctypes.byref(n),
                                    ctypes.byref(n), ctypes.byref(n)) == capi.LLK_ERR_ARG
    assert L.llk_diag_pair_schedule(1, 128, 128, 64, 74, 0, 0, None, 0, None, ctypes.byref(n),
                                    ctypes.byref(n), ctypes.byref(n)) == capi.LLK_ERR_ARG
