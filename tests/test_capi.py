"""The C-ABI library: it loads, exports every symbol include/llk_b200.h
declares, and its host-side logic (argument checks, shard assignment,
kernel keys, plan cache, status strings) behaves -- without a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

import dslcompiler_b200 as llk
from dslcompiler_b200 import capi, build
from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "llk_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(llk_[a-z0-9_]+)\s*\(", src)))


def test_library_builds_and_loads():
    build.build()
    assert os.path.exists(capi.LIB_PATH)
    assert capi.lib() is not None


def test_every_declared_symbol_is_exported():
    L = ctypes.CDLL(capi.LIB_PATH)
    syms = declared_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    # and the Python binding covers all of them
    assert set(syms) <= set(capi.PROTOTYPES), set(syms) - set(capi.PROTOTYPES)


def test_struct_layouts_match_reference():
    # JitCache.h:30-62 layouts: Tensor2D 40 B, MemRef2D 56 B, KernelContext 16 B
    assert ctypes.sizeof(capi.Tensor2D) == 40
    assert ctypes.sizeof(capi.MemRef2D) == 56
    assert ctypes.sizeof(capi.KernelContext) == 16


@pytest.mark.parametrize("M,bucket", [(1, 0), (3, 1), (8, 2), (32, 3), (128, 4), (2048, 4)])
def test_classify_m(M, bucket):
    assert llk.classify_m(M) == bucket


def test_shard_columns_even_and_uneven():
    # 11008 = 86 tiles of 128 -> 11,11,11,11,11,11,10,10 at 8 shards
    widths = []
    prev = 0
    for i in range(8):
        b, e = llk.shard_columns(11008, 8, i)
        assert b == prev
        prev = e
        widths.append(e - b)
    assert prev == 11008
    assert [w // 128 for w in widths] == [11, 11, 11, 11, 11, 11, 10, 10]
    # 28672 = 224 tiles -> 28 each
    assert {llk.shard_columns(28672, 8, i)[1] - llk.shard_columns(28672, 8, i)[0] for i in range(8)} == {3584}
    # ragged N, more shards than tiles
    spans = [llk.shard_columns(130, 4, i) for i in range(4)]
    assert spans[0] == (0, 128) and spans[1] == (128, 130) and spans[2] == (130, 130) and spans[3] == (130, 130)
    with pytest.raises(llk.LLKError):
        llk.shard_columns(100, 0, 0)
    with pytest.raises(llk.LLKError):
        llk.shard_columns(100, 2, 2)


def test_kernel_key_hash_deterministic_and_field_sensitive():
    a = llk.KernelKey(N=11008, K=4096, M_bucket=4)
    b = llk.KernelKey(N=11008, K=4096, M_bucket=4)
    c = llk.KernelKey(N=11008, K=4096, M_bucket=3)
    assert a.hash() == b.hash() != c.hash()


def test_plan_cache_lru_and_stats():
    llk.cache_clear()
    llk.cache_set_max_entries(2)
    try:
        p = llk.KernelKey(N=11008, K=4096, M_bucket=4).plan(2048)
        # M = 2048 > 128: CTA-pair kernel, 256-row tiles x 128 Y columns
        assert p["variant"] == capi.VARIANTS["tc"] and p["block_m"] == 256 and p["block_n"] == 128
        assert p["grid"] % 2 == 0
        assert p["grid"] >= 1 and p["smem_bytes"] > 100 * 1024
        llk.KernelKey(N=11008, K=4096, M_bucket=4).plan(2048)
        s = llk.cache_stats()
        assert s["hits"] == 1 and s["misses"] == 1 and s["size"] == 1
        for n in (128, 256, 384):
            llk.KernelKey(N=n, K=64).plan(128)
        s = llk.cache_stats()
        assert s["size"] == 2 and s["evictions"] == 2
    finally:
        llk.cache_set_max_entries(1024)
        llk.cache_clear()


def test_pair_schedule_choice_by_waves():
    """CTA-pair plans: static round-robin below 12 waves of tiles (config 3:
    688 tiles, 9.3 waves of 74 pairs), the dynamic work counter from there
    on (config 5: 7168 tiles)."""
    llk.cache_clear()
    assert llk.KernelKey(N=11008, K=4096, M_bucket=4).plan(2048)["sched"] == 1
    assert llk.KernelKey(N=28672, K=8192, M_bucket=4).plan(8192)["sched"] == 0
    mm = llk.KernelKey(operation=capi.LLK_OP_MATMUL, N=4096, K=4096, M_bucket=4, output_type=capi.LLK_DTYPE_FP32)
    assert mm.plan(4096)["sched"] == 1
    llk.cache_clear()


def test_shape_errors_reported_before_device_use():
    # LLKOps.cpp:42-83 rules: M/K/N mismatches are LLK_ERR_SHAPE even with no GPU
    x = np.zeros((4, 8), np.uint16)
    wg = np.zeros((7, 16), np.uint16)
    wu = np.zeros((8, 16), np.uint16)
    with pytest.raises(llk.LLKError) as e:
        llk.fused_swiglu(x, wg, wu)
    assert e.value.status == capi.LLK_ERR_SHAPE
    with pytest.raises(llk.LLKError) as e:
        llk.fused_swiglu(x, wu, np.zeros((8, 15), np.uint16))
    assert e.value.status == capi.LLK_ERR_SHAPE
    y = np.zeros((4, 16), np.uint16)
    st = llk.swiglu_c_abi(x, wu, wu, np.zeros((5, 16), np.uint16))
    assert st == capi.LLK_ERR_SHAPE
    with pytest.raises(TypeError):
        llk.fused_swiglu(x.astype(np.float32), wu, wu)
    del y


def test_no_cpu_fallback_without_gpu():
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        pytest.skip("a GPU is present")
    x = np.zeros((4, 8), np.uint16)
    w = np.zeros((8, 16), np.uint16)
    with pytest.raises(llk.LLKError) as e:
        llk.fused_swiglu(x, w, w)
    assert e.value.status == capi.LLK_ERR_DEVICE
    with pytest.raises(llk.LLKError) as e:
        llk.probe(0)
    assert e.value.status == capi.LLK_ERR_DEVICE


def test_status_strings():
    for s in range(10):
        assert capi.status_string(s) != "unknown status"
    assert capi.status_string(99) == "unknown status"


def test_memref_shim_reports_status():
    L = capi.lib()
    m = capi.MemRef2D()
    L.llk_swiglu_memref(None, ctypes.byref(m), ctypes.byref(m), None, ctypes.byref(m))
    assert L.llk_last_status() == capi.LLK_ERR_ARG


def _build_c_smoke(tmp_path):
    exe = tmp_path / "c_abi_smoke"
    cmd = ["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "c_abi_smoke.c"), "-L", os.path.dirname(capi.LIB_PATH), "-lllk_b200",
           "-Wl,-rpath," + os.path.dirname(capi.LIB_PATH), "-o", str(exe)]
    import subprocess
    subprocess.run(cmd, check=True)
    return exe


def test_header_is_c_and_links(tmp_path):
    import subprocess
    exe = _build_c_smoke(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok ")


@pytest.mark.gpu
def test_c_program_runs_swiglu_on_gpu(tmp_path):
    import subprocess
    exe = _build_c_smoke(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.startswith("ok 0 "), r.stdout + r.stderr


def _build_cpp_cache_smoke(tmp_path):
    import subprocess
    exe = tmp_path / "jitcache_smoke"
    cmd = ["g++", "-std=c++17", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "jitcache_smoke.cpp"), "-L", os.path.dirname(capi.LIB_PATH), "-lllk_b200",
           "-Wl,-rpath," + os.path.dirname(capi.LIB_PATH), "-o", str(exe)]
    subprocess.run(cmd, check=True)
    return exe


def test_jitcache_header_plan_levels(tmp_path):
    """llk_b200_jitcache.hpp: JitCache's method names over the C ABI (L3
    plans, L1/L2 always missing, L4 miss) from a C++ program."""
    import subprocess
    r = subprocess.run([str(_build_cpp_cache_smoke(tmp_path))], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr


@pytest.mark.gpu
def test_jitcache_header_packed_weights_on_gpu(tmp_path):
    import subprocess
    r = subprocess.run([str(_build_cpp_cache_smoke(tmp_path)), "gpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr


def test_weight_key_and_l4_miss():
    """WeightKey of a pair: pointer of Wg, a hash that changes with shape,
    strides and Wu, BK = BN = 64; an empty L4 misses."""
    wg = np.zeros((8, 128), np.uint16)
    wu = np.zeros((8, 128), np.uint16)
    k1 = llk.weight_key(wg, wu)
    assert k1.weight_ptr == wg.ctypes.data and k1.BK == 64 and k1.BN == 64
    assert llk.weight_key(wg, wu).shape_hash == k1.shape_hash
    assert llk.weight_key(wg, np.zeros((8, 128), np.uint16)).shape_hash != k1.shape_hash
    assert llk.weight_key(wg[:, :64], wu[:, :64]).shape_hash != k1.shape_hash
    llk.cache_level_clear(4)
    h = ctypes.c_void_p()
    assert capi.lib().llk_lookup_packed_weights(ctypes.byref(k1), ctypes.byref(h)) == capi.LLK_ERR_NOT_FOUND
    s = llk.cache_level_stats(4)
    assert s["misses"] == 1 and s["size"] == 0
    assert llk.cache_level_stats(1) == {"hits": 0, "misses": 0, "evictions": 0, "size": 0}
    with pytest.raises(capi.LLKError):
        llk.cache_level_stats(5)


def test_plan_find_is_pure_lookup():
    llk.cache_clear()
    key = llk.KernelKey(N=640, K=256, M_bucket=4)
    assert key.find() is None
    p = key.plan(300)
    assert key.find() == p
    llk.cache_clear()
