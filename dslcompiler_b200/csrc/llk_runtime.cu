// llk_runtime.cu -- host side of the C ABI declared in include/llk_b200.h:
// argument checks (the llk.fused_swiglu verifier rules), kernel selection,
// TMA descriptor encoding, host<->device staging for host buffers, the
// packed-weight store, the launch-plan cache and the device probe.
//
// Host code only; the kernels live in swiglu_tc.cu, swiglu_decode.cu and
// swiglu_simt.cu.  No CPU compute path exists: every result is produced by a
// CUDA kernel.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <list>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "attention_kernels.h"
#include "decode_kernels.h"
#include "llk_b200.h"
#include "tc_kernels.h"
#include "workspace.h"

using namespace llk_b200;

namespace {

constexpr uint64_t kLibraryVersion = 0x00010000ull;  // 0.1.0
constexpr int kMaxDevices = 64;

thread_local int g_last_status = LLK_OK;

// ------------------------------------------------------------ device state
struct DeviceBuffer {
  void *ptr = nullptr;
  size_t bytes = 0;
  // Grows the buffer to at least `need` bytes; a new buffer is zero-filled
  // when `zero` is set.
  cudaError_t ensure(size_t need, bool zero = false) {
    if (need <= bytes) return cudaSuccess;
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
    size_t alloc = need + need / 8;
    cudaError_t e = cudaMalloc(&ptr, alloc);
    if (e == cudaSuccess) bytes = alloc;
    if (e == cudaSuccess && zero) e = cudaMemset(ptr, 0, alloc);
    return e;
  }
};

struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  int *status = nullptr;       // device error word written by the kernels
  DeviceBuffer stage[4];       // host-staging buffers: x, wg, wu, y
  DeviceBuffer workspace;      // split-K partials when the caller gives no scratch
  // Pipelined host-buffer SwiGLU: double-buffered weight / Y column chunks,
  // a copy-in and a copy-out stream, and their events.
  DeviceBuffer chunk_w[2][2];  // [buffer][gate, up]
  DeviceBuffer chunk_y[2];
  DeviceBuffer chunk_x[2];
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  cudaEvent_t ev_x = nullptr, ev_in[2] = {nullptr, nullptr}, ev_k[2] = {nullptr, nullptr},
              ev_out[2] = {nullptr, nullptr};
  std::mutex mu;
};

DeviceState g_dev[kMaxDevices];
std::mutex g_init_mu;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int resolve_device(const llk_gpu_context *gpu, int *dev_out) {
  int dev = gpu ? gpu->device : -1;
  if (dev < 0) {
    if (cudaGetDevice(&dev) != cudaSuccess) return LLK_ERR_DEVICE;
  }
  if (dev >= kMaxDevices) return LLK_ERR_ARG;
  *dev_out = dev;
  return LLK_OK;
}

// Puts the caller's current device back when an entry point returns
// (device_init makes the call's device current).
struct DeviceRestore {
  int prev = -1;
  DeviceRestore() {
    if (cudaGetDevice(&prev) != cudaSuccess) {
      cudaGetLastError();
      prev = -1;
    }
  }
  ~DeviceRestore() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// Makes `dev` current and initialises its state once.
int device_init(int dev, DeviceState **out) {
  if (dev >= 0 && dev < kMaxDevices && g_dev[dev].ready) {  // fast path: no driver queries
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || (cur != dev && cudaSetDevice(dev) != cudaSuccess))
      return LLK_ERR_DEVICE;
    *out = &g_dev[dev];
    return LLK_OK;
  }
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
    cudaGetLastError();
    return LLK_ERR_DEVICE;
  }
  if (dev >= count) return LLK_ERR_ARG;
  if (cudaSetDevice(dev) != cudaSuccess) return LLK_ERR_DEVICE;
  DeviceState &s = g_dev[dev];
  std::lock_guard<std::mutex> lk(g_init_mu);
  if (!s.ready) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return LLK_ERR_DEVICE;
    s.cc_major = prop.major;
    s.cc_minor = prop.minor;
    s.sm_count = prop.multiProcessorCount;
    if (prop.major != 10 || prop.minor != 0) return LLK_ERR_DEVICE;  // sm_100 only
    if (cudaMalloc(&s.status, sizeof(int)) != cudaSuccess) return LLK_ERR_CUDA;
    if (cudaMemset(s.status, 0, sizeof(int)) != cudaSuccess) return LLK_ERR_CUDA;
    if (!g_encode) {
      void *fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || fn == nullptr)
        return LLK_ERR_DEVICE;
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    s.ready = true;
  }
  *out = &s;
  return LLK_OK;
}

// Where a buffer lives, from one pointer query: 0 = host (or unknown to
// CUDA), 1 = device memory of `dev` or managed memory, -1 = device memory
// of another GPU (the kernels on `dev` would fault on it unless peer access
// happens to be enabled, so the entry points that launch on `dev` refuse it).
int locate_ptr(const void *p, int dev) {
  if (!p) return 0;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (a.type == cudaMemoryTypeManaged) return 1;
  if (a.type != cudaMemoryTypeDevice) return 0;
  return a.device == dev ? 1 : -1;
}

bool is_device_ptr(const void *p) {
  if (!p) return false;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// Device memory of a GPU other than `dev` (managed memory is not): the
// kernels on `dev` would fault on it unless peer access happens to be
// enabled, so the entry points that launch on `dev` refuse it.
bool on_other_device(const void *p, int dev) {
  if (!p) return false;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice && a.device != dev;
}

// 2-D bf16 tensor map: dims {inner, outer}, row pitch in bytes, box
// {box_inner, box_outer}, 128-byte swizzle, zero fill out of bounds.
int encode_tmap(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer, uint64_t pitch_bytes,
                uint32_t box_inner, uint32_t box_outer) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LLK_OK : LLK_ERR_ALIGN;
}

// Store map of an output Y [M, N] (row pitch N elements) for the staged TMA
// stores of the CTA-pair epilogue: box {32, 32}; bf16 rows of a box are 64
// bytes (64-byte swizzle), f32 rows 128 bytes (128-byte swizzle).
int encode_ystore_map(CUtensorMap *m, void *base, uint64_t N, uint64_t M, int y_f32) {
  const uint64_t el = y_f32 ? 4 : 2;
  cuuint64_t dims[2] = {N, M};
  cuuint64_t strides[1] = {N * el};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, y_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        y_f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LLK_OK : LLK_ERR_ALIGN;
}

// Slab-major packed weights ([N/64][K][64] bf16, see llk_pack_weights) as a
// 3-D tensor map {64, K, N/64} with a {64, 64, 1} box: every box is one
// contiguous 8 KB block.
int encode_tmap_slabs(CUtensorMap *m, const void *base, uint64_t K, uint64_t n_slabs) {
  cuuint64_t dims[3] = {64, K, n_slabs};
  cuuint64_t strides[2] = {128, K * 128};
  cuuint32_t box[3] = {64, 64, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LLK_OK : LLK_ERR_ALIGN;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------- plan cache
struct PlanCache {
  struct Entry {
    std::string key;
    llk_launch_plan plan;
  };
  std::list<Entry> lru;
  std::unordered_map<std::string, std::list<Entry>::iterator> index;
  size_t max_entries = 1024;
  uint64_t hits = 0, misses = 0, evictions = 0;
  std::mutex mu;
};
PlanCache g_cache;

std::string key_bytes(const llk_kernel_key &k) {
  return std::string(reinterpret_cast<const char *>(&k), sizeof(k));
}

llk_kernel_key make_key(int op, int out_dtype, int64_t M, int64_t N, int64_t K, int variant) {
  llk_kernel_key k;
  std::memset(&k, 0, sizeof(k));
  k.operation = static_cast<uint8_t>(op);
  k.input_type = LLK_DTYPE_BF16;
  k.output_type = static_cast<uint8_t>(out_dtype);
  k.M_bucket = llk_classify_m(M);
  k.N = N;
  k.K = K;
  k.weight_layout = 0;
  k.isa = LLK_ISA_SM100A;
  k.math_mode = 0;  // strict exp, the fused path's epilogue
  k.thread_count = static_cast<uint16_t>(variant);
  k.compiler_version = kLibraryVersion;
  k.schedule_version = 1;
  return k;
}

// Kernel family for a request: the decode kernel for small M when its
// shape rules hold, the tcgen05 kernel otherwise; SIMT when TMA cannot
// describe the operands.
// A call's kernel request: the variant (enum llk_variant) in the low byte,
// the math mode (enum llk_math_mode) in the next, as carried from the
// llk_gpu_context through the staging and pipelining helpers.
int pack_request(const llk_gpu_context *gpu) {
  return gpu ? ((gpu->variant & 0xff) | ((gpu->math_mode & 0xff) << 8)) : LLK_VARIANT_AUTO;
}
int request_variant(int request) { return request & 0xff; }
int request_math_mode(int request) { return (request >> 8) & 0xff; }

int choose_variant(int requested, bool tma_ok, bool decode_ok, int64_t M, int64_t K) {
  if (requested == LLK_VARIANT_SIMT) return LLK_VARIANT_SIMT;
  if (!tma_ok || K == 0) return requested == LLK_VARIANT_AUTO ? LLK_VARIANT_SIMT : -1;
  if (requested == LLK_VARIANT_TC) return LLK_VARIANT_TC;
  if (requested == LLK_VARIANT_DECODE) return decode_ok ? LLK_VARIANT_DECODE : -1;
  if (decode_ok && M <= decode_max_m()) return LLK_VARIANT_DECODE;
  return LLK_VARIANT_TC;
}

llk_launch_plan build_plan(int variant, int op, int64_t M, int64_t N, int64_t K, int sm_count) {
  llk_launch_plan p;
  std::memset(&p, 0, sizeof(p));
  p.variant = variant;
  if (variant == LLK_VARIANT_TC) {
    const int mode = (op == LLK_OP_MATMUL) ? TC_MATMUL_F32 : TC_SWIGLU_BF16;
    // CTA pairs (256-row MMAs) once there are two row blocks; one CTA below.
    const bool pair = M > 128;
    p.block_m = pair ? 256 : 128;
    p.block_n = tc_tile_n(mode);
    p.block_k = 64;
    p.stages = pair ? 6 : 4;
    p.split_k = pair ? 0 : 1;  // pair kernel: 0 = choose the tail split
    const int64_t tiles = ((M + p.block_m - 1) / p.block_m) * ((N + p.block_n - 1) / p.block_n);
    // Static round-robin below 12 waves of tiles, the launch-wide work
    // counter from there on.  Measured on B200 in interleaved A/B: static is
    // 2-6 % faster for 3-9 waves (configs 2 and 3, 8-GPU shards); over many
    // waves static pairs drift apart, so the pairs sharing a weight tile no
    // longer read it from L2 together (M = K = 8192, N = 28672, 97 waves:
    // 4.8 GB of DRAM reads with the counter, 9.5 GB static; +6 % speed).
    p.sched = (pair && tiles >= 12 * (sm_count / 2)) ? 0 : 1;
    const int64_t ctas = pair ? 2 * tiles : tiles;
    p.grid = static_cast<int>(ctas < sm_count ? ctas : sm_count);
    if (pair) p.grid &= ~1;
    p.threads = tc_threads();
    p.smem_bytes = pair ? tc2_smem_bytes() : tc_smem_bytes();
  } else if (variant == LLK_VARIANT_DECODE) {
    DecodePlan d = decode_plan(M, N, K, sm_count);
    p.block_m = d.block_m;
    p.block_n = d.block_n;
    p.block_k = d.block_k;
    p.stages = d.stages;
    p.split_k = d.split_k;
    p.grid = d.grid;
    p.threads = d.threads;
    p.smem_bytes = d.smem_bytes;
    p.sched = d.cluster ? 1 : 0;  // decode: 1 = one cluster of split_k CTAs per tile
  } else {
    p.block_m = 1;
    p.block_n = 256;
    p.block_k = 1;
    p.stages = 1;
    p.split_k = 1;
    p.grid = static_cast<int>(((N + 255) / 256) * (M > 0 ? M : 1));
    p.threads = 256;
  }
  return p;
}

llk_launch_plan plan_for(const llk_kernel_key &key, int64_t M, int sm_count) {
  const std::string kb = key_bytes(key);
  {
    std::lock_guard<std::mutex> lk(g_cache.mu);
    auto it = g_cache.index.find(kb);
    if (it != g_cache.index.end()) {
      ++g_cache.hits;
      g_cache.lru.splice(g_cache.lru.begin(), g_cache.lru, it->second);
      return it->second->plan;
    }
    ++g_cache.misses;
  }
  llk_launch_plan plan = build_plan(key.thread_count, key.operation, M, key.N, key.K, sm_count);
  std::lock_guard<std::mutex> lk(g_cache.mu);
  if (g_cache.index.find(kb) == g_cache.index.end()) {
    g_cache.lru.push_front({kb, plan});
    g_cache.index[kb] = g_cache.lru.begin();
    while (g_cache.lru.size() > g_cache.max_entries) {
      g_cache.index.erase(g_cache.lru.back().key);
      g_cache.lru.pop_back();
      ++g_cache.evictions;
    }
  }
  return plan;
}

// ------------------------------------------------------- device launches
struct DevTensor {
  const void *data;
  int64_t rows, cols, ld, inner;  // ld = row stride, inner = column stride (elements)
  int slab_major = 0;             // weights only: slab-major packed layout
};

// TMA map for a weight operand: 2-D over row-major [K, N] or 3-D over the
// slab-major packed layout.
int encode_weight_tmap(CUtensorMap *m, const DevTensor &w) {
  if (w.slab_major) return encode_tmap_slabs(m, w.data, static_cast<uint64_t>(w.rows), (w.cols + 63) / 64);
  return encode_tmap(m, w.data, w.cols, w.rows, w.ld * 2, 64, 64);
}

// Y = SwiGLU(X, Wg, Wu) or C (+)= A B on device tensors.  op: LLK_OP_*.
// Called with ds.mu held (it guards the staging buffers and the workspace).
// Other GPUs' Y buffers (mapped here) that receive the same output columns.
struct PeerTargets {
  int n = 0;
  void *y[kMaxYPeers] = {};
  const YStoreMaps *maps = nullptr;  // TMA store maps (own Y first), when the rows allow them
};

// peers: when set, the CTA-pair kernel also stores every Y chunk to each
// peer (fused all-gather) and *peers_done is set; other variants leave the
// copies to the caller.
int launch_device(DeviceState &ds, int op, const DevTensor &x, const DevTensor &wg, const DevTensor &wu,
                  const DevTensor &y, int y_f32, int accumulate, int requested, void *scratch, size_t scratch_bytes,
                  cudaStream_t stream, const PeerTargets *peers = nullptr, bool *peers_done = nullptr) {
  const int64_t M = x.rows, K = x.cols, N = wg.cols;
  if (M == 0 || N == 0) return LLK_OK;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return LLK_ERR_SHAPE;
  const bool swiglu = (op == LLK_OP_FUSED_SWIGLU);
  const bool slab = wg.slab_major != 0;
  auto weight_ok = [&](const DevTensor &w) {
    return w.slab_major || (w.inner == 1 && aligned16(w.data) && (w.ld * 2) % 16 == 0 && w.ld >= N);
  };
  const bool tma_ok = x.inner == 1 && y.inner == 1 && aligned16(x.data) && (x.ld * 2) % 16 == 0 && x.ld >= K &&
                      weight_ok(wg) && (!swiglu || weight_ok(wu));
  const bool decode_ok = swiglu && tma_ok && decode_supported(M, N, K, y_f32);
  const int variant = choose_variant(request_variant(requested), tma_ok, decode_ok, M, K);
  const int math_mode = request_math_mode(requested);
  const bool fast_math = math_mode != LLK_MATH_STRICT;
  if (variant < 0) return LLK_ERR_UNSUPPORTED;

  llk_kernel_key key = make_key(op, y_f32 ? LLK_DTYPE_FP32 : LLK_DTYPE_BF16, M, N, K, variant);
  key.weight_layout = slab ? 1 : 0;  // Layout::PackedKN analogue
  key.math_mode = static_cast<uint8_t>(swiglu ? math_mode : LLK_MATH_STRICT);  // matmul has no epilogue math
  llk_launch_plan plan = plan_for(key, M, ds.sm_count);
  cudaError_t e = cudaSuccess;

  if (variant == LLK_VARIANT_SIMT) {
    int mode = swiglu ? 0 : (accumulate ? 2 : 1);
    e = simt_launch(mode, x.data, x.ld, x.inner, wg.data, swiglu ? wu.data : wg.data, wg.ld, wg.inner,
                    swiglu ? wu.ld : wg.ld, swiglu ? wu.inner : wg.inner, const_cast<void *>(y.data), y.ld, y.inner,
                    y_f32, M, N, K, slab ? 1 : 0, fast_math ? 1 : 0, stream);
    return e == cudaSuccess ? LLK_OK : LLK_ERR_CUDA;
  }

  if (variant == LLK_VARIANT_DECODE) {
    DecodePlan d = {plan.block_m, plan.block_n, plan.block_k, plan.stages,   plan.split_k,
                    plan.grid,    plan.threads, plan.smem_bytes, plan.sched ? plan.split_k : 0};
    if (!decode_plan_valid(M, N, K, d)) d = decode_plan(M, N, K, ds.sm_count);
    const size_t need = decode_workspace_bytes(M, N, K, d);
    void *ws = scratch;
    if (ws != nullptr) {
      // Caller scratch: its tile counters start from an unknown state.
      if (scratch_bytes < need) return LLK_ERR_NOMEM;
      const size_t off = decode_counter_offset(M, N);
      if (cudaMemsetAsync(static_cast<char *>(ws) + off, 0, decode_counter_bytes(N), stream) != cudaSuccess)
        return LLK_ERR_CUDA;
    } else {
      // ds.mu is held by the caller (run_op) for the whole launch.
      if (ds.workspace.ensure(need, true) != cudaSuccess) return LLK_ERR_NOMEM;
      ws = ds.workspace.ptr;
    }
    CUtensorMap tg, tu, tx;
    int rc;
    if ((rc = encode_weight_tmap(&tg, wg)) != LLK_OK) return rc;
    if ((rc = encode_weight_tmap(&tu, wu)) != LLK_OK) return rc;
    if ((rc = encode_tmap(&tx, x.data, K, M, x.ld * 2, 64, d.block_m)) != LLK_OK) return rc;
    e = decode_launch(tg, tu, tx, const_cast<void *>(y.data), y.ld, y_f32, M, N, K, ws, ds.status, d, slab ? 1 : 0,
                      fast_math ? 1 : 0, stream);
    return e == cudaSuccess ? LLK_OK : LLK_ERR_CUDA;
  }

  // tcgen05 path
  CUtensorMap ta, tb0, tb1;
  int rc;
  if ((rc = encode_tmap(&ta, x.data, K, M, x.ld * 2, 64, 128)) != LLK_OK) return rc;
  if ((rc = encode_weight_tmap(&tb0, wg)) != LLK_OK) return rc;
  if (swiglu) {
    if ((rc = encode_weight_tmap(&tb1, wu)) != LLK_OK) return rc;
  } else {
    tb1 = tb0;
  }
  const int mode = swiglu ? ((y_f32 ? TC_SWIGLU_F32 : TC_SWIGLU_BF16) | (fast_math ? TC_FAST_MATH : 0))
                          : (accumulate ? TC_MATMUL_F32_ACC : TC_MATMUL_F32);
  const int tile_n = tc_tile_n(mode);
  const int ysz = y_f32 ? 4 : 2;
  TcParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  // plan.block_m: 256 = CTA-pair kernel (swiglu_tc2.cu), 128 = one CTA per tile.
  const bool pair = plan.variant == LLK_VARIANT_TC ? plan.block_m == 256 : M > 128;
  const int rows = pair ? 256 : 128;
  p.m_tiles = static_cast<int>((M + rows - 1) / rows);
  p.n_tiles = static_cast<int>((N + tile_n - 1) / tile_n);
  p.num_tiles = p.m_tiles * p.n_tiles;
  p.k_blocks = static_cast<int>((K + 63) / 64);
  p.vec_ok = aligned16(y.data) && (y.ld * ysz) % 16 == 0;
  p.y = const_cast<void *>(y.data);
  p.ldy = y.ld;
  p.status = ds.status;
  p.b_lbo = 64 * 64 * 2;  // 8 KB between 64-column slabs
  p.b_sbo = 8 * 128;      // 1 KB between 8-row k groups
  p.slab_major = slab ? 1 : 0;
  if (pair) {
    const int max_pairs = plan.variant == LLK_VARIANT_TC && plan.grid >= 2 ? plan.grid / 2 : 0;
    // plan.split_k for the pair kernel: tail split of the leftover tiles (0 = choose,
    // 1/2/4 = that many column parts, -s = s K parts).
    const int tail_split = plan.variant == LLK_VARIANT_TC ? plan.split_k : 0;
    // The workspace: the library's (counter regions kept at zero by every
    // launch) or the caller's scratch, whose counter regions are cleared
    // here.  It holds the dynamic schedule's work counter (plan.sched = 0;
    // 1 selects the static schedule) and the K-split tail's counters and
    // partial sums.
    const bool dynamic = plan.variant == LLK_VARIANT_TC && plan.sched == 0;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    if (scratch != nullptr) {
      if (scratch_bytes >= kWsTc2CounterBytes) {
        if (cudaMemsetAsync(scratch, 0, kWsTc2CounterBytes, stream) != cudaSuccess) return LLK_ERR_CUDA;
        ws = scratch;
        ws_bytes = scratch_bytes;
      } else if (scratch_bytes >= kTc2SchedBytes) {
        // room for the work counter only (no K-split tail)
        if (cudaMemsetAsync(scratch, 0, sizeof(int), stream) != cudaSuccess) return LLK_ERR_CUDA;
        ws = scratch;
        ws_bytes = 0;
      } else if (dynamic) {
        return LLK_ERR_NOMEM;
      }
    } else {
      if (ds.workspace.ensure(tc2_tail_workspace_bytes(ds.sm_count), true) != cudaSuccess) return LLK_ERR_NOMEM;
      ws = ds.workspace.ptr;
      ws_bytes = ds.workspace.bytes;
    }
    int *counter = dynamic ? reinterpret_cast<int *>(static_cast<char *>(ws) + kWsTc2Counters) : nullptr;
    if (peers) {
      p.n_peers = peers->n;
      for (int i = 0; i < peers->n; ++i) p.y_peers[i] = peers->y[i];
      if (peers_done) *peers_done = true;
    }
    e = tc2_launch(mode, ta, tb0, tb1, p, max_pairs, tail_split, counter, ws_bytes ? ws : nullptr, ws_bytes, stream,
                   peers ? peers->maps : nullptr);
    return e == cudaSuccess ? LLK_OK : LLK_ERR_CUDA;
  }
  int grid = p.num_tiles < ds.sm_count ? p.num_tiles : ds.sm_count;
  if (plan.variant == LLK_VARIANT_TC && plan.grid >= 1 && plan.grid <= grid) grid = plan.grid;
  e = tc_launch(mode, ta, tb0, tb1, p, grid, stream);
  return e == cudaSuccess ? LLK_OK : LLK_ERR_CUDA;
}

// ------------------------------------------------------- argument checks
// The verifier rules of llk.fused_swiglu (lib/Dialect/LLK/LLKOps.cpp:42-83):
// X [M,K], Wg/Wu [K,N], Y [M,N], all consistent.
int check_swiglu(const Tensor2D *x, const Tensor2D *wg, const Tensor2D *wu, const Tensor2D *y) {
  if (!x || !wg || !wu || !y) return LLK_ERR_ARG;
  if (x->dim0 < 0 || x->dim1 < 0 || wg->dim0 < 0 || wg->dim1 < 0) return LLK_ERR_SHAPE;
  if (x->dim1 != wg->dim0 || x->dim1 != wu->dim0) return LLK_ERR_SHAPE;
  if (wg->dim1 != wu->dim1) return LLK_ERR_SHAPE;
  if (y->dim0 != x->dim0 || y->dim1 != wg->dim1) return LLK_ERR_SHAPE;
  const int64_t M = x->dim0, N = wg->dim1, K = x->dim1;
  if ((M > 0 && K > 0 && !x->data) || (K > 0 && N > 0 && (!wg->data || !wu->data)) || (M > 0 && N > 0 && !y->data))
    return LLK_ERR_ARG;
  return LLK_OK;
}

// One operand, device-resident view (staging host data when needed).
struct Staged {
  DevTensor t;
  bool host = false;
  const Tensor2D *src = nullptr;
};

// on_dev: whether src->data is device memory (queried once by the caller).
int stage_in(const Tensor2D *src, bool on_dev, int elem, DeviceBuffer &buf, bool copy, cudaStream_t stream,
             Staged *out) {
  out->src = src;
  out->t = {src->data, src->dim0, src->dim1, src->stride0, src->stride1};
  if (src->dim0 == 0 || src->dim1 == 0 || on_dev) return LLK_OK;
  if (src->stride1 != 1 || src->stride0 < src->dim1) return LLK_ERR_ALIGN;
  out->host = true;
  const size_t pitch = static_cast<size_t>(src->dim1) * elem;
  if (buf.ensure(pitch * static_cast<size_t>(src->dim0)) != cudaSuccess) return LLK_ERR_NOMEM;
  out->t = {buf.ptr, src->dim0, src->dim1, src->dim1, 1};
  if (copy) {
    cudaError_t e = cudaMemcpy2DAsync(buf.ptr, pitch, src->data, static_cast<size_t>(src->stride0) * elem, pitch,
                                      static_cast<size_t>(src->dim0), cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return LLK_ERR_CUDA;
  }
  return LLK_OK;
}

int stage_out(const Staged &s, int elem, cudaStream_t stream) {
  if (!s.host) return LLK_OK;
  const size_t pitch = static_cast<size_t>(s.src->dim1) * elem;
  cudaError_t e = cudaMemcpy2DAsync(s.src->data, static_cast<size_t>(s.src->stride0) * elem, s.t.data, pitch, pitch,
                                    static_cast<size_t>(s.src->dim0), cudaMemcpyDeviceToHost, stream);
  return e == cudaSuccess ? LLK_OK : LLK_ERR_CUDA;
}

int read_and_clear_status(DeviceState &ds, cudaStream_t stream) {
  int v = 0;
  if (cudaMemcpyAsync(&v, ds.status, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess) return LLK_ERR_CUDA;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return LLK_ERR_CUDA;
  if (v != 0) {
    cudaMemsetAsync(ds.status, 0, sizeof(int), stream);
    // A kernel that gave up may have left decode tile counters non-zero.
    if (ds.workspace.ptr) cudaMemsetAsync(ds.workspace.ptr, 0, ds.workspace.bytes, stream);
    cudaStreamSynchronize(stream);
    return LLK_ERR_TIMEOUT;
  }
  return LLK_OK;
}

// The copy streams and events of the pipelined host-buffer paths (once).
int copy_streams(DeviceState &ds) {
  if (ds.copy_in) return LLK_OK;
  if (cudaStreamCreateWithFlags(&ds.copy_in, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ds.copy_out, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&ds.ev_x, cudaEventDisableTiming) != cudaSuccess)
    return LLK_ERR_CUDA;
  for (int b = 0; b < 2; ++b)
    if (cudaEventCreateWithFlags(&ds.ev_in[b], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ds.ev_k[b], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ds.ev_out[b], cudaEventDisableTiming) != cudaSuccess)
      return LLK_ERR_CUDA;
  return LLK_OK;
}

// SwiGLU with X and Y in host memory and the weights on the device (packed
// weights, or device buffers), pipelined over row blocks of X: block b+1
// travels host->device while block b computes and block b-1's Y travels
// back.  LLK_ERR_UNSUPPORTED (before doing anything) when it does not suit.
// Called with ds.mu held.
int swiglu_rows_pipelined(DeviceState &ds, const Tensor2D *x, const DevTensor &wg, const DevTensor &wu, Tensor2D *y,
                          int y_f32, int requested, KernelContext *ctx, cudaStream_t stream) {
  const int64_t M = x->dim0, K = x->dim1, N = wg.cols;
  constexpr int kBlocks = 4;
  if (M == 0 || N == 0 || K == 0 || K % 8 != 0 || x->stride1 != 1 || y->stride1 != 1 || x->stride0 < K ||
      y->stride0 < N)
    return LLK_ERR_UNSUPPORTED;
  int64_t rb = (M + kBlocks - 1) / kBlocks;
  rb = (rb + 255) / 256 * 256;  // whole 256-row CTA-pair tiles per block
  if (rb >= M) return LLK_ERR_UNSUPPORTED;
  const int yel = y_f32 ? 4 : 2;
  if (copy_streams(ds) != LLK_OK) return LLK_ERR_CUDA;
  for (int b = 0; b < 2; ++b)
    if (ds.chunk_x[b].ensure(static_cast<size_t>(rb) * K * 2) != cudaSuccess ||
        ds.chunk_y[b].ensure(static_cast<size_t>(rb) * N * yel) != cudaSuccess)
      return LLK_ERR_NOMEM;
  if (cudaEventRecord(ds.ev_x, stream) != cudaSuccess || cudaStreamWaitEvent(ds.copy_in, ds.ev_x, 0) ||
      cudaStreamWaitEvent(ds.copy_out, ds.ev_x, 0))
    return LLK_ERR_CUDA;
  int blk = 0;
  for (int64_t r0 = 0; r0 < M; r0 += rb, ++blk) {
    const int b = blk & 1;
    const int64_t h = (M - r0) < rb ? (M - r0) : rb;
    if (blk >= 2 && (cudaStreamWaitEvent(ds.copy_in, ds.ev_k[b], 0) != cudaSuccess ||
                     cudaStreamWaitEvent(stream, ds.ev_out[b], 0) != cudaSuccess))
      return LLK_ERR_CUDA;
    if (cudaMemcpy2DAsync(ds.chunk_x[b].ptr, K * 2, static_cast<const char *>(x->data) + r0 * x->stride0 * 2,
                          x->stride0 * 2, K * 2, h, cudaMemcpyHostToDevice, ds.copy_in) != cudaSuccess ||
        cudaEventRecord(ds.ev_in[b], ds.copy_in) != cudaSuccess ||
        cudaStreamWaitEvent(stream, ds.ev_in[b], 0) != cudaSuccess)
      return LLK_ERR_CUDA;
    const DevTensor dx = {ds.chunk_x[b].ptr, h, K, K, 1};
    const DevTensor dy = {ds.chunk_y[b].ptr, h, N, N, 1};
    int rc = launch_device(ds, LLK_OP_FUSED_SWIGLU, dx, wg, wu, dy, y_f32, 0, requested, ctx ? ctx->scratch : nullptr,
                           ctx ? ctx->scratch_size : 0, stream);
    if (rc != LLK_OK) return rc;
    if (cudaEventRecord(ds.ev_k[b], stream) != cudaSuccess ||
        cudaStreamWaitEvent(ds.copy_out, ds.ev_k[b], 0) != cudaSuccess ||
        cudaMemcpy2DAsync(static_cast<char *>(y->data) + r0 * y->stride0 * yel, y->stride0 * yel, ds.chunk_y[b].ptr,
                          N * yel, N * yel, h, cudaMemcpyDeviceToHost, ds.copy_out) != cudaSuccess ||
        cudaEventRecord(ds.ev_out[b], ds.copy_out) != cudaSuccess)
      return LLK_ERR_CUDA;
  }
  if (cudaStreamWaitEvent(stream, ds.ev_out[(blk - 1) & 1], 0) != cudaSuccess) return LLK_ERR_CUDA;
  if (cudaStreamSynchronize(ds.copy_out) != cudaSuccess) return LLK_ERR_CUDA;
  return read_and_clear_status(ds, stream);
}

// SwiGLU with X, Wg, Wu and Y all in host memory, pipelined over column
// chunks of N: the weights of chunk c+1 travel host->device on one stream
// while chunk c computes, and Y of chunk c travels back on another -- so a
// call costs about the weight transfer instead of transfer + compute +
// transfer.  Falls back (returns LLK_ERR_UNSUPPORTED before doing anything)
// when the shape does not suit.  Called with ds.mu held.
int swiglu_host_pipelined(DeviceState &ds, const Tensor2D *x, const Tensor2D *wg, const Tensor2D *wu, Tensor2D *y,
                          int y_f32, int requested, KernelContext *ctx, cudaStream_t stream) {
  const int64_t M = x->dim0, K = x->dim1, N = wg->dim1;
  constexpr int kChunks = 8;
  if (M == 0 || N == 0 || K == 0 || K % 8 != 0) return LLK_ERR_UNSUPPORTED;
  if (x->stride1 != 1 || wg->stride1 != 1 || wu->stride1 != 1 || y->stride1 != 1) return LLK_ERR_UNSUPPORTED;
  if (x->stride0 < K || wg->stride0 < N || wu->stride0 < N || y->stride0 < N) return LLK_ERR_UNSUPPORTED;
  int64_t cw = (N + kChunks - 1) / kChunks;
  cw = (cw + 127) / 128 * 128;  // whole 128-column tiles per chunk
  if (cw >= N) return LLK_ERR_UNSUPPORTED;  // too narrow to pipeline
  const int yel = y_f32 ? 4 : 2;
  if (copy_streams(ds) != LLK_OK) return LLK_ERR_CUDA;
  const size_t xbytes = static_cast<size_t>(M) * K * 2;
  if (ds.stage[0].ensure(xbytes) != cudaSuccess) return LLK_ERR_NOMEM;
  for (int b = 0; b < 2; ++b) {
    if (ds.chunk_w[b][0].ensure(static_cast<size_t>(K) * cw * 2) != cudaSuccess ||
        ds.chunk_w[b][1].ensure(static_cast<size_t>(K) * cw * 2) != cudaSuccess ||
        ds.chunk_y[b].ensure(static_cast<size_t>(M) * cw * yel) != cudaSuccess)
      return LLK_ERR_NOMEM;
  }
  // The caller's stream is the compute stream; the copy streams start after
  // whatever the caller queued before this call.
  if (cudaEventRecord(ds.ev_k[0], stream) != cudaSuccess || cudaStreamWaitEvent(ds.copy_in, ds.ev_k[0], 0) ||
      cudaStreamWaitEvent(ds.copy_out, ds.ev_k[0], 0))
    return LLK_ERR_CUDA;
  if (cudaMemcpy2DAsync(ds.stage[0].ptr, K * 2, x->data, x->stride0 * 2, K * 2, M, cudaMemcpyHostToDevice,
                        ds.copy_in) != cudaSuccess ||
      cudaEventRecord(ds.ev_x, ds.copy_in) != cudaSuccess || cudaStreamWaitEvent(stream, ds.ev_x, 0) != cudaSuccess)
    return LLK_ERR_CUDA;
  const DevTensor dx = {ds.stage[0].ptr, M, K, K, 1};
  int chunk = 0;
  for (int64_t c0 = 0; c0 < N; c0 += cw, ++chunk) {
    const int b = chunk & 1;
    const int64_t w = (N - c0) < cw ? (N - c0) : cw;
    // buffer b was last read by chunk-2's kernel and written to host by its D2H
    if (chunk >= 2 && (cudaStreamWaitEvent(ds.copy_in, ds.ev_k[b], 0) != cudaSuccess ||
                       cudaStreamWaitEvent(stream, ds.ev_out[b], 0) != cudaSuccess))
      return LLK_ERR_CUDA;
    const Tensor2D *ws[2] = {wg, wu};
    for (int m = 0; m < 2; ++m)
      if (cudaMemcpy2DAsync(ds.chunk_w[b][m].ptr, cw * 2, static_cast<const char *>(ws[m]->data) + c0 * 2,
                            ws[m]->stride0 * 2, w * 2, K, cudaMemcpyHostToDevice, ds.copy_in) != cudaSuccess)
        return LLK_ERR_CUDA;
    if (cudaEventRecord(ds.ev_in[b], ds.copy_in) != cudaSuccess ||
        cudaStreamWaitEvent(stream, ds.ev_in[b], 0) != cudaSuccess)
      return LLK_ERR_CUDA;
    const DevTensor dg = {ds.chunk_w[b][0].ptr, K, w, cw, 1}, du = {ds.chunk_w[b][1].ptr, K, w, cw, 1};
    const DevTensor dy = {ds.chunk_y[b].ptr, M, w, cw, 1};
    int rc = launch_device(ds, LLK_OP_FUSED_SWIGLU, dx, dg, du, dy, y_f32, 0, requested,
                           ctx ? ctx->scratch : nullptr, ctx ? ctx->scratch_size : 0, stream);
    if (rc != LLK_OK) return rc;
    if (cudaEventRecord(ds.ev_k[b], stream) != cudaSuccess ||
        cudaStreamWaitEvent(ds.copy_out, ds.ev_k[b], 0) != cudaSuccess ||
        cudaMemcpy2DAsync(static_cast<char *>(y->data) + c0 * yel, y->stride0 * yel, ds.chunk_y[b].ptr, cw * yel,
                          w * yel, M, cudaMemcpyDeviceToHost, ds.copy_out) != cudaSuccess ||
        cudaEventRecord(ds.ev_out[b], ds.copy_out) != cudaSuccess)
      return LLK_ERR_CUDA;
  }
  // the call returns with Y on the host; the caller's stream waits for it too
  if (cudaStreamWaitEvent(stream, ds.ev_out[(chunk - 1) & 1], 0) != cudaSuccess) return LLK_ERR_CUDA;
  if (cudaStreamSynchronize(ds.copy_out) != cudaSuccess) return LLK_ERR_CUDA;
  return read_and_clear_status(ds, stream);
}

// Common body of the SwiGLU / matmul entry points.  wu may equal wg (matmul).
int run_op(int op, const Tensor2D *x, const Tensor2D *wg, const Tensor2D *wu, Tensor2D *y, int y_f32, int accumulate,
           KernelContext *ctx, const llk_gpu_context *gpu, const DevTensor *packed_g = nullptr,
           const DevTensor *packed_u = nullptr) {
  DeviceRestore restore;
  if (gpu && (gpu->y_dtype != LLK_DTYPE_BF16 && gpu->y_dtype != LLK_DTYPE_FP32)) return LLK_ERR_ARG;
  if (gpu && (gpu->variant < LLK_VARIANT_AUTO || gpu->variant > LLK_VARIANT_SIMT)) return LLK_ERR_ARG;
  if (gpu && (gpu->math_mode < LLK_MATH_STRICT || gpu->math_mode > LLK_MATH_UNSAFE_FAST)) return LLK_ERR_ARG;
  int dev, rc;
  if ((rc = resolve_device(gpu, &dev)) != LLK_OK) return rc;
  DeviceState *ds;
  if ((rc = device_init(dev, &ds)) != LLK_OK) return rc;
  cudaStream_t stream = gpu ? static_cast<cudaStream_t>(gpu->stream) : nullptr;
  const int requested = pack_request(gpu);
  const int yel = y_f32 ? 4 : 2;

  Staged sx, sg, su, sy;
  bool any_host;
  {
    // Where each buffer lives, asked once per call.
    const int lx = locate_ptr(x->data, dev), ly = locate_ptr(y->data, dev);
    const int lg = packed_g ? 1 : locate_ptr(wg->data, dev);
    const int lu = packed_g ? 1 : (wu == wg ? lg : locate_ptr(wu->data, dev));
    const bool dx = lx != 0, dy = ly != 0, dg = lg != 0, du = lu != 0;
    if (lx < 0 || ly < 0 || lg < 0 || lu < 0)
      return LLK_ERR_ARG;
    std::lock_guard<std::mutex> lk(ds->mu);
    if (op == LLK_OP_FUSED_SWIGLU && !packed_g && x->data && wg->data && wu->data && y->data && !dx && !dg && !du &&
        !dy) {
      rc = swiglu_host_pipelined(*ds, x, wg, wu, y, y_f32, requested, ctx, stream);
      if (rc != LLK_ERR_UNSUPPORTED) return rc;
    }
    if (op == LLK_OP_FUSED_SWIGLU && packed_g && x->data && y->data && !dx && !dy) {
      rc = swiglu_rows_pipelined(*ds, x, *packed_g, *packed_u, y, y_f32, requested, ctx, stream);
      if (rc != LLK_ERR_UNSUPPORTED) return rc;
    }
    if ((rc = stage_in(x, dx, 2, ds->stage[0], true, stream, &sx)) != LLK_OK) return rc;
    if (packed_g) {
      sg.t = *packed_g;
      su.t = *packed_u;
    } else if ((rc = stage_in(wg, dg, 2, ds->stage[1], true, stream, &sg)) != LLK_OK) {
      return rc;
    } else if (wu != wg) {
      if ((rc = stage_in(wu, du, 2, ds->stage[2], true, stream, &su)) != LLK_OK) return rc;
    } else {
      su = sg;
    }
    if ((rc = stage_in(y, dy, yel, ds->stage[3], accumulate != 0, stream, &sy)) != LLK_OK) return rc;
    any_host = sx.host || sg.host || su.host || sy.host;
    rc = launch_device(*ds, op, sx.t, sg.t, su.t, sy.t, y_f32, accumulate, requested, ctx ? ctx->scratch : nullptr,
                       ctx ? ctx->scratch_size : 0, stream);
    if (rc != LLK_OK) return rc;
    if ((rc = stage_out(sy, yel, stream)) != LLK_OK) return rc;
    if (any_host) return read_and_clear_status(*ds, stream);
  }
  return LLK_OK;
}

// ------------------------------------------------- column-parallel groups
// One per GPU of a column-parallel SwiGLU: a device allocation holding a
// flag block and two Y buffers [M, N], exported by CUDA IPC; every rank maps
// every other rank's allocation.  Call t computes this rank's columns, the
// CTA-pair epilogue storing each chunk into every rank's Y buffer t % 2
// (fused all-gather), then runs a barrier so that, in stream order, this
// GPU's buffer holds all columns.  Alternating buffers make an entry barrier
// unnecessary: a rank starts call t + 1 only after call t's barrier saw
// every peer's stream reach call t, i.e. past every peer's stream-ordered
// use of buffer (t + 1) % 2 = (t - 1) % 2.
constexpr int kGroupMax = 8;
constexpr size_t kFlagBytes = 4096;  // flag block at the start of each allocation
constexpr uint64_t kBarrierLimitNs = 2000000000ull;

struct BarrierArgs {
  unsigned int *peer_slot[kGroupMax];  // rank r's flag word for this rank (in r's allocation)
  unsigned int *own[kGroupMax];        // this rank's flag word for rank r (own allocation)
};

// Thread r < n: publish `epoch` in rank r's slot for this rank (system-scope
// release), then wait until rank r published it here.  Bounded: after the
// limit the status word gets LLK_ERR_TIMEOUT and the kernel returns.
// Launched as a programmatic dependent of the SwiGLU kernel before it: the
// launch overlaps that kernel's tail, and griddepcontrol.wait returns once
// it has completed and its memory operations (the peer stores) are
// performed, so nothing is published early.
__global__ void peer_barrier_kernel(BarrierArgs a, int n, unsigned int epoch, int *status) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int r = threadIdx.x;
  if (r >= n) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.peer_slot[r]), "r"(epoch) : "memory");
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a.own[r]) : "memory");
    if (static_cast<int>(v - epoch) >= 0) break;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > kBarrierLimitNs) {
      atomicExch(status, LLK_ERR_TIMEOUT);
      break;
    }
    __nanosleep(200);
  }
}

}  // namespace

struct llk_peer_group {
  int device = -1, n = 0, rank = 0;
  char *local = nullptr;          // [flags 4 KB][Y buffer 0][Y buffer 1]
  size_t y_bytes = 0;             // capacity of one Y buffer (multiple of 256)
  char *base[kGroupMax] = {};     // every rank's allocation as mapped here
  bool connected = false;
  unsigned int epoch = 0;
  cudaIpcMemHandle_t handle;
};

namespace {

// Flag words of barrier `which` at [8 * which, 8 * which + 8), one per rank.
BarrierArgs barrier_args(const llk_peer_group &g, int which) {
  BarrierArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int r = 0; r < g.n; ++r) {
    a.peer_slot[r] = reinterpret_cast<unsigned int *>(g.base[r]) + which * kGroupMax + g.rank;
    a.own[r] = reinterpret_cast<unsigned int *>(g.local) + which * kGroupMax + r;
  }
  return a;
}

DevTensor dev_tensor(const Tensor2D &t) {
  DevTensor d;
  d.data = t.data;
  d.rows = t.dim0;
  d.cols = t.dim1;
  d.ld = t.stride0;
  d.inner = t.stride1;
  return d;
}

}  // namespace

// ====================================================================== C ABI
extern "C" {

int llk_classify_m(int64_t M) {
  if (M == 1) return 0;
  if (M <= 4) return 1;
  if (M <= 16) return 2;
  if (M <= 64) return 3;
  return 4;
}

uint64_t llk_version(void) { return kLibraryVersion; }

int llk_last_status(void) { return g_last_status; }

const char *llk_status_string(int s) {
  switch (s) {
    case LLK_OK: return "ok";
    case LLK_ERR_SHAPE: return "shape mismatch";
    case LLK_ERR_ALIGN: return "unsupported stride or alignment";
    case LLK_ERR_CUDA: return "CUDA error";
    case LLK_ERR_NCCL: return "NCCL error";
    case LLK_ERR_TIMEOUT: return "device wait timed out";
    case LLK_ERR_ARG: return "invalid argument";
    case LLK_ERR_DEVICE: return "no usable sm_100 device";
    case LLK_ERR_UNSUPPORTED: return "unsupported request";
    case LLK_ERR_NOMEM: return "out of memory / scratch too small";
    case LLK_ERR_NOT_FOUND: return "no cache entry";
    default: return "unknown status";
  }
}

int llk_swiglu_ex(const Tensor2D *x, const Tensor2D *wg, const Tensor2D *wu, Tensor2D *y, KernelContext *ctx,
                  const llk_gpu_context *gpu) {
  int rc = check_swiglu(x, wg, wu, y);
  if (rc != LLK_OK) return rc;
  const int y_f32 = (gpu && gpu->y_dtype == LLK_DTYPE_FP32) ? 1 : 0;
  return run_op(LLK_OP_FUSED_SWIGLU, x, wg, wu, y, y_f32, 0, ctx, gpu);
}

void llk_swiglu(const Tensor2D *x, const Tensor2D *wg, const Tensor2D *wu, Tensor2D *y, KernelContext *ctx) {
  g_last_status = llk_swiglu_ex(x, wg, wu, y, ctx, nullptr);
}

void llk_swiglu_memref(MemRef2D *x, MemRef2D *wg, MemRef2D *wu, MemRef2D *init, MemRef2D *result) {
  (void)init;
  if (!x || !wg || !wu || !result) {
    g_last_status = LLK_ERR_ARG;
    return;
  }
  auto view = [](const MemRef2D *m) {
    Tensor2D t;
    t.data = static_cast<char *>(m->aligned) + m->offset * 2;
    t.dim0 = m->size0;
    t.dim1 = m->size1;
    t.stride0 = m->stride0;
    t.stride1 = m->stride1;
    return t;
  };
  Tensor2D tx = view(x), tg = view(wg), tu = view(wu), ty = view(result);
  g_last_status = llk_swiglu_ex(&tx, &tg, &tu, &ty, nullptr, nullptr);
}

int llk_matmul(const Tensor2D *a, const Tensor2D *b, Tensor2D *c, int accumulate, KernelContext *ctx,
               const llk_gpu_context *gpu) {
  if (!a || !b || !c) return LLK_ERR_ARG;
  // micro.mma verifier rules (MicroOps.cpp:246-291): lhs [M,K], rhs [K,N], acc [M,N].
  if (a->dim0 < 0 || a->dim1 < 0 || b->dim1 < 0) return LLK_ERR_SHAPE;
  if (a->dim1 != b->dim0 || c->dim0 != a->dim0 || c->dim1 != b->dim1) return LLK_ERR_SHAPE;
  if (gpu && gpu->variant == LLK_VARIANT_DECODE) return LLK_ERR_UNSUPPORTED;
  return run_op(LLK_OP_MATMUL, a, b, b, c, 1, accumulate ? 1 : 0, ctx, gpu);
}

// ------------------------------------------------- llk.rope / llk.attention
// Flat f32 / i64 arrays in host or device memory: host arrays are staged
// through the device (the call then returns with the result on the host),
// device arrays must live on the call's device.
namespace {
struct FlatArg {
  const void *p;
  int64_t n;     // elements
  int elem;      // bytes per element
  bool out;      // written by the kernel
  bool in;       // read by the kernel
};

int run_flat(const llk_gpu_context *gpu, FlatArg *args, int nargs,
             const std::function<cudaError_t(void **, cudaStream_t, bool, DeviceState &)> &launch) {
  DeviceRestore restore;
  if (gpu && (gpu->math_mode < LLK_MATH_STRICT || gpu->math_mode > LLK_MATH_UNSAFE_FAST)) return LLK_ERR_ARG;
  int dev, rc;
  if ((rc = resolve_device(gpu, &dev)) != LLK_OK) return rc;
  DeviceState *ds;
  if ((rc = device_init(dev, &ds)) != LLK_OK) return rc;
  cudaStream_t stream = gpu ? static_cast<cudaStream_t>(gpu->stream) : nullptr;
  const bool fast = gpu && gpu->math_mode != LLK_MATH_STRICT;
  std::lock_guard<std::mutex> lk(ds->mu);
  Tensor2D views[4];
  Staged st[4];
  void *ptrs[4] = {};
  bool any_host = false;
  for (int i = 0; i < nargs; ++i) {
    if (args[i].n > 0 && args[i].p == nullptr) return LLK_ERR_ARG;
    const bool on_dev = args[i].n == 0 || is_device_ptr(args[i].p);
    if (on_dev && args[i].n > 0 && on_other_device(args[i].p, dev)) return LLK_ERR_ARG;
    views[i] = {const_cast<void *>(args[i].p), 1, args[i].n, args[i].n, 1};
    if ((rc = stage_in(&views[i], on_dev, args[i].elem, ds->stage[i], args[i].in, stream, &st[i])) != LLK_OK)
      return rc;
    ptrs[i] = const_cast<void *>(st[i].t.data);
    any_host = any_host || st[i].host;
  }
  const cudaError_t le = launch(ptrs, stream, fast, *ds);
  if (le == cudaErrorMemoryAllocation) return LLK_ERR_NOMEM;
  if (le != cudaSuccess) return LLK_ERR_CUDA;
  for (int i = 0; i < nargs; ++i)
    if (args[i].out && (rc = stage_out(st[i], args[i].elem, stream)) != LLK_OK) return rc;
  if (any_host) return read_and_clear_status(*ds, stream);
  return LLK_OK;
}
}  // namespace

int llk_rope(const float *x, const int64_t *position_ids, float *y, int64_t B, int64_t H, int64_t L, int64_t D,
             double theta, const llk_gpu_context *gpu) {
  if (B < 0 || H < 0 || L < 0 || D < 0) return LLK_ERR_SHAPE;
  if (D % 2 != 0) return LLK_ERR_SHAPE;  // pairs of dimensions
  if (!rope_supported(B, H, L, D > 0 ? D : 2)) return LLK_ERR_UNSUPPORTED;
  const int64_t n = B * H * L * D;
  if (n == 0) return LLK_OK;
  if (!(theta > 0.0)) return LLK_ERR_ARG;
  // The (cos, sin) table goes to the partial-sum region of the device
  // workspace (written before it is read; calls on one device are serialised).
  auto table = [&](DeviceState &ds, void **out) {
    if (ds.workspace.ensure(kWsPartials + rope_table_bytes(L, D), true) != cudaSuccess)
      return cudaErrorMemoryAllocation;
    *out = static_cast<char *>(ds.workspace.ptr) + kWsPartials;
    return cudaSuccess;
  };
  if (x == y) {
    // in place: one buffer, read and written
    FlatArg b[2] = {{x, n, 4, true, true}, {position_ids, L, 8, false, true}};
    return run_flat(gpu, b, 2, [&](void **p, cudaStream_t s, bool fast, DeviceState &ds) {
      void *tab = nullptr;
      const cudaError_t e = table(ds, &tab);
      if (e != cudaSuccess) return e;
      return rope_launch(static_cast<float *>(p[0]), static_cast<const int64_t *>(p[1]), static_cast<float *>(p[0]),
                         B, H, L, D, theta, fast ? 1 : 0, tab, ds.sm_count, s);
    });
  }
  FlatArg a[3] = {{x, n, 4, false, true}, {position_ids, L, 8, false, true}, {y, n, 4, true, false}};
  return run_flat(gpu, a, 3, [&](void **p, cudaStream_t s, bool fast, DeviceState &ds) {
    void *tab = nullptr;
    const cudaError_t e = table(ds, &tab);
    if (e != cudaSuccess) return e;
    return rope_launch(static_cast<const float *>(p[0]), static_cast<const int64_t *>(p[1]), static_cast<float *>(p[2]),
                       B, H, L, D, theta, fast ? 1 : 0, tab, ds.sm_count, s);
  });
}

int llk_attention(const float *q, const float *k, const float *v, float *o, int64_t B, int64_t H, int64_t Lq,
                  int64_t Lk, int64_t D, float scale, int causal, const llk_gpu_context *gpu) {
  if (B < 0 || H < 0 || Lq < 0 || Lk < 0 || D < 0) return LLK_ERR_SHAPE;
  if (B * H * Lq * D == 0) return LLK_OK;
  if (!attention_supported(B, H, Lq, Lk, D)) return LLK_ERR_UNSUPPORTED;
  if (o == q || o == k || o == v) return LLK_ERR_ARG;  // O accumulates while Q, K, V are read
  const int64_t nq = B * H * Lq * D, nk = B * H * Lk * D;
  FlatArg a[4] = {{q, nq, 4, false, true}, {k, nk, 4, false, true}, {v, nk, 4, false, true}, {o, nq, 4, true, true}};
  return run_flat(gpu, a, 4, [&](void **p, cudaStream_t s, bool fast, DeviceState &) {
    return attention_launch(static_cast<const float *>(p[0]), static_cast<const float *>(p[1]),
                            static_cast<const float *>(p[2]), static_cast<float *>(p[3]), B, H, Lq, Lk, D, scale,
                            causal ? 1 : 0, fast ? 1 : 0, s);
  });
}

int llk_synchronize(int device, void *stream) {
  DeviceRestore restore;
  llk_gpu_context g;
  std::memset(&g, 0, sizeof(g));
  g.device = device;
  int dev, rc;
  if ((rc = resolve_device(&g, &dev)) != LLK_OK) return rc;
  DeviceState *ds;
  if ((rc = device_init(dev, &ds)) != LLK_OK) return rc;
  return read_and_clear_status(*ds, static_cast<cudaStream_t>(stream));
}

int llk_diag_reciprocal_check(int device, uint32_t lo_bits, uint32_t hi_bits, uint64_t *mismatches) {
  if (!mismatches || hi_bits < lo_bits) return LLK_ERR_ARG;
  DeviceRestore restore;
  llk_gpu_context g;
  std::memset(&g, 0, sizeof(g));
  g.device = device;
  int dev, rc;
  if ((rc = resolve_device(&g, &dev)) != LLK_OK) return rc;
  DeviceState *ds;
  if ((rc = device_init(dev, &ds)) != LLK_OK) return rc;
  unsigned long long *d = nullptr;
  if (cudaMalloc(&d, sizeof(*d)) != cudaSuccess) return LLK_ERR_NOMEM;
  unsigned long long h = 0;
  rc = LLK_OK;
  if (cudaMemset(d, 0, sizeof(*d)) != cudaSuccess ||
      diag_reciprocal_launch(d, lo_bits, hi_bits, ds->sm_count, nullptr) != cudaSuccess ||
      cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = LLK_ERR_CUDA;
  cudaFree(d);
  *mismatches = h;
  return rc;
}

int llk_diag_pair_schedule(int swiglu, int64_t M, int64_t N, int64_t K, int pairs, int tail_split, int dynamic,
                           int32_t *items, int max_items, int *n_items, int *n_pairs, int *ksplit, int *tail_split_out) {
  if (!n_items || !n_pairs || !ksplit || !tail_split_out || (max_items > 0 && !items) || max_items < 0)
    return LLK_ERR_ARG;
  // the library workspace of a 148-SM device (room for the K-split tail)
  return tc2_schedule_items(swiglu, M, N, K, pairs, tail_split, dynamic, tc2_tail_workspace_bytes(2 * pairs), items,
                            max_items, n_items, n_pairs, ksplit, tail_split_out) == 0
             ? LLK_OK
             : LLK_ERR_ARG;
}

int llk_diag_timeout_probe(int device, int64_t limit_ns) {
  if (limit_ns <= 0) return LLK_ERR_ARG;
  DeviceRestore restore;
  llk_gpu_context g;
  std::memset(&g, 0, sizeof(g));
  g.device = device;
  int dev, rc;
  if ((rc = resolve_device(&g, &dev)) != LLK_OK) return rc;
  DeviceState *ds;
  if ((rc = device_init(dev, &ds)) != LLK_OK) return rc;
  if (diag_timeout_launch(ds->status, static_cast<uint64_t>(limit_ns), nullptr) != cudaSuccess) return LLK_ERR_CUDA;
  return read_and_clear_status(*ds, nullptr);
}

// ---------------------------------------------------------- packed weights
// Layout: each matrix is stored slab-major, [ceil(N/64)][K][64] bf16 -- the
// 64-column slabs the kernels load as one TMA box each, so every box is a
// contiguous 8 KB block instead of 64 rows of 128 bytes strided by the row
// pitch.  This is runtime/PackedWeights.cpp's k-block packing turned
// around: there K is blocked and rows stay N wide (the CPU kernel walks n in
// the inner loop); here N is blocked at the TMA box width and K runs inside
// a block (the tensor cores consume [64 k x 64 n] tiles).  Columns past N in
// the last slab are zero.
struct llk_packed_weights {
  int device;
  int64_t K, N, n_slabs;
  void *wg;  // device, slab-major
  void *wu;
  int64_t bytes;
  std::atomic<int> refs{1};  // holders: the packing caller, lookups, the L4 cache
};

static int copy_weight_slabs(void *dst, int64_t K, int64_t N, const Tensor2D *w, cudaStream_t stream) {
  if (w->stride1 != 1 || w->stride0 < w->dim1) return LLK_ERR_ALIGN;
  const bool dev = is_device_ptr(w->data);
  const int64_t n_slabs = (N + 63) / 64;
  for (int64_t s = 0; s < n_slabs; ++s) {
    const int64_t cols = (N - 64 * s) < 64 ? (N - 64 * s) : 64;
    cudaError_t e = cudaMemcpy2DAsync(static_cast<char *>(dst) + s * K * 128, 128,
                                      static_cast<const char *>(w->data) + s * 64 * 2,
                                      static_cast<size_t>(w->stride0) * 2, static_cast<size_t>(cols) * 2,
                                      static_cast<size_t>(K), dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                                      stream);
    if (e != cudaSuccess) return LLK_ERR_CUDA;
  }
  return LLK_OK;
}

int llk_repack(llk_packed_weights *pw, const Tensor2D *wg, const Tensor2D *wu, const llk_gpu_context *gpu) {
  if (!pw || !wg || !wu) return LLK_ERR_ARG;
  if (wg->dim0 != pw->K || wg->dim1 != pw->N || wu->dim0 != pw->K || wu->dim1 != pw->N) return LLK_ERR_SHAPE;
  if (cudaSetDevice(pw->device) != cudaSuccess) return LLK_ERR_DEVICE;
  cudaStream_t stream = gpu ? static_cast<cudaStream_t>(gpu->stream) : nullptr;
  if (pw->K == 0 || pw->N == 0) return LLK_OK;
  int rc;
  if ((rc = copy_weight_slabs(pw->wg, pw->K, pw->N, wg, stream)) != LLK_OK) return rc;
  if ((rc = copy_weight_slabs(pw->wu, pw->K, pw->N, wu, stream)) != LLK_OK) return rc;
  return cudaStreamSynchronize(stream) == cudaSuccess ? LLK_OK : LLK_ERR_CUDA;
}

int llk_pack_weights(const Tensor2D *wg, const Tensor2D *wu, const llk_gpu_context *gpu, llk_packed_weights **out) {
  if (!wg || !wu || !out) return LLK_ERR_ARG;
  *out = nullptr;
  if (wg->dim0 != wu->dim0 || wg->dim1 != wu->dim1 || wg->dim0 < 0 || wg->dim1 < 0) return LLK_ERR_SHAPE;
  int dev, rc;
  if ((rc = resolve_device(gpu, &dev)) != LLK_OK) return rc;
  DeviceState *ds;
  if ((rc = device_init(dev, &ds)) != LLK_OK) return rc;
  llk_packed_weights *pw = new llk_packed_weights();
  pw->device = dev;
  pw->K = wg->dim0;
  pw->N = wg->dim1;
  pw->n_slabs = (pw->N + 63) / 64;
  const size_t bytes = static_cast<size_t>(pw->K) * pw->n_slabs * 128;
  pw->bytes = static_cast<int64_t>(2 * bytes);
  pw->wg = pw->wu = nullptr;
  if (bytes > 0) {
    if (cudaMalloc(&pw->wg, bytes) != cudaSuccess || cudaMalloc(&pw->wu, bytes) != cudaSuccess) {
      cudaFree(pw->wg);
      delete pw;
      return LLK_ERR_NOMEM;
    }
    cudaStream_t stream = gpu ? static_cast<cudaStream_t>(gpu->stream) : nullptr;
    cudaMemsetAsync(pw->wg, 0, bytes, stream);
    cudaMemsetAsync(pw->wu, 0, bytes, stream);
  }
  if ((rc = llk_repack(pw, wg, wu, gpu)) != LLK_OK) {
    llk_packed_weights_free(pw);
    return rc;
  }
  *out = pw;
  return LLK_OK;
}

void llk_packed_weights_free(llk_packed_weights *pw) {
  if (!pw) return;
  if (pw->refs.fetch_sub(1, std::memory_order_acq_rel) > 1) return;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(pw->device);
  cudaFree(pw->wg);
  cudaFree(pw->wu);
  cudaSetDevice(cur);
  delete pw;
}

int llk_packed_weights_info(const llk_packed_weights *pw, int64_t *K, int64_t *N, int64_t *bytes) {
  if (!pw) return LLK_ERR_ARG;
  if (K) *K = pw->K;
  if (N) *N = pw->N;
  if (bytes) *bytes = pw->bytes;
  return LLK_OK;
}

int llk_packed_weights_layout(const llk_packed_weights *pw, llk_packed_layout *out) {
  if (!pw || !out) return LLK_ERR_ARG;
  out->wg = pw->wg;
  out->wu = pw->wu;
  out->device = pw->device;
  out->box_n = 64;
  out->box_k = 64;
  out->slab_stride_bytes = pw->K * 64 * 2;
  return LLK_OK;
}

int llk_swiglu_packed(const Tensor2D *x, const llk_packed_weights *pw, Tensor2D *y, KernelContext *ctx,
                      const llk_gpu_context *gpu) {
  if (!x || !pw || !y) return LLK_ERR_ARG;
  if (x->dim1 != pw->K || y->dim0 != x->dim0 || y->dim1 != pw->N || x->dim0 < 0) return LLK_ERR_SHAPE;
  llk_gpu_context g;
  if (gpu) {
    g = *gpu;
  } else {
    std::memset(&g, 0, sizeof(g));
    g.device = pw->device;
  }
  if (g.device >= 0 && g.device != pw->device) return LLK_ERR_ARG;
  g.device = pw->device;
  if (g.y_dtype != LLK_DTYPE_BF16 && g.y_dtype != LLK_DTYPE_FP32) return LLK_ERR_ARG;
  DevTensor pg, pu;
  pg.data = pw->wg;
  pu.data = pw->wu;
  pg.rows = pu.rows = pw->K;
  pg.cols = pu.cols = pw->N;
  pg.ld = pu.ld = 64;
  pg.inner = pu.inner = 1;
  pg.slab_major = pu.slab_major = 1;
  Tensor2D wview = {pw->wg, pw->K, pw->N, pw->N, 1};  // shape carrier for the argument checks
  int rc = check_swiglu(x, &wview, &wview, y);
  if (rc != LLK_OK) return rc;
  return run_op(LLK_OP_FUSED_SWIGLU, x, &wview, &wview, y, g.y_dtype == LLK_DTYPE_FP32 ? 1 : 0, 0, ctx, &g, &pg, &pu);
}

// ---------------------------------------------------------------- sharding
int llk_shard_columns(int64_t N, int n_shards, int index, int64_t *begin, int64_t *end) {
  if (N < 0 || n_shards <= 0 || index < 0 || index >= n_shards || !begin || !end) return LLK_ERR_ARG;
  const int64_t tiles = (N + 127) / 128;
  const int64_t base = tiles / n_shards, rem = tiles % n_shards;
  const int64_t t0 = index * base + (index < rem ? index : rem);
  const int64_t t1 = t0 + base + (index < rem ? 1 : 0);
  *begin = t0 * 128 < N ? t0 * 128 : N;
  *end = t1 * 128 < N ? t1 * 128 : N;
  return LLK_OK;
}

// ------------------------------------------------------------------- probe
int llk_cuda_probe(int device, llk_cuda_target *out) {
  if (!out) return LLK_ERR_ARG;
  std::memset(out, 0, sizeof(*out));
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
    cudaGetLastError();
    return LLK_ERR_DEVICE;
  }
  if (device < 0 && cudaGetDevice(&device) != cudaSuccess) return LLK_ERR_DEVICE;
  if (device >= count) return LLK_ERR_ARG;
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return LLK_ERR_DEVICE;
  out->device = device;
  out->cc_major = p.major;
  out->cc_minor = p.minor;
  out->sm_count = p.multiProcessorCount;
  out->max_smem_per_block_optin = static_cast<int>(p.sharedMemPerBlockOptin);
  out->global_mem_bytes = static_cast<int64_t>(p.totalGlobalMem);
  out->l2_bytes = p.l2CacheSize;
  int clk = 0;
  cudaDeviceGetAttribute(&clk, cudaDevAttrClockRate, device);
  out->clock_khz = clk;
  std::strncpy(out->name, p.name, sizeof(out->name) - 1);
  out->is_sm100a = (p.major == 10 && p.minor == 0) ? 1 : 0;
  return LLK_OK;
}

// ------------------------------------------------------------- plan cache
uint64_t llk_kernel_key_hash(const llk_kernel_key *k) {
  // splitmix64 finaliser over each field (the mixing KernelKey::hash uses,
  // include/LLK/Runtime/KernelKey.h:60-84).
  auto mix = [](uint64_t x) {
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
    return x ^ (x >> 31);
  };
  uint64_t h = 0x9ae16a3b2f90404fULL;
  const uint64_t fields[] = {k->operation,    k->input_type,     k->output_type,          static_cast<uint64_t>(k->M_bucket),
                             static_cast<uint64_t>(k->N), static_cast<uint64_t>(k->K), k->weight_layout, k->isa,
                             k->math_mode,    k->thread_count,   k->compiler_version,     k->schedule_version};
  for (uint64_t f : fields) h = mix(h ^ f);
  return h;
}

int llk_plan_lookup(const llk_kernel_key *key, int64_t M, llk_launch_plan *out) {
  if (!key || !out || M < 0) return LLK_ERR_ARG;
  if (key->thread_count < LLK_VARIANT_TC || key->thread_count > LLK_VARIANT_SIMT) return LLK_ERR_ARG;
  int sm = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, dev) == cudaSuccess) sm = p.multiProcessorCount;
  } else {
    cudaGetLastError();
  }
  *out = plan_for(*key, M, sm);
  return LLK_OK;
}

int llk_plan_insert(const llk_kernel_key *key, const llk_launch_plan *plan) {
  if (!key || !plan) return LLK_ERR_ARG;
  if (plan->variant < LLK_VARIANT_TC || plan->variant > LLK_VARIANT_SIMT || plan->variant != key->thread_count)
    return LLK_ERR_ARG;
  const std::string kb = key_bytes(*key);
  std::lock_guard<std::mutex> lk(g_cache.mu);
  auto it = g_cache.index.find(kb);
  if (it != g_cache.index.end()) {
    it->second->plan = *plan;
    g_cache.lru.splice(g_cache.lru.begin(), g_cache.lru, it->second);
    return LLK_OK;
  }
  g_cache.lru.push_front({kb, *plan});
  g_cache.index[kb] = g_cache.lru.begin();
  while (g_cache.lru.size() > g_cache.max_entries) {
    g_cache.index.erase(g_cache.lru.back().key);
    g_cache.lru.pop_back();
    ++g_cache.evictions;
  }
  return LLK_OK;
}

void llk_cache_stats(uint64_t *hits, uint64_t *misses, uint64_t *evictions) {
  std::lock_guard<std::mutex> lk(g_cache.mu);
  if (hits) *hits = g_cache.hits;
  if (misses) *misses = g_cache.misses;
  if (evictions) *evictions = g_cache.evictions;
}

void llk_cache_set_max_entries(uint64_t max_entries) {
  std::lock_guard<std::mutex> lk(g_cache.mu);
  g_cache.max_entries = max_entries;
  while (g_cache.lru.size() > g_cache.max_entries) {
    g_cache.index.erase(g_cache.lru.back().key);
    g_cache.lru.pop_back();
    ++g_cache.evictions;
  }
}

void llk_cache_clear(void) {
  std::lock_guard<std::mutex> lk(g_cache.mu);
  g_cache.lru.clear();
  g_cache.index.clear();
  g_cache.hits = g_cache.misses = g_cache.evictions = 0;
}

uint64_t llk_cache_size(void) {
  std::lock_guard<std::mutex> lk(g_cache.mu);
  return g_cache.lru.size();
}

int llk_plan_find(const llk_kernel_key *key, llk_launch_plan *out) {
  if (!key || !out) return LLK_ERR_ARG;
  const std::string kb = key_bytes(*key);
  std::lock_guard<std::mutex> lk(g_cache.mu);
  auto it = g_cache.index.find(kb);
  if (it == g_cache.index.end()) {
    ++g_cache.misses;
    return LLK_ERR_NOT_FOUND;
  }
  ++g_cache.hits;
  g_cache.lru.splice(g_cache.lru.begin(), g_cache.lru, it->second);
  *out = it->second->plan;
  return LLK_OK;
}

int llk_weight_key_for(const Tensor2D *wg, const Tensor2D *wu, llk_weight_key *out) {
  if (!wg || !wu || !out) return LLK_ERR_ARG;
  std::memset(out, 0, sizeof(*out));
  out->weight_ptr = wg->data;
  // splitmix64 finaliser over the fields that tell two packings apart
  auto mix = [](uint64_t x) {
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
  };
  uint64_t h = 0x6a09e667f3bcc909ull;
  for (uint64_t v : {static_cast<uint64_t>(wg->dim0), static_cast<uint64_t>(wg->dim1),
                     static_cast<uint64_t>(wg->stride0), static_cast<uint64_t>(wu->stride0),
                     static_cast<uint64_t>(reinterpret_cast<uintptr_t>(wu->data))})
    h = mix(h ^ v);
  out->shape_hash = h;
  out->BK = 64;
  out->BN = 64;
  return LLK_OK;
}

}  // extern "C"

namespace {
struct WeightCache {
  struct Entry {
    std::string key;
    llk_packed_weights *pw;
  };
  std::list<Entry> lru;
  std::unordered_map<std::string, std::list<Entry>::iterator> index;
  size_t max_entries = 64;
  uint64_t hits = 0, misses = 0, evictions = 0;
  std::mutex mu;
};
WeightCache g_wcache;

std::string wkey_bytes(const llk_weight_key &k) {
  // field by field: the struct's padding is not part of the key
  std::string b;
  const uintptr_t p = reinterpret_cast<uintptr_t>(k.weight_ptr);
  b.append(reinterpret_cast<const char *>(&p), sizeof(p));
  b.append(reinterpret_cast<const char *>(&k.shape_hash), sizeof(k.shape_hash));
  b.append(reinterpret_cast<const char *>(&k.BK), sizeof(k.BK));
  b.append(reinterpret_cast<const char *>(&k.BN), sizeof(k.BN));
  return b;
}

// Drops entries beyond the maximum; returns the handles to release outside
// the lock (freeing device memory synchronises the device).
std::vector<llk_packed_weights *> wcache_trim() {
  std::vector<llk_packed_weights *> out;
  while (g_wcache.lru.size() > g_wcache.max_entries) {
    out.push_back(g_wcache.lru.back().pw);
    g_wcache.index.erase(g_wcache.lru.back().key);
    g_wcache.lru.pop_back();
    ++g_wcache.evictions;
  }
  return out;
}

void release_all(const std::vector<llk_packed_weights *> &v) {
  for (llk_packed_weights *pw : v) llk_packed_weights_free(pw);
}
}  // namespace

extern "C" {

int llk_lookup_packed_weights(const llk_weight_key *key, llk_packed_weights **out) {
  if (!key || !out) return LLK_ERR_ARG;
  *out = nullptr;
  const std::string kb = wkey_bytes(*key);
  std::lock_guard<std::mutex> lk(g_wcache.mu);
  auto it = g_wcache.index.find(kb);
  if (it == g_wcache.index.end()) {
    ++g_wcache.misses;
    return LLK_ERR_NOT_FOUND;
  }
  ++g_wcache.hits;
  g_wcache.lru.splice(g_wcache.lru.begin(), g_wcache.lru, it->second);
  it->second->pw->refs.fetch_add(1, std::memory_order_relaxed);
  *out = it->second->pw;
  return LLK_OK;
}

int llk_insert_packed_weights(const llk_weight_key *key, llk_packed_weights *pw) {
  if (!key || !pw) return LLK_ERR_ARG;
  const std::string kb = wkey_bytes(*key);
  std::vector<llk_packed_weights *> drop;
  {
    std::lock_guard<std::mutex> lk(g_wcache.mu);
    pw->refs.fetch_add(1, std::memory_order_relaxed);
    auto it = g_wcache.index.find(kb);
    if (it != g_wcache.index.end()) {
      drop.push_back(it->second->pw);
      it->second->pw = pw;
      g_wcache.lru.splice(g_wcache.lru.begin(), g_wcache.lru, it->second);
    } else {
      g_wcache.lru.push_front({kb, pw});
      g_wcache.index[kb] = g_wcache.lru.begin();
      drop = wcache_trim();
    }
  }
  release_all(drop);
  return LLK_OK;
}

int llk_cache_level_stats(int level, uint64_t *hits, uint64_t *misses, uint64_t *evictions, uint64_t *size) {
  uint64_t h = 0, m = 0, e = 0, n = 0;
  if (level == 3) {
    std::lock_guard<std::mutex> lk(g_cache.mu);
    h = g_cache.hits, m = g_cache.misses, e = g_cache.evictions, n = g_cache.lru.size();
  } else if (level == 4) {
    std::lock_guard<std::mutex> lk(g_wcache.mu);
    h = g_wcache.hits, m = g_wcache.misses, e = g_wcache.evictions, n = g_wcache.lru.size();
  } else if (level != 1 && level != 2) {
    return LLK_ERR_ARG;
  }
  if (hits) *hits = h;
  if (misses) *misses = m;
  if (evictions) *evictions = e;
  if (size) *size = n;
  return LLK_OK;
}

int llk_cache_level_set_max_entries(int level, uint64_t max_entries) {
  if (level == 3) {
    llk_cache_set_max_entries(max_entries);
    return LLK_OK;
  }
  if (level == 4) {
    std::vector<llk_packed_weights *> drop;
    {
      std::lock_guard<std::mutex> lk(g_wcache.mu);
      g_wcache.max_entries = max_entries;
      drop = wcache_trim();
    }
    release_all(drop);
    return LLK_OK;
  }
  return level == 1 || level == 2 ? LLK_ERR_UNSUPPORTED : LLK_ERR_ARG;
}

int llk_cache_level_clear(int level) {
  if (level == 3) {
    llk_cache_clear();
    return LLK_OK;
  }
  if (level == 4) {
    std::vector<llk_packed_weights *> drop;
    {
      std::lock_guard<std::mutex> lk(g_wcache.mu);
      for (auto &e : g_wcache.lru) drop.push_back(e.pw);
      g_wcache.lru.clear();
      g_wcache.index.clear();
      g_wcache.hits = g_wcache.misses = g_wcache.evictions = 0;
    }
    release_all(drop);
    return LLK_OK;
  }
  return level == 1 || level == 2 ? LLK_OK : LLK_ERR_ARG;
}


// ------------------------------------------------- column-parallel groups
int llk_peer_group_create(int n_ranks, int rank, int64_t y_bytes, const llk_gpu_context *gpu, llk_peer_group **out,
                          unsigned char *ipc_handle) {
  if (!out || !ipc_handle || n_ranks < 1 || n_ranks > kGroupMax || rank < 0 || rank >= n_ranks || y_bytes < 0)
    return LLK_ERR_ARG;
  *out = nullptr;
  int dev, rc;
  if ((rc = resolve_device(gpu, &dev)) != LLK_OK) return rc;
  DeviceState *ds;
  if ((rc = device_init(dev, &ds)) != LLK_OK) return rc;
  llk_peer_group *g = new llk_peer_group();
  g->device = dev;
  g->n = n_ranks;
  g->rank = rank;
  g->y_bytes = (static_cast<size_t>(y_bytes) + 255) & ~static_cast<size_t>(255);
  if (cudaMalloc(&g->local, kFlagBytes + 2 * g->y_bytes) != cudaSuccess) {
    delete g;
    return LLK_ERR_NOMEM;
  }
  if (cudaMemset(g->local, 0, kFlagBytes) != cudaSuccess || cudaIpcGetMemHandle(&g->handle, g->local) != cudaSuccess) {
    cudaFree(g->local);
    delete g;
    return LLK_ERR_CUDA;
  }
  std::memcpy(ipc_handle, &g->handle, sizeof(g->handle));
  g->base[rank] = g->local;
  *out = g;
  return LLK_OK;
}

int llk_peer_group_connect(llk_peer_group *g, const unsigned char *all_handles) {
  if (!g || !all_handles) return LLK_ERR_ARG;
  if (g->connected) return LLK_OK;
  if (cudaSetDevice(g->device) != cudaSuccess) return LLK_ERR_DEVICE;
  for (int r = 0; r < g->n; ++r) {
    if (r == g->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, all_handles + static_cast<size_t>(r) * LLK_IPC_HANDLE_BYTES, sizeof(h));
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      for (int q = 0; q < r; ++q)
        if (q != g->rank && g->base[q]) cudaIpcCloseMemHandle(g->base[q]);
      for (int q = 0; q < g->n; ++q)
        if (q != g->rank) g->base[q] = nullptr;
      return LLK_ERR_CUDA;
    }
    g->base[r] = static_cast<char *>(p);
  }
  g->connected = true;
  return LLK_OK;
}

int llk_peer_group_y(const llk_peer_group *g, void **y, int64_t *bytes) {
  if (!g) return LLK_ERR_ARG;
  if (y) *y = g->local + kFlagBytes + (g->epoch & 1u) * g->y_bytes;
  if (bytes) *bytes = static_cast<int64_t>(g->y_bytes);
  return LLK_OK;
}

void llk_peer_group_destroy(llk_peer_group *g) {
  if (!g) return;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(g->device);
  for (int r = 0; r < g->n; ++r)
    if (r != g->rank && g->base[r]) cudaIpcCloseMemHandle(g->base[r]);
  cudaFree(g->local);
  cudaSetDevice(cur);
  delete g;
}

int llk_swiglu_column_parallel(const Tensor2D *x, const Tensor2D *wg_shard, const Tensor2D *wu_shard,
                               const llk_packed_weights *pw_shard, int64_t N, llk_peer_group *g,
                               const llk_gpu_context *gpu) {
  if (!x || !g || (!pw_shard && (!wg_shard || !wu_shard)) || N < 0) return LLK_ERR_ARG;
  if (!g->connected) return LLK_ERR_ARG;
  if (gpu && (gpu->math_mode < LLK_MATH_STRICT || gpu->math_mode > LLK_MATH_UNSAFE_FAST)) return LLK_ERR_ARG;
  DeviceRestore restore;
  if (gpu && gpu->device >= 0 && gpu->device != g->device) return LLK_ERR_ARG;
  const int y_f32 = (gpu && gpu->y_dtype == LLK_DTYPE_FP32) ? 1 : 0;
  if (gpu && gpu->y_dtype != LLK_DTYPE_BF16 && gpu->y_dtype != LLK_DTYPE_FP32) return LLK_ERR_ARG;
  const int requested = pack_request(gpu);
  const int64_t M = x->dim0, K = x->dim1;
  int64_t b, e;
  if (llk_shard_columns(N, g->n, g->rank, &b, &e) != LLK_OK) return LLK_ERR_ARG;
  const int64_t w = e - b;
  const int yel = y_f32 ? 4 : 2;
  if (static_cast<size_t>(M) * static_cast<size_t>(N) * yel > g->y_bytes) return LLK_ERR_NOMEM;
  // shapes: X [M, K]; this rank's weights [K, e - b]
  DevTensor dg, du;
  if (pw_shard) {
    if (pw_shard->K != K || pw_shard->N != w || pw_shard->device != g->device) return LLK_ERR_SHAPE;
    dg.data = pw_shard->wg;
    du.data = pw_shard->wu;
    dg.rows = du.rows = K;
    dg.cols = du.cols = w;
    dg.ld = du.ld = 64;
    dg.inner = du.inner = 1;
    dg.slab_major = du.slab_major = 1;
  } else {
    if (wg_shard->dim0 != K || wg_shard->dim1 != w || wu_shard->dim0 != K || wu_shard->dim1 != w)
      return LLK_ERR_SHAPE;
    if (!is_device_ptr(wg_shard->data) || !is_device_ptr(wu_shard->data) ||
        on_other_device(wg_shard->data, g->device) || on_other_device(wu_shard->data, g->device))
      return LLK_ERR_ARG;
    dg = dev_tensor(*wg_shard);
    du = dev_tensor(*wu_shard);
  }
  if (M > 0 && (!is_device_ptr(x->data) || on_other_device(x->data, g->device))) return LLK_ERR_ARG;
  DeviceState *ds;
  int rc;
  if ((rc = device_init(g->device, &ds)) != LLK_OK) return rc;
  cudaStream_t stream = gpu ? static_cast<cudaStream_t>(gpu->stream) : nullptr;
  ++g->epoch;
  const size_t ybuf = kFlagBytes + (g->epoch & 1u) * g->y_bytes;
  char *y_local = g->local + ybuf;
  BarrierArgs exit_ = barrier_args(*g, 0);
  if (M > 0 && w > 0) {
    DevTensor dx = dev_tensor(*x), dy;
    dy.data = y_local + static_cast<size_t>(b) * yel;
    dy.rows = M;
    dy.cols = w;
    dy.ld = N;
    dy.inner = 1;
    PeerTargets peers;
    for (int r = 0; r < g->n; ++r)
      if (r != g->rank) peers.y[peers.n++] = g->base[r] + ybuf + static_cast<size_t>(b) * yel;
    // TMA store maps over every rank's whole buffer (own first) when the
    // row pitch is a multiple of 16 bytes; else per-thread stores.
    YStoreMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    if ((N * yel) % 16 == 0) {
      maps.col0 = static_cast<int>(b);
      if (encode_ystore_map(&maps.m[maps.n++], y_local, N, M, y_f32) != LLK_OK) return LLK_ERR_ALIGN;
      for (int r = 0; r < g->n; ++r)
        if (r != g->rank && encode_ystore_map(&maps.m[maps.n++], g->base[r] + ybuf, N, M, y_f32) != LLK_OK)
          return LLK_ERR_ALIGN;
      peers.maps = &maps;
    }
    bool fused = false;
    {
      std::lock_guard<std::mutex> lk(ds->mu);
      rc = launch_device(*ds, LLK_OP_FUSED_SWIGLU, dx, dg, du, dy, y_f32, 0, requested, nullptr, 0, stream,
                         &peers, &fused);
    }
    if (rc != LLK_OK) return rc;
    if (!fused) {
      // Kernels without the fused epilogue (small M): copy engines move
      // this rank's columns to every peer over NVLink.
      for (int i = 0; i < peers.n; ++i)
        if (cudaMemcpy2DAsync(peers.y[i], static_cast<size_t>(N) * yel, dy.data, static_cast<size_t>(N) * yel,
                              static_cast<size_t>(w) * yel, static_cast<size_t>(M), cudaMemcpyDeviceToDevice,
                              stream) != cudaSuccess)
          return LLK_ERR_CUDA;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, peer_barrier_kernel, exit_, g->n, g->epoch, ds->status) == cudaSuccess
             ? LLK_OK
             : LLK_ERR_CUDA;
}

}  // extern "C"
