// swiglu_decode_noalloc.cu -- llk_swiglu_decode_noalloc: the small-M
// (decode) fused SwiGLU for callers that must not allocate device memory.
//
// Who needs it: code that runs where cudaMalloc/cudaFree is not allowed or
// not safe -- a serving loop whose device memory is entirely owned by
// another allocator (a framework's caching allocator that has reserved the
// HBM, so a raw cudaMalloc fails or fragments it), or a latency-critical
// path where cudaMalloc/cudaFree would add host round trips and implicit
// device-wide synchronisation.  The ordinary decode path (llk_swiglu_ex)
// grows a library-owned workspace with cudaMalloc on first use unless the
// caller hands it scratch; this entry point instead uses the fixed array
// below, which the CUDA runtime places in device memory when the library's
// module is loaded, so a call never allocates.
//
// The array, g_decode_scratch, is a file-scope __device__ variable: every
// GPU that loads the library holds LLK_DECODE_NOALLOC_SCRATCH_BYTES of it
// until the process exits.  In host code its name is only a host-side
// stand-in, not a device address, so the host looks its address up with
// cudaGetSymbolAddress -- once per device, with that device current -- and
// passes that address to the kernel.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "decode_kernels.h"
#include "llk_b200.h"

namespace {

using namespace llk_b200;

constexpr int kMaxDevices = 64;

// The scratch every call of llk_swiglu_decode_noalloc shares.
static __device__ __align__(256) unsigned char g_decode_scratch[LLK_DECODE_NOALLOC_SCRATCH_BYTES];

struct DeviceSetup {
  std::mutex mu;
  std::atomic<bool> ready{false};  // set once a set-up succeeded; a failed one is retried
  void *scratch = nullptr;         // device address of g_decode_scratch on this device
  int sm_count = 0;
};
DeviceSetup g_setup[kMaxDevices];

PFN_cuTensorMapEncodeTiled_v12000 g_encode_fn = nullptr;
std::mutex g_encode_mu;

// One-time set-up for `dev`, which the caller has made current: the device
// address of the scratch array, the SM count, the tensor-map encoder.
// Returns LLK_OK and marks the device ready, or an error and leaves it
// unmarked so that a later call tries again.
int setup_device(int dev, DeviceSetup &s) {
  std::lock_guard<std::mutex> lk(s.mu);
  if (s.ready) return LLK_OK;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
    cudaGetLastError();
    return LLK_ERR_DEVICE;
  }
  if (prop.major != 10 || prop.minor != 0) return LLK_ERR_DEVICE;
  void *ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_decode_scratch) != cudaSuccess || ptr == nullptr) {
    cudaGetLastError();
    return LLK_ERR_CUDA;
  }
  {
    std::lock_guard<std::mutex> ek(g_encode_mu);
    if (!g_encode_fn) {
      void *fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || fn == nullptr) {
        cudaGetLastError();
        return LLK_ERR_DEVICE;
      }
      g_encode_fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  s.scratch = ptr;
  s.sm_count = prop.multiProcessorCount;
  s.ready = true;
  return LLK_OK;
}

// Whether the kernel on `dev` may read / write p: device memory of `dev` or
// managed memory.  Host memory (even pinned and mapped) is refused, since
// staging it would need device memory; so is another GPU's memory, which the
// kernel could only reach through peer access this call cannot vouch for.
bool usable_on(const void *p, int dev) {
  cudaPointerAttributes a;
  if (p == nullptr || cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (a.type == cudaMemoryTypeManaged) return true;
  return a.type == cudaMemoryTypeDevice && a.device == dev;
}

// Restores the caller's current device when the call returns.
struct DeviceGuard {
  int prev = -1;
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 2-D bf16 tensor map over a row-major matrix, 128-byte swizzle, zero fill.
bool encode(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer, uint64_t pitch_bytes,
            uint32_t box_inner, uint32_t box_outer) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return g_encode_fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int llk_swiglu_decode_noalloc(const Tensor2D *x, const Tensor2D *wg, const Tensor2D *wu, Tensor2D *y,
                                         int *device_status, const llk_gpu_context *gpu) {
  if (!x || !wg || !wu || !y) return LLK_ERR_ARG;
  if (x->dim1 != wg->dim0 || x->dim1 != wu->dim0 || wg->dim1 != wu->dim1 || y->dim0 != x->dim0 ||
      y->dim1 != wg->dim1)
    return LLK_ERR_SHAPE;
  const int64_t M = x->dim0, K = x->dim1, N = wg->dim1;
  if (M < 1 || K < 1 || N < 1 || M > 128) return LLK_ERR_UNSUPPORTED;
  const int y_dtype = gpu ? gpu->y_dtype : LLK_DTYPE_BF16;
  if (y_dtype != LLK_DTYPE_BF16 && y_dtype != LLK_DTYPE_FP32) return LLK_ERR_ARG;
  const int y_f32 = y_dtype == LLK_DTYPE_FP32 ? 1 : 0;
  if (gpu && (gpu->math_mode < LLK_MATH_STRICT || gpu->math_mode > LLK_MATH_UNSAFE_FAST)) return LLK_ERR_ARG;

  // The array's fixed size is the limit: the per-tile arrival counters
  // (one int per 128 columns, up to N = LLK_DECODE_NOALLOC_MAX_N) and at
  // least one CTA's partial-sum slots must fit.  Beyond that the call is
  // refused, never allocated.
  if (N > LLK_DECODE_NOALLOC_MAX_N || decode_max_grid_for(M, LLK_DECODE_NOALLOC_SCRATCH_BYTES) < 1)
    return LLK_ERR_NOMEM;
  if (!decode_supported(M, N, K, y_f32)) return LLK_ERR_UNSUPPORTED;

  int dev = gpu ? gpu->device : -1;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) return LLK_ERR_DEVICE;
  if (dev < 0) dev = cur;
  if (dev >= kMaxDevices) return LLK_ERR_ARG;
  DeviceGuard restore;
  if (cur != dev) {
    if (cudaSetDevice(dev) != cudaSuccess) {
      cudaGetLastError();
      return LLK_ERR_DEVICE;
    }
    restore.prev = cur;
  }
  DeviceSetup &s = g_setup[dev];
  if (!s.ready) {
    const int rc = setup_device(dev, s);
    if (rc != LLK_OK) return rc;
  }

  // Device buffers reachable from `dev` only: staging host data would need
  // device memory, and a buffer on an unreachable GPU would fault the kernel.
  if (!usable_on(x->data, dev) || !usable_on(wg->data, dev) || !usable_on(wu->data, dev) ||
      !usable_on(y->data, dev))
    return LLK_ERR_ARG;
  const uintptr_t y_align = y_f32 ? 4u : 2u;
  if (x->stride1 != 1 || wg->stride1 != 1 || wu->stride1 != 1 || y->stride1 != 1) return LLK_ERR_ALIGN;
  if (!aligned16(x->data) || !aligned16(wg->data) || !aligned16(wu->data) || (x->stride0 * 2) % 16 != 0 ||
      (wg->stride0 * 2) % 16 != 0 || (wu->stride0 * 2) % 16 != 0 || x->stride0 < K || wg->stride0 < N ||
      wu->stride0 < N || y->stride0 < N || (reinterpret_cast<uintptr_t>(y->data) & (y_align - 1)) != 0)
    return LLK_ERR_ALIGN;

  cudaStream_t stream = gpu ? static_cast<cudaStream_t>(gpu->stream) : nullptr;
  DecodePlan d = decode_plan(M, N, K, s.sm_count);
  // Fewer CTAs when a stream-K grid's partial-sum slots would not fit the
  // array (only for M > 32).
  if (decode_workspace_bytes(M, N, K, d) > LLK_DECODE_NOALLOC_SCRATCH_BYTES)
    d.grid = decode_max_grid_for(M, LLK_DECODE_NOALLOC_SCRATCH_BYTES);
  CUtensorMap tg, tu, tx;
  if (!encode(&tg, wg->data, N, K, wg->stride0 * 2, 64, 64) ||
      !encode(&tu, wu->data, N, K, wu->stride0 * 2, 64, 64) ||
      !encode(&tx, x->data, K, M, x->stride0 * 2, 64, d.block_m))
    return LLK_ERR_ALIGN;

  // The array keeps whatever the previous call left in it.  The per-tile
  // arrival counters must start at zero, so clear them (a memset, not an
  // allocation); the partial-sum slots are always written before they are read.
  char *scratch = static_cast<char *>(s.scratch);
  if (cudaMemsetAsync(scratch + decode_counter_offset(M, N), 0, decode_counter_bytes(N), stream) != cudaSuccess)
    return LLK_ERR_CUDA;
  cudaError_t e =
      decode_launch(tg, tu, tx, y->data, y->stride0, y_f32, M, N, K, scratch, device_status, d, 0,
                    gpu && gpu->math_mode != LLK_MATH_STRICT ? 1 : 0, stream);
  return e == cudaSuccess ? LLK_OK : LLK_ERR_CUDA;
}
