// swiglu_simt.cu -- CUDA-core kernel for the fused SwiGLU / matmul on any
// strides and alignments (shapes the TMA path cannot describe: odd row
// pitches such as N = 127, non-unit inner strides, unaligned pointers).
// It is a correctness path for small or irregular shapes, not a fast path;
// it keeps the reference's accumulation contract (f32, k ascending;
// lib/Transforms/FuseDoubleContraction.cpp:155-173) and epilogue (:179-199).
#include <cuda_runtime.h>

#include <cstdint>

#include "sm100_ptx.cuh"
#include "tc_kernels.h"

namespace llk_b200 {

namespace {

__device__ __forceinline__ float bf16_at(const uint16_t *p, int64_t i) {
  return __uint_as_float(static_cast<uint32_t>(p[i]) << 16);
}

// One thread per output element; 32 consecutive columns per warp so the
// weight reads of a warp are contiguous when the inner stride is 1.
// MODE: 0 = SwiGLU (strict epilogue), 3 = SwiGLU (fast epilogue), 1 = matmul,
// 2 = matmul accumulating into y.
template <int MODE>
__global__ void __launch_bounds__(256) simt_kernel(const uint16_t *__restrict__ x, int64_t ldx, int64_t sxk,
                                                   const uint16_t *__restrict__ wg, int64_t ldw, int64_t swn,
                                                   const uint16_t *__restrict__ wu, int64_t ldwu, int64_t swun,
                                                   void *y, int64_t ldy, int64_t syn, int y_f32, int64_t M,
                                                   int64_t N, int64_t K, int slab_major) {
  const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t m = blockIdx.y;
  if (n >= N || m >= M) return;
  // Element (k, n) of a weight: row-major with strides, or slab-major
  // packed ([n / 64][k][n % 64]).
  int64_t wbase = 0, wk = ldw, wbase_u = 0, wk_u = ldwu;
  if (slab_major) {
    wbase = wbase_u = (n >> 6) * K * 64 + (n & 63);
    wk = wk_u = 64;
  } else {
    wbase = n * swn;
    wbase_u = n * swun;
  }
  float g = 0.0f, u = 0.0f;
  for (int64_t k = 0; k < K; ++k) {
    const float xv = bf16_at(x, m * ldx + k * sxk);
    g = fmaf(xv, bf16_at(wg, wbase + k * wk), g);
    if (MODE == 0 || MODE == 3) u = fmaf(xv, bf16_at(wu, wbase_u + k * wk_u), u);
  }
  float r;
  if (MODE == 0 || MODE == 3) {
    r = silu_mul_mode<MODE == 3>(g, u);
  } else {
    r = g;
  }
  const int64_t o = m * ldy + n * syn;
  if (y_f32) {
    float *yf = static_cast<float *>(y);
    if (MODE == 2) r += yf[o];
    yf[o] = r;
  } else {
    static_cast<uint16_t *>(y)[o] = static_cast<uint16_t>(pack_bf16x2(r, 0.0f));
  }
}

}  // namespace

cudaError_t simt_launch(int mode, const void *x, int64_t ldx, int64_t sxk, const void *wg, const void *wu,
                        int64_t ldw, int64_t swn, int64_t ldwu, int64_t swun, void *y, int64_t ldy, int64_t syn,
                        int y_f32, int64_t M, int64_t N, int64_t K, int slab_major, int fast_math,
                        cudaStream_t stream) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  if (M > 65535) return cudaErrorInvalidValue;
  dim3 block(256);
  dim3 grid(static_cast<unsigned>((N + 255) / 256), static_cast<unsigned>(M));
  const uint16_t *xp = static_cast<const uint16_t *>(x);
  const uint16_t *gp = static_cast<const uint16_t *>(wg);
  const uint16_t *up = static_cast<const uint16_t *>(wu);
  switch (mode) {
    case 0:
      if (fast_math)
        simt_kernel<3><<<grid, block, 0, stream>>>(xp, ldx, sxk, gp, ldw, swn, up, ldwu, swun, y, ldy, syn, y_f32, M,
                                                   N, K, slab_major);
      else
        simt_kernel<0><<<grid, block, 0, stream>>>(xp, ldx, sxk, gp, ldw, swn, up, ldwu, swun, y, ldy, syn, y_f32, M,
                                                   N, K, slab_major);
      break;
    case 1:
      simt_kernel<1><<<grid, block, 0, stream>>>(xp, ldx, sxk, gp, ldw, swn, gp, ldw, swn, y, ldy, syn, 1, M, N, K,
                                                 slab_major);
      break;
    case 2:
      simt_kernel<2><<<grid, block, 0, stream>>>(xp, ldx, sxk, gp, ldw, swn, gp, ldw, swn, y, ldy, syn, 1, M, N, K,
                                                 slab_major);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace llk_b200

// ------------------------------------------------------------------ diag
// A kernel that waits on an mbarrier nothing will ever arrive at, with the
// same bounded wait the production kernels use.  The wait gives up after
// `limit_ns`, records LLK_ERR_TIMEOUT in the device status word and the
// kernel returns normally, leaving the context usable.  It exists so the
// timeout path can be exercised on a GPU without faulting or hanging it.
namespace llk_b200 {
namespace {
__global__ void diag_timeout_kernel(int *status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!mbar_wait_bounded(&bar, 0, &abort, LLK_ERR_TIMEOUT, limit_ns)) atomicExch(status, abort);
  }
}
}  // namespace

cudaError_t diag_timeout_launch(int *status, uint64_t limit_ns, cudaStream_t stream) {
  diag_timeout_kernel<<<1, 32, 0, stream>>>(status, limit_ns);
  return cudaGetLastError();
}

// The strict epilogue's reciprocal (rcp_rn_ge1) against CUDA's correctly
// rounded reciprocal on every float whose bit pattern is in [lo, hi).
namespace {
__global__ void diag_reciprocal_kernel(unsigned long long *mismatches, uint32_t lo, uint32_t hi) {
  unsigned long long n = 0;
  for (uint64_t i = lo + static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < hi;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const float b = __uint_as_float(static_cast<uint32_t>(i));
    if (__float_as_uint(rcp_rn_ge1(b)) != __float_as_uint(__frcp_rn(b))) ++n;
  }
  if (n) atomicAdd(mismatches, n);
}
}  // namespace

cudaError_t diag_reciprocal_launch(unsigned long long *mismatches, uint32_t lo, uint32_t hi, int sm_count,
                                   cudaStream_t stream) {
  diag_reciprocal_kernel<<<8 * sm_count, 256, 0, stream>>>(mismatches, lo, hi);
  return cudaGetLastError();
}
}  // namespace llk_b200
