// shard_gather.cu -- relayout after an all-gather of column shards.
//
// Column-parallel SwiGLU leaves rank r with Y[:, b_r:e_r].  An all-gather of
// equal-sized (padded) shard buffers yields shard-major data
// [n_shards][M][width]; this kernel writes it into the row-major Y[M, N] the
// caller wants.  The shard offsets travel as a kernel argument (at most
// kMaxShards), so the call allocates nothing.
#include <cuda_runtime.h>

#include <cstdint>

#include "llk_b200.h"

namespace llk_b200 {
namespace {

constexpr int kMaxShards = 64;

struct ShardBegins {
  int64_t b[kMaxShards + 1];
};

// grid.y = shard, grid.z strides over rows; x over the shard's columns.
template <typename T>
__global__ void gather_columns_kernel(const T *__restrict__ src, int64_t width, int64_t M, const ShardBegins begins,
                                      T *__restrict__ y, int64_t ldy) {
  const int s = blockIdx.y;
  const int64_t b = begins.b[s], w = begins.b[s + 1] - b;
  const T *shard = src + static_cast<int64_t>(s) * M * width;
  for (int64_t m = blockIdx.z; m < M; m += gridDim.z)
    for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < w;
         c += static_cast<int64_t>(gridDim.x) * blockDim.x)
      y[m * ldy + b + c] = shard[m * width + c];
}

}  // namespace
}  // namespace llk_b200

using namespace llk_b200;

extern "C" int llk_gather_columns(const void *shards, int n_shards, int64_t M, int64_t width, const int64_t *begins,
                                  void *y, int64_t ldy, int elem_bytes, const llk_gpu_context *gpu) {
  if (!shards || !y || !begins || n_shards < 1 || n_shards > kMaxShards || M < 0 || width < 0) return LLK_ERR_ARG;
  if (elem_bytes != 2 && elem_bytes != 4) return LLK_ERR_ARG;
  ShardBegins sb;
  for (int i = 0; i <= n_shards; ++i) {
    sb.b[i] = begins[i];
    if (i > 0 && (begins[i] < begins[i - 1] || begins[i] - begins[i - 1] > width)) return LLK_ERR_SHAPE;
  }
  if (begins[n_shards] > ldy) return LLK_ERR_SHAPE;
  if (M == 0 || width == 0) return LLK_OK;
  cudaStream_t stream = gpu ? static_cast<cudaStream_t>(gpu->stream) : nullptr;
  if (gpu && gpu->device >= 0 && cudaSetDevice(gpu->device) != cudaSuccess) return LLK_ERR_DEVICE;
  const int64_t rows = M < 2048 ? M : 2048;
  dim3 block(256);
  dim3 grid(static_cast<unsigned>((width + 255) / 256 < 32 ? (width + 255) / 256 : 32),
            static_cast<unsigned>(n_shards), static_cast<unsigned>(rows));
  if (elem_bytes == 2)
    gather_columns_kernel<uint16_t><<<grid, block, 0, stream>>>(static_cast<const uint16_t *>(shards), width, M, sb,
                                                                 static_cast<uint16_t *>(y), ldy);
  else
    gather_columns_kernel<float><<<grid, block, 0, stream>>>(static_cast<const float *>(shards), width, M, sb,
                                                              static_cast<float *>(y), ldy);
  return cudaGetLastError() == cudaSuccess ? LLK_OK : LLK_ERR_CUDA;
}
