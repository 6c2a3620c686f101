// attention_kernels.h -- launch interface of the llk.rope and llk.attention
// kernels (rope_attention.cu).  All tensors are contiguous, row-major, f32
// (position ids i64), device memory.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace llk_b200 {

bool rope_supported(int64_t B, int64_t H, int64_t L, int64_t D);
// Device bytes of the (cos, sin) table a launch builds: L x D/2 float2.
size_t rope_table_bytes(int64_t L, int64_t D);
// y [B,H,L,D] = RoPE(x [B,H,L,D], position_ids [L], theta); y may be x.
// table: rope_table_bytes(L, D) of device scratch (16-byte aligned).
cudaError_t rope_launch(const float *x, const int64_t *pos, float *y, int64_t B, int64_t H, int64_t L, int64_t D,
                        double theta, int fast_math, void *table, int sm_count, cudaStream_t stream);

bool attention_supported(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D);
// o [B,H,Lq,D] += softmax(scale * q k^T (+ causal mask)) v, with q
// [B,H,Lq,D], k / v [B,H,Lk,D]; o must not alias q, k or v.
cudaError_t attention_launch(const float *q, const float *k, const float *v, float *o, int64_t B, int64_t H,
                             int64_t Lq, int64_t Lk, int64_t D, float scale, int causal, int fast_math,
                             cudaStream_t stream);

}  // namespace llk_b200
