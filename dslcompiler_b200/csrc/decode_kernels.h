// decode_kernels.h -- launch interface of the small-M (decode) SwiGLU kernel.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace llk_b200 {

struct DecodePlan {
  int block_m, block_n, block_k, stages, split_k, grid, threads, smem_bytes;
  // 0: stream-K split of the (tile, k-block) units over `grid` CTAs,
  // partial sums through the workspace.  s >= 2: grid = tiles x s CTAs in
  // clusters of s, one cluster per tile, partial sums through distributed
  // shared memory.
  int cluster;
};

// Largest M the decode kernel serves.
int decode_max_m();
// Whether the decode kernel handles this shape / output type.
bool decode_supported(int64_t M, int64_t N, int64_t K, int y_f32);
DecodePlan decode_plan(int64_t M, int64_t N, int64_t K, int sm_count);
// Device workspace a launch of plan d needs (layout in workspace.h): the
// counter regions, and for a stream-K plan whose CTA ranges start inside
// tiles two partial-sum slots per CTA.
size_t decode_workspace_bytes(int64_t M, int64_t N, int64_t K, const DecodePlan &d);
// Largest grid whose partial-sum slots fit in `workspace_bytes`.
int decode_max_grid_for(int64_t M, size_t workspace_bytes);
// Byte offset and size of the per-tile counters inside the workspace; they
// must be zero before the first launch (each launch leaves them zero again).
size_t decode_counter_offset(int64_t M, int64_t N);
size_t decode_counter_bytes(int64_t N);
// Whether a plan (possibly a tuned override) is launchable for this shape.
bool decode_plan_valid(int64_t M, int64_t N, int64_t K, const DecodePlan &d);
// wg, wu: weight tensor maps with a 64-column x 64-k box (2-D over
// row-major [K, N], or 3-D over slab-major packed weights when slab_major);
// x: token tensor map, box {64 k, d.block_m rows}.  fast_math: the fast
// SwiGLU epilogue instead of the strict one (separate kernel instantiations).
cudaError_t decode_launch(const CUtensorMap &wg, const CUtensorMap &wu, const CUtensorMap &x, void *y, int64_t ldy,
                          int y_f32, int64_t M, int64_t N, int64_t K, void *workspace, int *status,
                          const DecodePlan &d, int slab_major, int fast_math, cudaStream_t stream);

}  // namespace llk_b200
