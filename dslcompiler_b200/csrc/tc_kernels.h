// tc_kernels.h -- launch interface of the device kernels (host side).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace llk_b200 {

// Output modes of the tcgen05 kernel.
enum TcMode { TC_SWIGLU_BF16 = 0, TC_SWIGLU_F32 = 1, TC_MATMUL_F32 = 2, TC_MATMUL_F32_ACC = 3 };
// Flag or-ed into a SwiGLU mode: the fast epilogue (__expf, __fdividef:
// math_mode bounded_fast / unsafe_fast) instead of the strict one (expf and
// an IEEE division).  Each combination is its own kernel instantiation.
constexpr int TC_FAST_MATH = 8;

struct TcParams {
  int M, N, K;        // problem: Y[M,N], reduction K
  int m_tiles;        // ceil(M / 128)
  int n_tiles;        // ceil(N / tile_n)
  int num_tiles;      // m_tiles * n_tiles
  int k_blocks;       // ceil(K / 64)
  int vec_ok;         // Y base and row stride allow 16-byte stores
  void *y;            // Y (bf16 or f32), row stride ldy elements
  int64_t ldy;
  int *status;        // device-visible error word (LLK_ERR_TIMEOUT on a wait that gave up)
  uint32_t b_lbo;     // MN-major B descriptor: bytes between 64-column slabs
  uint32_t b_sbo;     // MN-major B descriptor: bytes between 8-row k groups
  int slab_major;     // B tensor maps describe slab-major packed weights (3-D)
  // CTA-pair kernel work split (filled by tc2_launch): dp_waves waves of
  // whole tiles, one pair per tile; the tiles left over are cut along N into
  // tail_split narrower tiles (1, 2 or 4) dealt round-robin over the pairs.
  int dp_waves;
  int tail_split;
  // Dynamic scheduling (dynamic != 0): each pair's leader draws work items
  // 0 .. n_items-1 (whole tiles, then tail parts) from *sched_counter, a
  // zeroed device int that the last draw of a launch sets back to zero.
  int dynamic;
  int n_items;
  int *sched_counter;
  // Tile order (CTA-pair kernel, filled by tc2_launch): tiles run in bands of
  // group_m row blocks; inside a band the row block varies fastest, then the
  // column tile, so one band's X rows stay in L2 while the band sweeps N.
  int group_m;
  // K-split tail (CTA-pair kernel, static schedule): when ksplit >= 2 the
  // leftover tiles are not cut along N but along K into ksplit parts, each on
  // its own pair in the last wave.  Every part writes the accumulator columns
  // it does not own to tail_ws, waits (bounded) until all parts of the tile
  // have written, then sums the columns it owns over all parts in part order
  // (deterministic) and runs the epilogue on them.  tail_cnt: zeroed device
  // ints, two per (leftover tile, CTA of the pair, epilogue warp); the last
  // part to finish sets them back to zero.
  int ksplit;
  float *tail_ws;
  int *tail_cnt;
  // Column-parallel all-gather fused into the epilogue (CTA-pair kernel):
  // every Y chunk is also stored at the same offsets from y_peers[0..n_peers)
  // -- other GPUs' Y buffers mapped into this process -- so the shards
  // travel over NVLink while later tiles compute.
  int n_peers;
  void *y_peers[7];
};
constexpr int kMaxYPeers = 7;

// TMA store maps of the output (CTA-pair kernel): when n > 0 the SwiGLU
// epilogue stages each 32 x 32 chunk in shared memory and stores it with
// TMA through every map -- this GPU's Y and the peers' -- at column
// col0 + (column in this launch's Y).  Maps: dims {N_full, M}, box {32, 32},
// bf16 with 64-byte swizzle or f32 with 128-byte swizzle.
struct YStoreMaps {
  CUtensorMap m[kMaxYPeers + 1];
  int n;
  int col0;
};

int tc_smem_bytes();
// CTA-pair (cta_group::2) variant: m_tiles counts 256-row blocks; grid =
// 2 x min(tiles, co-resident pairs, max_pairs if > 0).  tail_split: 0 =
// choose, 1/2/4 = cut the leftover tiles into that many column parts.
int tc2_smem_bytes();
// tail_split: 0 = choose, 1/2/4 = cut the leftover tiles into that many
// column parts, -s (2 <= s <= 8) = split them along K into s parts.
// sched_counter: a zeroed device int for the dynamic scheduler, or nullptr
// for the static round-robin schedule.
// workspace / workspace_bytes: the call's workspace (layout in workspace.h,
// counter regions zero) for the K-split tail, or nullptr; without room for
// the chosen split's partial sums the tail is cut along N instead.
// ym: TMA store maps of Y (nullptr: per-thread stores to p.y / p.y_peers).
cudaError_t tc2_launch(int mode, const CUtensorMap &a, const CUtensorMap &b0, const CUtensorMap &b1,
                       TcParams p, int max_pairs, int tail_split, int *sched_counter, void *workspace,
                       size_t workspace_bytes, cudaStream_t stream, const YStoreMaps *ym = nullptr);
// Device bytes the dynamic scheduler needs (one zeroed int).
constexpr size_t kTc2SchedBytes = 256;
// Workspace the K-split tail may need on a GPU with `sm_count` SMs: the
// counter regions and the partial sums of at most one part per pair.
size_t tc2_tail_workspace_bytes(int sm_count);
// The CTA-pair kernel's schedule enumerated on the host (the planner and the
// item mapping the kernel runs): per work item 9 ints {pair (-1: dynamic),
// row tile, column tile, first column, width, first k-block, end k-block,
// K part, K parts}.  Returns 0, or -1 on bad arguments.
int tc2_schedule_items(int swiglu, int64_t M, int64_t N, int64_t K, int pairs, int tail_split, int dynamic,
                       size_t workspace_bytes, int *items, int max_items, int *n_items, int *n_pairs, int *ksplit,
                       int *tail_split_out);
int tc_threads();
int tc_tile_n(int mode);
cudaError_t tc_launch(int mode, const CUtensorMap &a, const CUtensorMap &b0, const CUtensorMap &b1,
                      const TcParams &p, int grid, cudaStream_t stream);

// CUDA-core kernel for any strides / alignment (small or odd shapes).
// x, wg, wu bf16; y bf16 (y_f32 == 0) or f32.  mode 0 = swiglu, 1 = matmul,
// 2 = matmul accumulating into y.  slab_major: wg/wu are slab-major packed
// weights ([N/64][K][64]; ld/stride arguments ignored).  fast_math: the fast
// SwiGLU epilogue instead of the strict one.
cudaError_t simt_launch(int mode, const void *x, int64_t ldx, int64_t sxk, const void *wg, const void *wu,
                        int64_t ldw, int64_t swn, int64_t ldwu, int64_t swun, void *y, int64_t ldy, int64_t syn,
                        int y_f32, int64_t M, int64_t N, int64_t K, int slab_major, int fast_math,
                        cudaStream_t stream);

// Diagnostic: a bounded wait that is made to expire (see swiglu_simt.cu).
cudaError_t diag_timeout_launch(int *status, uint64_t limit_ns, cudaStream_t stream);
// Diagnostic: counts the floats with bit patterns in [lo, hi) on which the
// strict epilogue's reciprocal differs from CUDA's correctly rounded one.
cudaError_t diag_reciprocal_launch(unsigned long long *mismatches, uint32_t lo, uint32_t hi, int sm_count,
                                   cudaStream_t stream);

}  // namespace llk_b200
