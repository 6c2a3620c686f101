// swiglu_tc2.cu -- the prefill SwiGLU / micro.mma kernel on CTA PAIRS
// (tcgen05 cta_group::2): one MMA instruction spans two SMs.
//
// Why: with one CTA issuing 128x256x16 MMAs, every MMA reads 4 KB of A and
// 8 KB of B from that SM's shared memory while TMA fills the next stages;
// the shared-memory operand path, not the tensor pipe, is the limiter (ncu:
// ~80 % busy with the tensor pipe at ~71 %).  A pair issues 256x256x16 MMAs in
// which each SM supplies 128 rows of A and HALF of B (128 columns), so the B
// bytes each SM reads and loads per FLOP halve.
//
// Per pair and tile: Y rows [m0, m0+256) x 128 columns (SwiGLU: B = [Wg 128
// columns from the leader CTA | Wu 128 columns from the peer CTA], so gate
// lands in TMEM columns 0-127 and up in 128-255 of each CTA's accumulator),
// or a 256 x 256 C tile (matmul: B columns n0.. from the leader, n0+128..
// from the peer).
//
// Roles per CTA (6 warps), cluster = the pair:
//   warp 0     TMA producer, both CTAs: own 128 rows of X and own B half into
//              own shared memory; completion bytes go to the LEADER's full
//              barrier (2-SM TMA form).  The leader alone posts the expected
//              byte count of both CTAs.
//   warp 1     TMEM owner in both CTAs (paired alloc); in the leader, the
//              single MMA-issuing thread; its commits arrive on the stage /
//              accumulator barriers of both CTAs.
//   warps 2-5  epilogue in both CTAs on their own TMEM rows; each thread
//              releases the accumulator by arriving on the leader's barrier.
// Work split: floor(tiles / pairs) waves of whole tiles, one pair per tile;
// the tiles left over would run as a partly idle last wave, so they may be
// cut along N into 2 or 4 narrower tiles (MMA N = 128 or 64) dealt
// round-robin over all pairs -- whichever split makes the last wave shortest
// under the measured cost of a part.  No partial sums, no fix-up: every
// output is still written once from TMEM.
//
// All waits bounded; no TMA multicast (each CTA loads its own tiles).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>

#include "sm100_ptx.cuh"
#include "tc_kernels.h"
#include "workspace.h"

namespace llk_b200 {

namespace {

constexpr int kThreads = 192;
constexpr int kStages = 6;
constexpr int kRows = 128;                          // rows of X per CTA
constexpr int kBK = 64;
constexpr int kMmaN = 256;
constexpr uint32_t kABytes = kRows * kBK * 2;       // 16 KB
constexpr uint32_t kSlabBytes = 64 * kBK * 2;       // 8 KB
constexpr uint32_t kBBytes = 2 * kSlabBytes;        // 16 KB: this CTA's 128 columns
constexpr uint32_t kStageBytes = kABytes + kBBytes;  // 32 KB
constexpr uint32_t kTmemCols = 512;
// Epilogue staging for TMA stores of Y: 8 KB per epilogue warp (4 chunks of
// 32 x 32 bf16 or 2 of 32 x 32 f32), 1024-byte aligned after the stages.
constexpr uint32_t kStagingPerWarp = 8192;
constexpr uint32_t kStagingBytes = 4 * kStagingPerWarp;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// One unit of a pair's work: Y columns [c0, c0 + wn) of tile `tile`, over
// the k-blocks [kb0, kb1); part `part` of `nparts` K parts of the tile
// (nparts = 1: the whole reduction).
struct Work {
  int tile, c0, wn;
  int kb0, kb1, part, nparts;
};

// Work item `item` of the launch: items [0, whole) are whole tiles (whole =
// dp_waves x pairs), the rest are the parts of the leftover tiles: ksplit
// K parts each, or else tail_split column parts.  False past the last item.
template <int TILE_N>
__host__ __device__ __forceinline__ bool item_to_work(const TcParams &p, int n_pairs, int item, Work &w) {
  const int whole = p.dp_waves * n_pairs;
  w.c0 = 0;
  w.wn = TILE_N;
  w.kb0 = 0;
  w.kb1 = p.k_blocks;
  w.part = 0;
  w.nparts = 1;
  if (item < whole) {
    w.tile = item;
    return true;
  }
  const int j = item - whole;
  if (p.ksplit > 1) {
    if (j >= (p.num_tiles - whole) * p.ksplit) return false;
    w.tile = whole + j / p.ksplit;
    w.part = j % p.ksplit;
    w.nparts = p.ksplit;
    w.kb0 = w.part * p.k_blocks / p.ksplit;
    w.kb1 = (w.part + 1) * p.k_blocks / p.ksplit;
    return true;
  }
  if (j >= (p.num_tiles - whole) * p.tail_split) return false;
  w.tile = whole + j / p.tail_split;
  w.wn = TILE_N / p.tail_split;
  w.c0 = (j % p.tail_split) * w.wn;
  return true;
}

// Epilogue of one K part of a K-split leftover tile, for one epilogue warp
// (TMEM lane quarter q = rows q*32 .. q*32+31 of this CTA's 128).  The
// accumulator columns are cut into 16-column chunks of Y (SwiGLU: gate and
// up columns of those Y columns; matmul: C columns), chunk c owned by part
// c % nparts.  1. Write the chunks this part does not own to its partial
// block.  2. Publish (fence + counter) and wait, bounded, until every part
// of the tile has.  3. For each owned chunk, add the parts' sums in part
// order -- this part's straight from TMEM -- and run the epilogue.  4. The
// last part to get here sets the tile's counters back to zero.
// Partial block of (leftover tile, part, CTA rank): 64 float4 columns x 128
// rows, float4-column-major, so a warp's 32 rows of one float4 column are
// 512 contiguous bytes.  Returns false when the wait gave up.
template <int MODE>
__device__ __forceinline__ bool ksplit_epilogue(const TcParams &p, const Work &w, int tl, uint32_t rank, int q,
                                                int lane, uint32_t t_row, int m0, int n0, volatile int *abort,
                                                float4 *stash) {
  constexpr int kMode = MODE & ~TC_FAST_MATH;
  constexpr bool kFast = (MODE & TC_FAST_MATH) != 0;
  constexpr bool kSwiglu = (kMode == TC_SWIGLU_BF16 || kMode == TC_SWIGLU_F32);
  constexpr int kChunks = kSwiglu ? 8 : 16;
  constexpr size_t kBlock = 64 * 128;  // float4s per partial block
  const int s = w.nparts;
  const int r = q * 32 + lane;
  float4 *const tail = reinterpret_cast<float4 *>(p.tail_ws);
  const size_t tile_base = (size_t)tl * s * 2;
  float4 *mine = tail + ((tile_base + w.part * 2 + rank) * kBlock);
#pragma unroll 1
  for (int c = 0; c < kChunks; ++c) {
    if (c % s == w.part) continue;
    uint32_t a[16];
    tmem_ld_32x32b_x16(t_row + 16 * c, a);
    if (kSwiglu) {
      uint32_t b[16];
      tmem_ld_32x32b_x16(t_row + 128 + 16 * c, b);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 4; ++i)
        mine[(size_t)(32 + 4 * c + i) * 128 + r] = make_float4(__uint_as_float(b[4 * i]), __uint_as_float(b[4 * i + 1]),
                                                               __uint_as_float(b[4 * i + 2]),
                                                               __uint_as_float(b[4 * i + 3]));
    } else {
      tmem_ld_wait();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      mine[(size_t)(4 * c + i) * 128 + r] = make_float4(__uint_as_float(a[4 * i]), __uint_as_float(a[4 * i + 1]),
                                                        __uint_as_float(a[4 * i + 2]), __uint_as_float(a[4 * i + 3]));
  }
  __threadfence();
  __syncwarp();
  int *cnt = p.tail_cnt + ((tl * 2 + static_cast<int>(rank)) * 4 + q) * 2;
  int ok = 1;
  if (lane == 0) {
    atomicAdd(cnt, 1);
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1; ld_acquire_gpu(cnt) < s; ++i) {
      if ((i & 63u) == 0) {
        if (*abort != 0) {
          ok = 0;
          break;
        }
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          *abort = LLK_ERR_TIMEOUT;
          ok = 0;
          break;
        }
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok) return false;
  __threadfence();
  // Gather the other parts' sums of this thread's row for every owned chunk
  // into shared memory at once (cp.async: one round trip through L2 for all
  // of them instead of one per part), then add in part order.  The stash is
  // the pipeline ring, idle once this pair's last item -- the tail part --
  // has its accumulator complete: entry k of thread r at float4 k * 128 + r
  // (consecutive lanes, consecutive 16 bytes).  At most 96 entries per
  // thread (7 other parts x 2 owned chunks x 8 float4): 192 KB, the ring.
  constexpr int kPer = kSwiglu ? 8 : 4;  // float4s of one row per (chunk, part)
  int k = 0;
#pragma unroll 1
  for (int c = w.part; c < kChunks; c += s) {
    for (int part = 0; part < s; ++part) {
      if (part == w.part) continue;
      const float4 *pb = tail + ((tile_base + part * 2 + rank) * kBlock) + r;
#pragma unroll
      for (int i = 0; i < 4; ++i) cp_async_16(stash + (size_t)(k + i) * 128 + r, pb + (size_t)(4 * c + i) * 128);
      if (kSwiglu) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          cp_async_16(stash + (size_t)(k + 4 + i) * 128 + r, pb + (size_t)(32 + 4 * c + i) * 128);
      }
      k += kPer;
    }
  }
  cp_async_commit_wait_all();
  const int row = m0 + r;
  k = 0;
#pragma unroll 1
  for (int c = w.part; c < kChunks; c += s) {
    uint32_t a[16], b[16];
    tmem_ld_32x32b_x16(t_row + 16 * c, a);
    if (kSwiglu) tmem_ld_32x32b_x16(t_row + 128 + 16 * c, b);
    tmem_ld_wait();
    float ga[16], ua[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) ga[j] = ua[j] = 0.f;
    for (int part = 0; part < s; ++part) {
      if (part == w.part) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          ga[j] += __uint_as_float(a[j]);
          if (kSwiglu) ua[j] += __uint_as_float(b[j]);
        }
        continue;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 v = stash[(size_t)(k + i) * 128 + r];
        ga[4 * i] += v.x;
        ga[4 * i + 1] += v.y;
        ga[4 * i + 2] += v.z;
        ga[4 * i + 3] += v.w;
        if (kSwiglu) {
          const float4 u = stash[(size_t)(k + 4 + i) * 128 + r];
          ua[4 * i] += u.x;
          ua[4 * i + 1] += u.y;
          ua[4 * i + 2] += u.z;
          ua[4 * i + 3] += u.w;
        }
      }
      k += kPer;
    }
    const int col = n0 + 16 * c;
    if (row >= p.M || col >= p.N) continue;
    const int64_t off = (int64_t)row * p.ldy + col;
    const bool vec = p.vec_ok && col + 16 <= p.N;
    if (kSwiglu) {
      float y[16];
      silu_mul_block<kFast, 16>(ga, ua, y);
      for (int t = -1; t < p.n_peers; ++t) {
        void *base = t < 0 ? p.y : p.y_peers[t];
        if (kMode == TC_SWIGLU_BF16) {
          uint16_t *dst = reinterpret_cast<uint16_t *>(base) + off;
          if (vec) {
            uint4 *d4 = reinterpret_cast<uint4 *>(dst);
            d4[0] = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                               pack_bf16x2(y[6], y[7]));
            d4[1] = make_uint4(pack_bf16x2(y[8], y[9]), pack_bf16x2(y[10], y[11]), pack_bf16x2(y[12], y[13]),
                               pack_bf16x2(y[14], y[15]));
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (col + j < p.N) dst[j] = static_cast<uint16_t>(pack_bf16x2(y[j], 0.f));
          }
        } else {
          float *dst = reinterpret_cast<float *>(base) + off;
          if (vec) {
            float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
            for (int v = 0; v < 4; ++v) d4[v] = make_float4(y[4 * v], y[4 * v + 1], y[4 * v + 2], y[4 * v + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (col + j < p.N) dst[j] = y[j];
          }
        }
      }
    } else {
      float *dst = reinterpret_cast<float *>(p.y) + off;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (col + j < p.N) {
          float o = ga[j];
          if (kMode == TC_MATMUL_F32_ACC) o += dst[j];
          dst[j] = o;
          for (int t = 0; t < p.n_peers; ++t) reinterpret_cast<float *>(p.y_peers[t])[off + j] = o;
        }
      }
    }
  }
  __syncwarp();
  if (lane == 0 && atomicAdd(cnt + 1, 1) == s - 1) {
    atomicExch(cnt, 0);
    atomicExch(cnt + 1, 0);
  }
  return true;
}

// Row block and column tile of a tile index: bands of p.group_m row blocks,
// row block fastest inside a band (the last band may be narrower).
__host__ __device__ __forceinline__ void tile_coords(const TcParams &p, int tile, int &mt, int &nt) {
  const int per_band = p.group_m * p.n_tiles;
  const int band = tile / per_band;
  const int r = tile - band * per_band;
  const int rows = p.group_m < p.m_tiles - band * p.group_m ? p.group_m : p.m_tiles - band * p.group_m;
  mt = band * p.group_m + r % rows;
  nt = r / rows;
}

// Static schedule: pair `pair` takes items pair, pair + pairs, ...
template <int TILE_N>
__device__ __forceinline__ bool get_work(const TcParams &p, int pair, int n_pairs, int idx, Work &w) {
  return item_to_work<TILE_N>(p, n_pairs, pair + idx * n_pairs, w);
}

#ifndef LLK_TC2_BAND_BLOCKS
#define LLK_TC2_BAND_BLOCKS 8
#endif
#ifndef LLK_TC2_HINTS
#define LLK_TC2_HINTS 0
#endif
// Row blocks per band of the tile order.  A wave of P pairs then covers
// g row blocks x P/g column tiles; its L2 footprint, g X blocks plus P/g
// weight tiles (both 256 x K bf16), is smallest at g = sqrt(P) ~ 8.6 for
// 74 pairs, whatever K is.
constexpr int kBandBlocks = LLK_TC2_BAND_BLOCKS;
constexpr int kRing = 8;  // work items in flight between the leader's draw and the last role reading it

struct __align__(8) PairTail {
  uint64_t sched_full[kRing];   // both CTAs: an item index was posted in sched_ring
  uint64_t sched_empty[kRing];  // leader: all 10 readers of the pair took the slot
  int sched_ring[kRing];
  uint64_t full[kStages];   // leader's copy is the one used
  uint64_t empty[kStages];  // both CTAs
  uint64_t tmem_full[2];    // both CTAs
  uint64_t tmem_empty[2];   // leader's copy is the one used (256 arrivals)
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

enum Role { ROLE_PRODUCER = 0, ROLE_MMA = 1, ROLE_EPILOGUE = 2 };

// The i-th work item of this pair for one role.  Static schedule: computed.
// Dynamic schedule: the leader's producer draws the next item index from the
// launch-wide counter and posts it in ring slot i % kRing of both CTAs; every
// other role of the pair (peer producer, leader MMA thread, the 8 epilogue
// warps) waits for the slot, copies the index and releases the slot on the
// leader.  All waits bounded; `ok` turns false when one gives up.
template <int TILE_N>
__device__ __forceinline__ bool next_work(const TcParams &p, PairTail *st, uint32_t rank, int role, int pair,
                                          int n_pairs, int i, Work &w, volatile int *abort, bool &ok,
                                          int &posted, bool &drew_end) {
  if (!p.dynamic) return get_work<TILE_N>(p, pair, n_pairs, i, w);
  const int slot = i % kRing;
  const uint32_t ph = static_cast<uint32_t>(i / kRing) & 1u;
  int idx;
  if (role == ROLE_PRODUCER && rank == 0) {
    // Keep one item posted ahead of the one starting, so the counter's round
    // trip and the hand-off to the peer overlap the current item's loads.
    while (!drew_end && posted <= i + 1) {
      const int ps = posted % kRing;
      const uint32_t pph = static_cast<uint32_t>(posted / kRing) & 1u;
      if (!mbar_wait_bounded(&st->sched_empty[ps], pph ^ 1u, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) {
        ok = false;
        return false;
      }
      const int d = atomicAdd(p.sched_counter, 1);
      st->sched_ring[ps] = d;
      st_shared_cluster_u32(map_shared_rank(smem_u32(&st->sched_ring[ps]), 1), static_cast<uint32_t>(d));
      mbar_arrive(&st->sched_full[ps]);
      mbar_arrive_cluster(map_shared_rank(smem_u32(&st->sched_full[ps]), 1));
      ++posted;
      if (d >= p.n_items) {
        drew_end = true;
        // Every pair draws exactly one index past the end; the last of those
        // draws is the launch's last use of the counter: leave it at zero.
        if (d == p.n_items + n_pairs - 1) atomicExch(p.sched_counter, 0);
      }
    }
    if (i >= posted) return false;
    idx = st->sched_ring[slot];
  } else {
    if (!mbar_wait_cluster_bounded(&st->sched_full[slot], ph, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) {
      ok = false;
      return false;
    }
    idx = *reinterpret_cast<volatile int *>(&st->sched_ring[slot]);
    const uint32_t leader_empty = map_shared_rank(smem_u32(&st->sched_empty[slot]), 0);
    if (role == ROLE_EPILOGUE) {
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive_cluster(leader_empty);
    } else {
      mbar_arrive_cluster(leader_empty);
    }
  }
  if (idx >= p.n_items) return false;
  return item_to_work<TILE_N>(p, n_pairs, idx, w);
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    tc2_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b0,
               const __grid_constant__ CUtensorMap tm_b1, const TcParams p,
               const __grid_constant__ YStoreMaps ym) {
  constexpr int kMode = MODE & ~TC_FAST_MATH;
  constexpr bool kFast = (MODE & TC_FAST_MATH) != 0;
  constexpr bool kSwiglu = (kMode == TC_SWIGLU_BF16 || kMode == TC_SWIGLU_F32);
  constexpr int kTileN = kSwiglu ? 128 : 256;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *staging = smem + kStages * kStageBytes;
  PairTail *st = reinterpret_cast<PairTail *>(staging + kStagingBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader, 1 = peer
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&st->full[s], 1);
      mbar_init(&st->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&st->tmem_full[a], 1);
      mbar_init(&st->tmem_empty[a], 256);
    }
    mbar_init(&st->mma_done, 1);
    for (int r = 0; r < kRing; ++r) {
      mbar_init(&st->sched_full[r], 1);
      mbar_init(&st->sched_empty[r], 10);  // peer producer + leader MMA + 8 epilogue warps
    }
    st->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b0);
    if (kSwiglu) tma_prefetch_desc(&tm_b1);
  }
  if (warp == 1) {
    tmem_alloc_pair(&st->tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer may only signal the leader's barriers once they exist
  tc_fence_after();
  pdl_launch_dependents();
  pdl_wait();  // the previous kernel's writes (X, W, the workspace) are visible from here on
  const uint32_t tmem_base = st->tmem_base;
  volatile int *abort = &st->abort;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t leader_full = map_shared_rank(smem_u32(&st->full[0]), 0);
#if LLK_TC2_HINTS
      const uint64_t pol_x = l2_policy_evict_last();
      const uint64_t pol_w = l2_policy_evict_first();
#endif
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      Work w;
      int posted = 0;
      bool drew_end = false;
      for (int idx = 0; ok && next_work<kTileN>(p, st, rank, ROLE_PRODUCER, pair, n_pairs, idx, w, abort, ok, posted, drew_end);
           ++idx) {
        int mt, nt;
        tile_coords(p, w.tile, mt, nt);
        const int m0 = mt * (2 * kRows) + static_cast<int>(rank) * kRows;
        const int n0 = nt * kTileN + w.c0;
        // B columns this CTA supplies: SwiGLU w.wn of its matrix (leader Wg,
        // peer Wu); matmul w.wn/2, the peer's after the leader's.
        const int cta_cols = kSwiglu ? w.wn : w.wn / 2;
        const int nb = kSwiglu ? n0 : n0 + static_cast<int>(rank) * cta_cols;
        const int slabs = cta_cols > 64 ? 2 : 1;
        const uint32_t stage_tx = 2u * (kABytes + slabs * kSlabBytes);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait_bounded(&st->empty[stage], phase ^ 1u, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + stage * kStageBytes;
          uint8_t *sb = sa + kABytes;
          const uint32_t bar = leader_full + stage * 8u;
          if (rank == 0) mbar_arrive_expect_tx(&st->full[stage], stage_tx);
          const int k0 = kb * kBK;
          const CUtensorMap *wmap = (kSwiglu && rank == 1) ? &tm_b1 : &tm_b0;
          // A 32-column part still loads a whole 64-column box (the MMA reads
          // the first 32); its start stays 64-byte aligned.
#if LLK_TC2_HINTS
          if (LLK_TC2_HINTS & 1) tma_load_2d_pair_hint(sa, &tm_a, bar, k0, m0, pol_x);
          else tma_load_2d_pair(sa, &tm_a, bar, k0, m0);
          if (LLK_TC2_HINTS & 2) {
            tma_load_weight_slab_pair_hint(sb, wmap, bar, nb, k0, p.slab_major, pol_w);
            if (slabs == 2) tma_load_weight_slab_pair_hint(sb + kSlabBytes, wmap, bar, nb + 64, k0, p.slab_major, pol_w);
          } else {
            tma_load_weight_slab_pair(sb, wmap, bar, nb, k0, p.slab_major);
            if (slabs == 2) tma_load_weight_slab_pair(sb + kSlabBytes, wmap, bar, nb + 64, k0, p.slab_major);
          }
#else
          tma_load_2d_pair(sa, &tm_a, bar, k0, m0);
          tma_load_weight_slab_pair(sb, wmap, bar, nb, k0, p.slab_major);
          if (slabs == 2) tma_load_weight_slab_pair(sb + kSlabBytes, wmap, bar, nb + 64, k0, p.slab_major);
#endif
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && rank == 0) {
        // Loads in flight land on the leader's barriers: wait (bounded) for them.
        const uint32_t n = issued < kStages ? issued : kStages;
        for (uint32_t i = 0; i < n; ++i) {
          const uint32_t idx = issued - 1 - i;
          int dummy = 0;
          mbar_wait_bounded(&st->full[idx % kStages], (idx / kStages) & 1u, &dummy, 1, 100000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t smem_base = smem_u32(smem);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      Work w;
      int posted = 0;
      bool drew_end = false;
      for (int local = 0; ok && next_work<kTileN>(p, st, rank, ROLE_MMA, pair, n_pairs, local, w, abort, ok, posted, drew_end);
           ++local) {
        // MMA N = the B columns of both CTAs: SwiGLU 2 x wn (gate | up), matmul wn.
        const uint32_t idesc = make_idesc_bf16_f32(2 * kRows, kSwiglu ? 2 * w.wn : w.wn, false, true);
        const uint32_t acc = local & 1;
        if (!mbar_wait_bounded(&st->tmem_empty[acc], ((local >> 1) & 1) ^ 1u, abort, LLK_ERR_TIMEOUT,
                               kWaitLimitNs)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kMmaN;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait_bounded(&st->full[stage], phase, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_base + stage * kStageBytes;
          const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t a_desc = make_smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t b_desc = make_smem_desc_sw128(b_addr + kk * 2048, kSlabBytes, 1024);
            tc_mma_bf16_pair(d_tmem, a_desc, b_desc, idesc, (kb > w.kb0 || kk > 0) ? 1u : 0u);
          }
          tc_commit_pair_mc(&st->empty[stage], 0x3);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair_mc(&st->tmem_full[acc], 0x3);
      }
      tc_commit_pair_mc(&st->mma_done, 0x1);
      int dummy = 0;
      mbar_wait_bounded(&st->mma_done, 0, &dummy, 1, 100000000ull);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    const uint32_t leader_tmem_empty = map_shared_rank(smem_u32(&st->tmem_empty[0]), 0);
    uint32_t y_chunks = 0;  // chunks this warp staged for TMA stores
    Work w;
    bool ok = true;
    int posted = 0;
    bool drew_end = false;
    for (int local = 0; ok && next_work<kTileN>(p, st, rank, ROLE_EPILOGUE, pair, n_pairs, local, w, abort, ok, posted, drew_end);
         ++local) {
      const uint32_t acc = local & 1;
      if (!mbar_wait_bounded(&st->tmem_full[acc], (local >> 1) & 1, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) break;
      tc_fence_after();
      int mt, nt;
      tile_coords(p, w.tile, mt, nt);
      const int m0 = mt * (2 * kRows) + static_cast<int>(rank) * kRows;
      const int n0 = nt * kTileN + w.c0;
      const int row = m0 + row_in_tile;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kMmaN;
      if (w.nparts > 1) {
        if (!ksplit_epilogue<MODE>(p, w, w.tile - p.dp_waves * n_pairs, rank, q, lane, t_row, m0, n0, abort,
                                   reinterpret_cast<float4 *>(smem))) {
          ok = false;
          break;
        }
      } else if (kSwiglu && ym.n > 0) {
        // Staged TMA stores: lane = row; the chunk goes to shared memory in
        // the map's swizzled layout (64-byte rows for bf16, 128-byte for
        // f32; the XOR keeps each 8-lane phase of the 16-byte stores on
        // distinct banks), then one lane stores it through every map.
        constexpr bool kBf16 = (kMode == TC_SWIGLU_BF16);
        constexpr uint32_t kBuf = kBf16 ? 2048 : 4096;
        constexpr int kNBuf = kStagingPerWarp / kBuf;
        const uint32_t wstage = smem_u32(staging) + q * kStagingPerWarp;
        const int r0 = m0 + q * 32;
#pragma unroll 1
        for (int c = 0; c < w.wn; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(t_row + c, g);
          tmem_ld_32x32b_x32(t_row + w.wn + c, u);
          tmem_ld_wait();
          const int col = n0 + c;
          if (r0 >= p.M || col >= p.N) continue;  // warp-uniform
          float y[32];
          silu_mul_block<kFast, 32>(g, u, y);
          const uint32_t buf = wstage + static_cast<uint32_t>(y_chunks % kNBuf) * kBuf;
          // lanes that store (one per map) wait until their store of this
          // buffer's previous chunk has read it
          if (lane < ym.n) bulk_wait_group_read<kNBuf - 1>();
          __syncwarp();
          if (kBf16) {
            const uint32_t rowa = buf + lane * 64;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t phys = static_cast<uint32_t>(j) ^ ((lane >> 1) & 3u);
              st_shared_v4(rowa + phys * 16, pack_bf16x2(y[8 * j], y[8 * j + 1]), pack_bf16x2(y[8 * j + 2], y[8 * j + 3]),
                           pack_bf16x2(y[8 * j + 4], y[8 * j + 5]), pack_bf16x2(y[8 * j + 6], y[8 * j + 7]));
            }
          } else {
            const uint32_t rowa = buf + lane * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t phys = static_cast<uint32_t>(j) ^ (lane & 7u);
              st_shared_v4(rowa + phys * 16, __float_as_uint(y[4 * j]), __float_as_uint(y[4 * j + 1]),
                           __float_as_uint(y[4 * j + 2]), __float_as_uint(y[4 * j + 3]));
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          // one lane per map (this GPU's Y, then each peer's): the stores to
          // the GPUs go out side by side instead of one after another
          if (lane < ym.n) {
            tma_store_2d(&ym.m[lane], buf, ym.col0 + col, r0);
            bulk_commit_group();
          }
          ++y_chunks;
        }
      } else if (kSwiglu) {
#pragma unroll 1
        for (int c = 0; c < w.wn; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(t_row + c, g);
          tmem_ld_32x32b_x32(t_row + w.wn + c, u);
          tmem_ld_wait();
          const int col = n0 + c;
          if (row < p.M && col < p.N) {
            float y[32];
            silu_mul_block<kFast, 32>(g, u, y);
            const int64_t off = (int64_t)row * p.ldy + col;
            const bool vec = p.vec_ok && col + 32 <= p.N;
            if (kMode == TC_SWIGLU_BF16) {
              uint32_t pk[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(y[2 * j], y[2 * j + 1]);
              // t = -1: this GPU's Y; t >= 0: the peers' (fused all-gather)
              for (int t = -1; t < p.n_peers; ++t) {
                uint16_t *dst = reinterpret_cast<uint16_t *>(t < 0 ? p.y : p.y_peers[t]) + off;
                if (vec) {
                  uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll
                  for (int v = 0; v < 4; ++v) d4[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    if (col + j < p.N) dst[j] = static_cast<uint16_t>(pk[j >> 1] >> ((j & 1) * 16));
                }
              }
            } else {
              for (int t = -1; t < p.n_peers; ++t) {
                float *dst = reinterpret_cast<float *>(t < 0 ? p.y : p.y_peers[t]) + off;
                if (vec) {
                  float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
                  for (int v = 0; v < 8; ++v) d4[v] = make_float4(y[4 * v], y[4 * v + 1], y[4 * v + 2], y[4 * v + 3]);
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    if (col + j < p.N) dst[j] = y[j];
                }
              }
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < w.wn; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c, r);
          tmem_ld_wait();
          const int col = n0 + c;
          if (row < p.M && col < p.N) {
            const int64_t off = (int64_t)row * p.ldy + col;
            float *dst = reinterpret_cast<float *>(p.y) + off;
            const bool vec = p.vec_ok && col + 32 <= p.N;
            if (vec) {
              float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                float4 o = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                       __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                if (kMode == TC_MATMUL_F32_ACC) {
                  const float4 c4 = d4[v];
                  o.x += c4.x;
                  o.y += c4.y;
                  o.z += c4.z;
                  o.w += c4.w;
                }
                d4[v] = o;
                for (int t = 0; t < p.n_peers; ++t) reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.y_peers[t]) + off)[v] = o;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (col + j < p.N) {
                  float o = __uint_as_float(r[j]);
                  if (kMode == TC_MATMUL_F32_ACC) o += dst[j];
                  dst[j] = o;
                  for (int t = 0; t < p.n_peers; ++t) reinterpret_cast<float *>(p.y_peers[t])[off + j] = o;
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(leader_tmem_empty + acc * 8u);
    }
    if (lane < ym.n) bulk_wait_group_all();  // staging is read and the stores done before exit
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its partner may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && st->abort != 0 && p.status != nullptr) atomicExch(p.status, st->abort);
}

// Per device: the smem attribute was set and how many pairs can be resident
// (a cluster occupancy query costs far more than a launch, so it runs once).
template <int MODE>
int resident_pairs() {
  constexpr int kDevs = 64;
  static std::atomic<int> cache[kDevs];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDevs) return -1;
  const int c = cache[dev].load(std::memory_order_relaxed);
  if (c > 0) return c;
  auto kern = tc2_kernel<MODE>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, tc2_smem_bytes()) != cudaSuccess)
    return -1;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = tc2_smem_bytes();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters < 1) {
    cudaGetLastError();
    clusters = 1;
  }
  cache[dev].store(clusters, std::memory_order_relaxed);
  return clusters;
}

// Partial-sum bytes of the K-split tail: one 128-row x 256-column f32 block
// per (leftover tile, part, CTA of the pair).
constexpr size_t kTailBlockBytes = 128 * 256 * sizeof(float);
// Tail counters available in the workspace's counter region (two per
// leftover tile, CTA and epilogue warp).
constexpr int kMaxTailTiles = static_cast<int>((kWsTc2CounterBytes - kWsTc2TailCounters) / (2 * 4 * 2 * sizeof(int)));

// The pair kernel's work split for `pairs` resident CTA pairs (host): fills
// p's tile order, whole-tile waves, tail split / K split, item count and
// dynamic flag; returns the number of pairs to launch.  Needs p.m_tiles,
// n_tiles, num_tiles and k_blocks.  The K split needs the static schedule
// and room for its partial sums in the workspace (workspace_bytes, 0 = no
// workspace); the caller points p.tail_ws / tail_cnt / sched_counter at it.
int plan_pair_schedule(TcParams &p, int pairs, int tail_split, bool dynamic, size_t workspace_bytes) {
  // Whole-tile waves, then the leftover tiles cut into g column parts.  A
  // part of width 256/g does not take 1/g of a tile: its k-blocks keep a
  // cost that does not shrink with the MMA's N (it still loads the tile's
  // whole X block; measured on B200: a quarter part takes ~0.63 of a whole
  // tile), so a part is charged (1 + 1/g) / 2 tile-times.  The last wave
  // then takes ceil(left * g / pairs) * (1 + 1/g) / 2; pick the g that
  // makes it shortest (ties: the wider tiles).
  //
  // Or, with the static schedule and room in the workspace, the leftover
  // tiles are cut along K into s = pairs / left parts (at most 8), one per
  // pair: a part costs 1/s of a tile plus its share of the partial-sum
  // exchange, charged 0.12 of a tile (each CTA writes and reads about
  // (s-1)/s x 128 KB through L2).
  p.group_m = kBandBlocks < p.m_tiles ? kBandBlocks : p.m_tiles;
  p.dp_waves = p.num_tiles / pairs;
  const int left = p.num_tiles - p.dp_waves * pairs;
  auto ksplit_fits = [&](int ks) {
    return ks >= 2 && ks <= 8 && ks <= p.k_blocks && left > 0 && left * ks <= pairs && left <= kMaxTailTiles &&
           !dynamic && workspace_bytes >= kWsPartials + static_cast<size_t>(left) * ks * 2 * kTailBlockBytes;
  };
  int g = 1, ks = 0;
  if (tail_split < 0 && ksplit_fits(-tail_split)) {
    ks = -tail_split;
  } else if (tail_split == 1 || tail_split == 2 || tail_split == 4) {
    g = tail_split;
  } else if (left > 0) {
    double best = 1e30;
    for (int cand = 1; cand <= 4; cand *= 2) {
      const double t = static_cast<double>((left * cand + pairs - 1) / pairs) * (1.0 + 1.0 / cand) / 2.0;
      if (t < best - 1e-9) {
        best = t;
        g = cand;
      }
    }
    int cand = pairs / left;
    if (cand > 8) cand = 8;
    if (cand > p.k_blocks) cand = p.k_blocks;
    if (ksplit_fits(cand) && 1.0 / cand + 0.12 < best - 1e-9) ks = cand;
  }
  p.ksplit = ks;
  p.tail_split = ks ? 1 : g;
  const int parts = ks ? ks : g;
  // No pair without work: at most all tiles' parts.
  if (p.dp_waves == 0 && pairs > left * parts) pairs = left * parts;
  p.n_items = p.dp_waves * pairs + left * parts;
  p.dynamic = dynamic ? 1 : 0;
  return pairs;
}

template <int MODE>
cudaError_t launch_pair_mode(const CUtensorMap &a, const CUtensorMap &b0, const CUtensorMap &b1, TcParams p,
                             int max_pairs, int tail_split, int *sched_counter, void *workspace,
                             size_t workspace_bytes, cudaStream_t stream, const YStoreMaps &ym) {
  auto kern = tc2_kernel<MODE>;
  const int clusters = resident_pairs<MODE>();
  if (clusters < 1) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // CTAs may start and set up while the previous kernel finishes; the kernel
  // waits for it before its first memory access (pdl_wait).
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = tc2_smem_bytes();
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaSuccess;
  int pairs = clusters;
  if (max_pairs >= 1 && pairs > max_pairs) pairs = max_pairs;
  pairs = plan_pair_schedule(p, pairs, tail_split, sched_counter != nullptr, workspace ? workspace_bytes : 0);
  if (p.ksplit) {
    p.tail_ws = reinterpret_cast<float *>(static_cast<char *>(workspace) + kWsPartials);
    p.tail_cnt = reinterpret_cast<int *>(static_cast<char *>(workspace) + kWsTc2TailCounters);
  }
  p.sched_counter = sched_counter;
  cfg.gridDim = dim3(2 * pairs);
  e = cudaLaunchKernelEx(&cfg, kern, a, b0, b1, p, ym);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

int tc2_smem_bytes() { return kStages * kStageBytes + kStagingBytes + static_cast<int>(sizeof(PairTail)) + 1024; }
static_assert(kStages * kStageBytes + kStagingBytes + sizeof(PairTail) + 1024 <= 227 * 1024,
              "CTA-pair kernel shared memory over the 227 KB opt-in limit");

size_t tc2_tail_workspace_bytes(int sm_count) {
  return kWsPartials + static_cast<size_t>(sm_count / 2) * 2 * kTailBlockBytes;
}

int tc2_schedule_items(int swiglu, int64_t M, int64_t N, int64_t K, int pairs, int tail_split, int dynamic,
                       size_t workspace_bytes, int *items, int max_items, int *n_items, int *n_pairs, int *ksplit,
                       int *tail_split_out) {
  if (M < 1 || N < 1 || K < 1 || pairs < 1 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return -1;
  const int tile_n = swiglu ? 128 : 256;
  TcParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.m_tiles = static_cast<int>((M + 255) / 256);
  p.n_tiles = static_cast<int>((N + tile_n - 1) / tile_n);
  p.num_tiles = p.m_tiles * p.n_tiles;
  p.k_blocks = static_cast<int>((K + 63) / 64);
  const int used = plan_pair_schedule(p, pairs, tail_split, dynamic != 0, workspace_bytes);
  *n_items = p.n_items;
  *n_pairs = used;
  *ksplit = p.ksplit;
  *tail_split_out = p.tail_split;
  for (int i = 0; i < p.n_items && i < max_items; ++i) {
    Work w;
    const bool ok = swiglu ? item_to_work<128>(p, used, i, w) : item_to_work<256>(p, used, i, w);
    int mt = -1, nt = -1;
    if (ok) tile_coords(p, w.tile, mt, nt);
    int *o = items + 9 * static_cast<size_t>(i);
    // static schedule: pair q takes items q, q + pairs, ...; dynamic: drawn
    o[0] = dynamic ? -1 : i % used;
    o[1] = ok ? mt : -1;
    o[2] = nt;
    o[3] = w.c0;
    o[4] = w.wn;
    o[5] = w.kb0;
    o[6] = w.kb1;
    o[7] = w.part;
    o[8] = w.nparts;
  }
  return 0;
}

cudaError_t tc2_launch(int mode, const CUtensorMap &a, const CUtensorMap &b0, const CUtensorMap &b1, TcParams p,
                       int max_pairs, int tail_split, int *sched_counter, void *workspace, size_t workspace_bytes,
                       cudaStream_t stream, const YStoreMaps *ym) {
  static const YStoreMaps kNoMaps = {};
  const YStoreMaps &m = ym ? *ym : kNoMaps;
  switch (mode) {
    case TC_SWIGLU_BF16:
      return launch_pair_mode<TC_SWIGLU_BF16>(a, b0, b1, p, max_pairs, tail_split, sched_counter, workspace,
                                              workspace_bytes, stream, m);
    case TC_SWIGLU_F32:
      return launch_pair_mode<TC_SWIGLU_F32>(a, b0, b1, p, max_pairs, tail_split, sched_counter, workspace,
                                             workspace_bytes, stream, m);
    case TC_SWIGLU_BF16 | TC_FAST_MATH:
      return launch_pair_mode<TC_SWIGLU_BF16 | TC_FAST_MATH>(a, b0, b1, p, max_pairs, tail_split, sched_counter,
                                                             workspace, workspace_bytes, stream, m);
    case TC_SWIGLU_F32 | TC_FAST_MATH:
      return launch_pair_mode<TC_SWIGLU_F32 | TC_FAST_MATH>(a, b0, b1, p, max_pairs, tail_split, sched_counter,
                                                            workspace, workspace_bytes, stream, m);
    case TC_MATMUL_F32:
      return launch_pair_mode<TC_MATMUL_F32>(a, b0, b1, p, max_pairs, tail_split, sched_counter, workspace,
                                             workspace_bytes, stream, kNoMaps);
    case TC_MATMUL_F32_ACC:
      return launch_pair_mode<TC_MATMUL_F32_ACC>(a, b0, b1, p, max_pairs, tail_split, sched_counter, workspace,
                                                 workspace_bytes, stream, kNoMaps);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace llk_b200
