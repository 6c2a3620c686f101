// swiglu_decode.cu -- small-M (decode) fused SwiGLU on sm_100a.
//
// For M <= 128 tokens the op is bound by streaming Wg and Wu (4*K*N bytes)
// from HBM.  The kernel computes the transposed product
//     Y^T[n, m] = SiLU(sum_k Wg[k,n] X[m,k]) * (sum_k Wu[k,n] X[m,k])
// so the weights are the 128-row A operand of tcgen05.mma (MN-major: the
// row-major [K, N] weights have n contiguous) and the padded token block
// X[Mp, K] (Mp = 16/32/64/128, K-major) is the narrow B operand.  Gate and up
// accumulate in two TMEM blocks of Mp columns.
//
// Work split ("stream-K"): the (128-column tile, 64-deep k-block) pairs are
// laid out tile-major and cut into gridDim.x equal contiguous ranges, one
// per CTA, so every SM streams the same number of weight bytes whatever N/128
// is.  A CTA's range covers one or more tile segments.  A tile owned by a
// single CTA is finished straight from TMEM; a tile shared by several CTAs
// has each contributor write its f32 partial sums (token rows < M only) to a
// slot of its own, and the last contributor to arrive (per-tile counter)
// adds the contributors' slots in CTA order -- deterministic -- applies the
// SiLU * up epilogue, stores Y and resets the counter to zero for the next
// launch.  Only a CTA's first and last tile can be shared, so the workspace
// holds two slots per CTA and a tile may have any number of contributors:
// a narrow column shard (a few tiles) still spreads over every SM.
//
// Roles: warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 2-5
// epilogue (one TMEM lane = one output column each).  All waits bounded.
// No TMA multicast.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <map>
#include <mutex>
#include <tuple>

#include "decode_kernels.h"
#include "sm100_ptx.cuh"
#include "workspace.h"

namespace llk_b200 {

namespace {

constexpr int kThreads = 192;
constexpr int kTileN = 128;        // weight columns per tile (MMA M)
constexpr int kBK = 64;            // k per stage
constexpr uint32_t kSlab = 64 * kBK * 2;  // 64 n x 64 k bf16 = 8 KB
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr int kSmemBudget = 220 * 1024;
// Workspace layout (workspace.h), the same for every shape so a workspace
// reused across shapes never has a counter landing on another call's partial
// sums: per-tile arrival counters at kWsDecodeCounters (65536 tiles, N <= 8 M),
// partial sums, two slots per CTA, from kWsPartials.
constexpr size_t kCounterOffset = kWsDecodeCounters;
constexpr size_t kCounterRegion = kWsDecodeCounterBytes;
constexpr size_t kPartialsOffset = kWsPartials;

struct DecodeParams {
  int M, N, K;
  int Mp;            // padded token count = MMA N (16, 32, 64 or 128)
  int n_tiles;       // ceil(N / 128)
  int kb_per_tile;   // ceil(K / 64)
  long long total;   // n_tiles * kb_per_tile work units
  int stages;
  int y_f32;
  int slab_major;    // weight tensor maps describe slab-major packed weights
  void *y;
  long long ldy;
  float *partials;   // [gridDim.x][2 slots][2 (gate, up)][Mp][128] f32
  int *counters;     // [n_tiles]
  int *status;
  // Cluster mode (cluster_s >= 2): the grid is n_tiles x cluster_s CTAs in
  // clusters of cluster_s, cluster t splitting tile t's k-blocks evenly; the
  // partial sums meet in distributed shared memory instead of the workspace.
  int cluster_s;
};

struct __align__(8) DecodeTail {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  int is_last;
};

__device__ __forceinline__ long long range_begin(long long c, long long total, long long G) {
  return c * total / G;
}
// The CTA whose range contains unit u.
__device__ __forceinline__ long long cta_of(long long u, long long total, long long G) {
  return ((u + 1) * G - 1) / total;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void store_y(const DecodeParams &p, int m, int n, float v) {
  if (p.y_f32) {
    reinterpret_cast<float *>(p.y)[(long long)m * p.ldy + n] = v;
  } else {
    reinterpret_cast<uint16_t *>(p.y)[(long long)m * p.ldy + n] = static_cast<uint16_t>(pack_bf16x2(v, 0.f));
  }
}

// The last contributor's sum over a shared tile's partial-sum slots for
// column n (this thread's TMEM lane r): rows in groups of R, contributors
// c_first .. c_last in batches of B whose loads are issued together, added
// in CTA order.  Adding the zeros of a batch's unused entries leaves every
// sum unchanged, so the order and result are those of a plain loop.
template <bool kFast, int R, int B>
__device__ __forceinline__ void fixup_tile(const DecodeParams &p, long long t, long long c_first, long long c_last,
                                           long long G, int r, int n, size_t slot_floats) {
  for (int m0 = 0; m0 < p.M; m0 += R) {
    const int rows = p.M - m0 < R ? p.M - m0 : R;
    float gs[R], us[R];
#pragma unroll
    for (int j = 0; j < R; ++j) gs[j] = us[j] = 0.f;
    for (long long cb = c_first; cb <= c_last; cb += B) {
      float gv[B][R], uv[B][R];
#pragma unroll
      for (int i = 0; i < B; ++i) {
        const long long c = cb + i;
        const bool live = c <= c_last;
        // contributor c's slot for tile t (the same rule the writer used)
        const int which = live && range_begin(c, p.total, G) / p.kb_per_tile == t ? 0 : 1;
        const float *ps = p.partials + ((size_t)(live ? c : c_first) * 2 + which) * slot_floats + (size_t)m0 * kTileN + r;
#pragma unroll
        for (int j = 0; j < R; ++j) {
          gv[i][j] = live && j < rows ? __ldcg(ps + (size_t)j * kTileN) : 0.f;
          uv[i][j] = live && j < rows ? __ldcg(ps + (size_t)(p.Mp + j) * kTileN) : 0.f;
        }
      }
#pragma unroll
      for (int i = 0; i < B; ++i) {
#pragma unroll
        for (int j = 0; j < R; ++j) {
          gs[j] += gv[i][j];
          us[j] += uv[i][j];
        }
      }
    }
    if (n < p.N) {
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (j < rows) store_y(p, m0 + j, n, silu_mul_mode<kFast>(gs[j], us[j]));
    }
  }
}

#ifdef LLK_DECODE_TRACE
// Debug builds only: per-CTA %globaltimer stamps of the kernel's phases.
__device__ unsigned long long g_decode_trace[4096][8];
#define DECODE_TRACE(slot) g_decode_trace[blockIdx.x & 4095][slot] = global_timer_ns()
#else
#define DECODE_TRACE(slot) \
  do {                     \
  } while (0)
#endif

template <bool kFast>
__global__ void __launch_bounds__(kThreads, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tm_wg, const __grid_constant__ CUtensorMap tm_wu,
                  const __grid_constant__ CUtensorMap tm_x, const DecodeParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t x_bytes = static_cast<uint32_t>(p.Mp) * kBK * 2;
  const uint32_t stage_bytes = 4 * kSlab + ((x_bytes + 1023u) & ~1023u);
  DecodeTail *st = reinterpret_cast<DecodeTail *>(smem + p.stages * stage_bytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long G = gridDim.x;
  const long long w0 = range_begin(blockIdx.x, p.total, G);
  const long long w1 = range_begin(blockIdx.x + 1, p.total, G);
  const uint32_t acc_cols = 2u * p.Mp;  // gate block + up block
  uint32_t tmem_cols = 32;
  while (tmem_cols < 2 * acc_cols) tmem_cols <<= 1;
  if (threadIdx.x == 0) DECODE_TRACE(0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&st->full[s], 1);
      mbar_init(&st->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&st->tmem_full[a], 1);
      mbar_init(&st->tmem_empty[a], 128);
    }
    mbar_init(&st->mma_done, 1);
    st->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_wg);
    tma_prefetch_desc(&tm_wu);
    tma_prefetch_desc(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc(&st->tmem_base, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  pdl_wait();  // the previous kernel's writes (X, the workspace) are visible from here on
  if (threadIdx.x == 0) DECODE_TRACE(1);
  const uint32_t tmem_base = st->tmem_base;
  volatile int *abort = &st->abort;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      for (long long u = w0; u < w1; ++u) {
        const int t = static_cast<int>(u / p.kb_per_tile);
        const int kb = static_cast<int>(u % p.kb_per_tile);
        if (!mbar_wait_bounded(&st->empty[stage], phase ^ 1u, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) break;
        uint8_t *s = smem + stage * stage_bytes;
        mbar_arrive_expect_tx(&st->full[stage], 4 * kSlab + x_bytes);
        const int n0 = t * kTileN, k0 = kb * kBK;
        tma_load_weight_slab(s + 0 * kSlab, &tm_wg, &st->full[stage], n0, k0, p.slab_major);
        tma_load_weight_slab(s + 1 * kSlab, &tm_wg, &st->full[stage], n0 + 64, k0, p.slab_major);
        tma_load_weight_slab(s + 2 * kSlab, &tm_wu, &st->full[stage], n0, k0, p.slab_major);
        tma_load_weight_slab(s + 3 * kSlab, &tm_wu, &st->full[stage], n0 + 64, k0, p.slab_major);
        tma_load_2d(s + 4 * kSlab, &tm_x, &st->full[stage], k0, 0);
        ++issued;
        if (++stage == static_cast<uint32_t>(p.stages)) {
          stage = 0;
          phase ^= 1u;
        }
      }
      DECODE_TRACE(3);
      if (*abort != 0) {
        const uint32_t n = issued < static_cast<uint32_t>(p.stages) ? issued : p.stages;
        for (uint32_t i = 0; i < n; ++i) {
          const uint32_t idx = issued - 1 - i;
          int dummy = 0;
          mbar_wait_bounded(&st->full[idx % p.stages], (idx / p.stages) & 1u, &dummy, 1, 100000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // A = weights (M = 128, MN-major), B = X (N = Mp, K-major).
      const uint32_t idesc = make_idesc_bf16_f32(128, p.Mp, true, false);
      const uint32_t sbase = smem_u32(smem);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      int seg = 0;
      for (long long u = w0; u < w1 && ok; ++seg) {
        const long long t = u / p.kb_per_tile;
        const long long seg_end = (t + 1) * p.kb_per_tile < w1 ? (t + 1) * p.kb_per_tile : w1;
        const uint32_t acc = seg & 1;
        if (!mbar_wait_bounded(&st->tmem_empty[acc], ((seg >> 1) & 1) ^ 1u, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_gate = tmem_base + acc * acc_cols;
        const uint32_t d_up = d_gate + p.Mp;
        bool first = true;
        for (; u < seg_end; ++u) {
          if (!mbar_wait_bounded(&st->full[stage], phase, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) {
            ok = false;
            break;
          }
          if (u == w0) DECODE_TRACE(2);
          tc_fence_after();
          const uint32_t s = sbase + stage * stage_bytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // A (weights) MN-major: two 64-column slabs 8 KB apart, 16 k = 2 KB.
            const uint64_t ag = make_smem_desc_sw128(s + 0 * kSlab + kk * 2048, kSlab, 1024);
            const uint64_t au = make_smem_desc_sw128(s + 2 * kSlab + kk * 2048, kSlab, 1024);
            // B (tokens) K-major: 16 k = 32 bytes inside the swizzle atom.
            const uint64_t bx = make_smem_desc_sw128(s + 4 * kSlab + kk * 32, 16, 1024);
            const uint32_t accum = first && kk == 0 ? 0u : 1u;
            tc_mma_bf16(d_gate, ag, bx, idesc, accum);
            tc_mma_bf16(d_up, au, bx, idesc, accum);
          }
          first = false;
          tc_commit(&st->empty[stage]);
          if (++stage == static_cast<uint32_t>(p.stages)) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&st->tmem_full[acc]);
      }
      tc_commit(&st->mma_done);
      int dummy = 0;
      mbar_wait_bounded(&st->mma_done, 0, &dummy, 1, 100000000ull);
      DECODE_TRACE(4);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int r = q * 32 + lane;  // TMEM lane = column within the tile
    const int etid = (warp - 2) * 32 + lane;
    int seg = 0;
    for (long long u = w0; u < w1; ++seg) {
      const long long t = u / p.kb_per_tile;
      const long long t_begin = t * p.kb_per_tile, t_end = t_begin + p.kb_per_tile;
      u = t_end < w1 ? t_end : w1;
      const uint32_t acc = seg & 1;
      if (!mbar_wait_bounded(&st->tmem_full[acc], (seg >> 1) & 1, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) break;
      tc_fence_after();
      const long long c_first = cta_of(t_begin, p.total, G);
      const long long c_last = cta_of(t_end - 1, p.total, G);
      const int n_contrib = static_cast<int>(c_last - c_first + 1);
      const int n = static_cast<int>(t) * kTileN + r;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * acc_cols;
      const size_t slot_floats = (size_t)2 * p.Mp * kTileN;

      if (p.cluster_s > 1) {
        // Cluster mode: park this CTA's partial sums (rows < M) in its own
        // shared memory -- the pipeline stages, all consumed once the
        // accumulator is complete -- as [gate | up][Mp][128] f32; the
        // cluster reduces them after the role loops.
        float *part = reinterpret_cast<float *>(smem);
        for (int m0 = 0; m0 < p.M; m0 += 16) {
          uint32_t g[16], uu[16];
          tmem_ld_32x32b_x16(t_row + m0, g);
          tmem_ld_32x32b_x16(t_row + p.Mp + m0, uu);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (m0 + j < p.M) {
              part[(m0 + j) * kTileN + r] = __uint_as_float(g[j]);
              part[(p.Mp + m0 + j) * kTileN + r] = __uint_as_float(uu[j]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&st->tmem_empty[acc]);
        continue;
      }

      if (n_contrib == 1) {
        for (int m0 = 0; m0 < p.Mp; m0 += 16) {
          uint32_t g[16], uu[16];
          tmem_ld_32x32b_x16(t_row + m0, g);
          tmem_ld_32x32b_x16(t_row + p.Mp + m0, uu);
          tmem_ld_wait();
          if (n < p.N) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (m0 + j < p.M) store_y(p, m0 + j, n, silu_mul_mode<kFast>(__uint_as_float(g[j]), __uint_as_float(uu[j])));
          }
        }
        tc_fence_before();
        mbar_arrive(&st->tmem_empty[acc]);
        continue;
      }

      // Shared tile: park this CTA's partial sums in its slot -- slot 0 when
      // the tile is the one its range starts in, slot 1 for its last tile.
      float *mine = p.partials + ((size_t)blockIdx.x * 2 + (t == w0 / p.kb_per_tile ? 0 : 1)) * slot_floats;
      for (int m0 = 0; m0 < p.M; m0 += 16) {
        uint32_t g[16], uu[16];
        tmem_ld_32x32b_x16(t_row + m0, g);
        tmem_ld_32x32b_x16(t_row + p.Mp + m0, uu);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (m0 + j < p.M) {
            mine[(size_t)(m0 + j) * kTileN + r] = __uint_as_float(g[j]);
            mine[(size_t)(p.Mp + m0 + j) * kTileN + r] = __uint_as_float(uu[j]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&st->tmem_empty[acc]);
      __threadfence();
      epi_bar();
      if (etid == 0) {
        const int old = atomicAdd(&p.counters[t], 1);
        st->is_last = (old == n_contrib - 1) ? 1 : 0;
      }
      epi_bar();
      if (st->is_last) {
        __threadfence();
        // Sum the contributors' slots in CTA order (deterministic), with
        // 64 loads in flight: 4 token rows x 8 contributors at a time for
        // M <= 4, 16 rows x 2 contributors above.
        if (p.M <= 4)
          fixup_tile<kFast, 4, 8>(p, t, c_first, c_last, G, r, n, slot_floats);
        else
          fixup_tile<kFast, 16, 2>(p, t, c_first, c_last, G, r, n, slot_floats);
        if (etid == 0) p.counters[t] = 0;
      }
    }
  }

  if (p.cluster_s > 1) {
    __syncwarp();
    // Every CTA of the cluster has its partial sums in shared memory: CTA
    // `rank` of tile t sums its share of the tile's columns (4-column groups
    // [rank*32/s, (rank+1)*32/s)) over the cluster's CTAs in rank order
    // (deterministic), applies SiLU * up and stores Y.  The second barrier keeps every CTA (and its shared memory)
    // alive until its peers have read it.
    cluster_sync_all();
    if (warp >= 2) {
      const int s = p.cluster_s;
      const int rank = static_cast<int>(cluster_ctarank());
      const int t = static_cast<int>(blockIdx.x) / s;
      // groups of 4 columns: this CTA owns groups [rank*32/s, (rank+1)*32/s)
      const int g_lo = rank * (kTileN / 4) / s, g_hi = (rank + 1) * (kTileN / 4) / s;
      const int ngroups = g_hi - g_lo;
      const uint32_t part = smem_u32(smem);
      const int etid = threadIdx.x - 64;
      for (int e = etid; e < p.M * ngroups; e += 128) {
        const int m = e / ngroups, c = (g_lo + e % ngroups) * 4;
        const uint32_t og = part + static_cast<uint32_t>(m * kTileN + c) * 4u;
        const uint32_t ou = part + static_cast<uint32_t>((p.Mp + m) * kTileN + c) * 4u;
        float4 gv[8], uv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          gv[j] = j < s ? ld_shared_cluster_v4f32(map_shared_rank(og, j)) : make_float4(0.f, 0.f, 0.f, 0.f);
          uv[j] = j < s ? ld_shared_cluster_v4f32(map_shared_rank(ou, j)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float4 gs = make_float4(0.f, 0.f, 0.f, 0.f), us = gs;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          gs.x += gv[j].x;
          gs.y += gv[j].y;
          gs.z += gv[j].z;
          gs.w += gv[j].w;
          us.x += uv[j].x;
          us.y += uv[j].y;
          us.z += uv[j].z;
          us.w += uv[j].w;
        }
        const int n = t * kTileN + c;
        if (n < p.N) store_y(p, m, n, silu_mul_mode<kFast>(gs.x, us.x));
        if (n + 1 < p.N) store_y(p, m, n + 1, silu_mul_mode<kFast>(gs.y, us.y));
        if (n + 2 < p.N) store_y(p, m, n + 2, silu_mul_mode<kFast>(gs.z, us.z));
        if (n + 3 < p.N) store_y(p, m, n + 3, silu_mul_mode<kFast>(gs.w, us.w));
      }
    }
    cluster_sync_all();
  }
  if (threadIdx.x == 64) DECODE_TRACE(5);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
  if (threadIdx.x == 0 && st->abort != 0 && p.status != nullptr) atomicExch(p.status, st->abort);
  if (threadIdx.x == 0) DECODE_TRACE(6);
}


int padded_m(int64_t M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  return 128;
}

int stage_bytes_for(int Mp) { return 4 * static_cast<int>(kSlab) + ((Mp * kBK * 2 + 1023) & ~1023); }

}  // namespace

// Above 16 tokens the tcgen05 prefill kernel streams the weights as fast
// (measured on B200 for N = 14336, K = 4096) and needs no workspace.
int decode_max_m() { return 16; }

bool decode_supported(int64_t M, int64_t N, int64_t K, int) {
  return M >= 1 && M <= 128 && N >= 1 && K >= 1 && N <= INT32_MAX && K <= INT32_MAX &&
         static_cast<size_t>((N + kTileN - 1) / kTileN) * sizeof(int) <= kCounterRegion;
}

// Clusters of s CTAs with `smem` bytes each that the current device holds
// at once (cached per device, s and smem; 0 when the query fails).
int max_active_clusters(int s, int smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_tuple(dev, s, smem);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = 0;
  if (cudaFuncSetAttribute(decode_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) ==
      cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = s;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(s);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, decode_kernel<false>, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = n;
  return n;
}

// Shared memory the cluster mode's partial sums take: [gate | up][Mp][128] f32.
int cluster_partial_bytes(int Mp) { return 2 * Mp * kTileN * static_cast<int>(sizeof(float)); }

DecodePlan decode_plan(int64_t M, int64_t N, int64_t K, int sm_count) {
  DecodePlan d;
  const int Mp = padded_m(M);
  d.block_m = Mp;
  d.block_n = kTileN;
  d.block_k = kBK;
  d.cluster = 0;
  const int sb = stage_bytes_for(Mp);
  int stages = (kSmemBudget - 1024 - static_cast<int>(sizeof(DecodeTail))) / sb;
  d.stages = stages > 8 ? 8 : stages;
  const long long n_tiles = (N + kTileN - 1) / kTileN;
  const long long kb_per_tile = (K + kBK - 1) / kBK;
  const long long total = n_tiles * kb_per_tile;
  long long grid = sm_count;
  if (n_tiles * 2 >= sm_count && n_tiles <= sm_count) {
    // When the column tiles alone fill at least half the SMs, one CTA per
    // tile (no split, no fix-up) streams fastest: measured on B200 for
    // N = 14336, K = 4096 (112 tiles): 41 us at M = 1 against 49 us split
    // over 148 CTAs, with 4 stages in flight.
    grid = n_tiles;
    d.stages = d.stages < 4 ? d.stages : 4;
  } else if (n_tiles * 2 < sm_count) {
    // Fewer tiles than half the SMs (a column shard): split every tile's
    // k-blocks over a cluster of s CTAs, s = SMs / tiles (at most 8, the
    // portable cluster size), and reduce through distributed shared memory.
    // Measured on B200 (M = 1, K = 4096, N = 1792, 14 tiles): the workspace
    // fix-up of the stream-K split (fence, counter, loads through L2 by the
    // last CTA to arrive) kept the kernel at 12-17 us whatever the grid.
    // The largest s whose n_tiles clusters are all resident at once (a
    // second wave of clusters would double the time; GPCs hold whole
    // clusters only).
    long long cs = sm_count / n_tiles;
    if (cs > 8) cs = 8;
    if (cs > kb_per_tile) cs = kb_per_tile;
    const int smem = d.stages * sb + static_cast<int>(sizeof(DecodeTail)) + 1024;
    for (; cs >= 2; --cs)
      if (d.stages * sb >= cluster_partial_bytes(Mp) && max_active_clusters(static_cast<int>(cs), smem) >= n_tiles)
        break;
    if (cs >= 2) {
      d.cluster = static_cast<int>(cs);
      grid = n_tiles * cs;
    }
  }
  // every CTA streams at least one work unit
  if (grid > total) grid = total;
  if (grid < 1) grid = 1;
  d.grid = static_cast<int>(grid);
  d.split_k = d.cluster ? d.cluster : static_cast<int>((grid + n_tiles - 1) / n_tiles);
  d.threads = kThreads;
  d.smem_bytes = d.stages * sb + static_cast<int>(sizeof(DecodeTail)) + 1024;
  return d;
}

size_t decode_workspace_bytes(int64_t M, int64_t N, int64_t K, const DecodePlan &d) {
  if (d.cluster >= 2) return kPartialsOffset;  // partial sums stay in shared memory
  const long long kb_per_tile = (K + kBK - 1) / kBK;
  const long long total = ((N + kTileN - 1) / kTileN) * kb_per_tile;
  // Partial-sum slots only when some CTA range starts inside a tile.
  bool shared = false;
  for (long long c = 1; c < d.grid && !shared; ++c) shared = (c * total / d.grid) % kb_per_tile != 0;
  if (!shared) return kPartialsOffset;
  return kPartialsOffset + static_cast<size_t>(d.grid) * 2 * 2 * padded_m(M) * kTileN * sizeof(float);
}

int decode_max_grid_for(int64_t M, size_t workspace_bytes) {
  if (workspace_bytes <= kPartialsOffset) return 0;
  const size_t per_cta = static_cast<size_t>(2) * 2 * padded_m(M) * kTileN * sizeof(float);
  const size_t g = (workspace_bytes - kPartialsOffset) / per_cta;
  return g > INT32_MAX ? INT32_MAX : static_cast<int>(g);
}

size_t decode_counter_offset(int64_t, int64_t) { return kCounterOffset; }
size_t decode_counter_bytes(int64_t N) { return static_cast<size_t>((N + kTileN - 1) / kTileN) * sizeof(int); }

bool decode_plan_valid(int64_t M, int64_t N, int64_t K, const DecodePlan &d) {
  if (d.block_m != padded_m(M) || d.block_n != kTileN || d.block_k != kBK) return false;
  if (d.stages < 2 || d.stages > 8 || d.grid < 1) return false;
  const int sb = stage_bytes_for(d.block_m);
  if (d.stages * sb + static_cast<int>(sizeof(DecodeTail)) + 1024 > 227 * 1024) return false;
  const long long kb_per_tile = (K + kBK - 1) / kBK;
  const long long n_tiles = (N + kTileN - 1) / kTileN;
  const long long total = n_tiles * kb_per_tile;
  if (d.cluster != 0) {
    return d.cluster >= 2 && d.cluster <= 8 && d.cluster <= kb_per_tile && d.grid == n_tiles * d.cluster &&
           d.stages * sb >= cluster_partial_bytes(d.block_m);
  }
  return d.grid <= total;
}

cudaError_t decode_launch(const CUtensorMap &wg, const CUtensorMap &wu, const CUtensorMap &x, void *y, int64_t ldy,
                          int y_f32, int64_t M, int64_t N, int64_t K, void *workspace, int *status,
                          const DecodePlan &d, int slab_major, int fast_math, cudaStream_t stream) {
  if (!decode_plan_valid(M, N, K, d)) return cudaErrorInvalidValue;
  DecodeParams p;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.Mp = d.block_m;
  p.n_tiles = static_cast<int>((N + kTileN - 1) / kTileN);
  p.kb_per_tile = static_cast<int>((K + kBK - 1) / kBK);
  p.total = static_cast<long long>(p.n_tiles) * p.kb_per_tile;
  p.stages = d.stages;
  p.y_f32 = y_f32;
  p.slab_major = slab_major;
  p.y = y;
  p.ldy = ldy;
  p.counters = reinterpret_cast<int *>(static_cast<char *>(workspace) + kCounterOffset);
  p.partials = reinterpret_cast<float *>(static_cast<char *>(workspace) + kPartialsOffset);
  p.status = status;
  p.cluster_s = d.cluster;
  const int smem = d.stages * stage_bytes_for(d.block_m) + static_cast<int>(sizeof(DecodeTail)) + 1024;
  // The attribute is set once per device to the most any plan may use.
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set.load(std::memory_order_relaxed) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  // Programmatic stream serialisation: this launch's CTAs may start (and set
  // up) while the previous kernel in the stream finishes; the kernel waits
  // for it before touching memory.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = d.cluster >= 2 ? d.cluster : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.gridDim = dim3(d.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = d.cluster >= 2 ? 2 : 1;
  cudaError_t e = fast_math ? cudaLaunchKernelEx(&cfg, decode_kernel<true>, wg, wu, x, p)
                            : cudaLaunchKernelEx(&cfg, decode_kernel<false>, wg, wu, x, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace llk_b200

#ifdef LLK_DECODE_TRACE
extern "C" int llk_trace_decode_read(void *host, size_t bytes) {
  return cudaMemcpyFromSymbol(host, llk_b200::g_decode_trace, bytes) == cudaSuccess ? 0 : 3;
}
#endif
