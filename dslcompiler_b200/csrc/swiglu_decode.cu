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

#include "decode_kernels.h"
#include "sm100_ptx.cuh"

namespace llk_b200 {

namespace {

constexpr int kThreads = 192;
constexpr int kTileN = 128;        // weight columns per tile (MMA M)
constexpr int kBK = 64;            // k per stage
constexpr uint32_t kSlab = 64 * kBK * 2;  // 64 n x 64 k bf16 = 8 KB
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr int kSmemBudget = 220 * 1024;
// Workspace layout, the same for every shape so a workspace reused across
// shapes never has a counter landing on another call's partial sums:
//   [0, 256)                 reserved for the CTA-pair kernel's work counter
//   [256, 256 + 256 KB)      per-tile arrival counters (65536 tiles, N <= 8 M)
//   [256 + 256 KB, ...)      partial sums, two slots per CTA.
constexpr size_t kCounterOffset = 256;
constexpr size_t kCounterRegion = 256 * 1024;
constexpr size_t kPartialsOffset = kCounterOffset + kCounterRegion;

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

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void store_y(const DecodeParams &p, int m, int n, float v) {
  if (p.y_f32) {
    reinterpret_cast<float *>(p.y)[(long long)m * p.ldy + n] = v;
  } else {
    reinterpret_cast<uint16_t *>(p.y)[(long long)m * p.ldy + n] = static_cast<uint16_t>(pack_bf16x2(v, 0.f));
  }
}

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

      if (n_contrib == 1) {
        for (int m0 = 0; m0 < p.Mp; m0 += 16) {
          uint32_t g[16], uu[16];
          tmem_ld_32x32b_x16(t_row + m0, g);
          tmem_ld_32x32b_x16(t_row + p.Mp + m0, uu);
          tmem_ld_wait();
          if (n < p.N) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (m0 + j < p.M) store_y(p, m0 + j, n, silu_mul(__uint_as_float(g[j]), __uint_as_float(uu[j])));
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
        // Sum the contributors' slots in slot order (deterministic), 16
        // token rows at a time so the loads of a row block are in flight
        // together.
        for (int m0 = 0; m0 < p.M; m0 += 16) {
          const int rows = p.M - m0 < 16 ? p.M - m0 : 16;
          float gs[16], us[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) gs[j] = us[j] = 0.f;
          for (long long c = c_first; c <= c_last; ++c) {
            // contributor c's slot for tile t (the same rule the writer used)
            const int which = range_begin(c, p.total, G) / p.kb_per_tile == t ? 0 : 1;
            const float *ps = p.partials + ((size_t)c * 2 + which) * slot_floats + (size_t)m0 * kTileN + r;
            float gv[16], uv[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              gv[j] = j < rows ? __ldcg(ps + (size_t)j * kTileN) : 0.f;
              uv[j] = j < rows ? __ldcg(ps + (size_t)(p.Mp + j) * kTileN) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              gs[j] += gv[j];
              us[j] += uv[j];
            }
          }
          if (n < p.N) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (m0 + j < p.M) store_y(p, m0 + j, n, silu_mul(gs[j], us[j]));
          }
        }
        if (etid == 0) p.counters[t] = 0;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
  if (threadIdx.x == 0 && st->abort != 0 && p.status != nullptr) atomicExch(p.status, st->abort);
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

DecodePlan decode_plan(int64_t M, int64_t N, int64_t K, int sm_count) {
  DecodePlan d;
  const int Mp = padded_m(M);
  d.block_m = Mp;
  d.block_n = kTileN;
  d.block_k = kBK;
  const int sb = stage_bytes_for(Mp);
  int stages = (kSmemBudget - 1024 - static_cast<int>(sizeof(DecodeTail))) / sb;
  d.stages = stages > 8 ? 8 : stages;
  const long long n_tiles = (N + kTileN - 1) / kTileN;
  const long long total = n_tiles * ((K + kBK - 1) / kBK);
  long long grid = sm_count;
  // When the column tiles alone fill at least half the SMs, one CTA per tile
  // (no split, no fix-up) streams fastest: measured on B200 for N = 14336,
  // K = 4096 (112 tiles): 41 us at M = 1 against 49 us split over 148 CTAs,
  // with 4 stages in flight.
  if (n_tiles * 2 >= sm_count && n_tiles <= sm_count) {
    grid = n_tiles;
    d.stages = d.stages < 4 ? d.stages : 4;
  }
  // every CTA streams at least one work unit
  if (grid > total) grid = total;
  if (grid < 1) grid = 1;
  d.grid = static_cast<int>(grid);
  d.split_k = static_cast<int>((grid + ((N + kTileN - 1) / kTileN) - 1) / ((N + kTileN - 1) / kTileN));
  d.threads = kThreads;
  d.smem_bytes = d.stages * sb + static_cast<int>(sizeof(DecodeTail)) + 1024;
  return d;
}

size_t decode_workspace_bytes(int64_t M, int64_t N, int64_t K, int grid) {
  const long long kb_per_tile = (K + kBK - 1) / kBK;
  const long long total = ((N + kTileN - 1) / kTileN) * kb_per_tile;
  // Partial-sum slots only when some CTA range starts inside a tile.
  bool shared = false;
  for (long long c = 1; c < grid && !shared; ++c) shared = (c * total / grid) % kb_per_tile != 0;
  if (!shared) return kPartialsOffset;
  return kPartialsOffset + static_cast<size_t>(grid) * 2 * 2 * padded_m(M) * kTileN * sizeof(float);
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
  const long long total = ((N + kTileN - 1) / kTileN) * kb_per_tile;
  return d.grid <= total;
}

cudaError_t decode_launch(const CUtensorMap &wg, const CUtensorMap &wu, const CUtensorMap &x, void *y, int64_t ldy,
                          int y_f32, int64_t M, int64_t N, int64_t K, void *workspace, int *status,
                          const DecodePlan &d, int slab_major, cudaStream_t stream) {
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
  const int smem = d.stages * stage_bytes_for(d.block_m) + static_cast<int>(sizeof(DecodeTail)) + 1024;
  // The attribute is set once per device to the most any plan may use.
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set.load(std::memory_order_relaxed) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  decode_kernel<<<d.grid, kThreads, smem, stream>>>(wg, wu, x, p);
  return cudaGetLastError();
}

}  // namespace llk_b200
