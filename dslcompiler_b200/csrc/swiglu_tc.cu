// swiglu_tc.cu -- persistent tcgen05 kernel for the fused SwiGLU and the
// micro.mma matmul on sm_100a.
//
// Computes, per 128-row tile of X:
//   SwiGLU:  Y[:, n0:n0+128] = SiLU(X Wg[:, n0:n0+128]) * (X Wu[:, n0:n0+128])
//            as ONE 128x256 MMA per K step whose B operand is
//            [Wg slab | Wu slab] -- gate in TMEM columns 0-127, up in 128-255
//            (the two f32 accumulators of
//            lib/Transforms/FuseDoubleContraction.cpp:119-173);
//   matmul:  C[:, n0:n0+256] (+)= A B  (micro.mma, MicroOps.td:196-222).
//
// Roles (6 warps):
//   warp 0    TMA producer: X tile (128 x 64, K-major, 128B swizzle) and four
//             64 x 64 B slabs per stage (MN-major: the weights are row-major
//             [K, N] so N is contiguous), 4-stage shared-memory ring.
//   warp 1    allocates 512 TMEM columns (two 256-column accumulators) and
//             issues tcgen05.mma from one thread; commits free smem stages
//             and hand finished accumulators to the epilogue.
//   warps 2-5 epilogue: tcgen05.ld 32 columns at a time, SiLU * up (or the
//             plain accumulator, + C when accumulating), one vector store.
// The second accumulator lets the epilogue of tile i overlap the MMAs of
// tile i+1.  Every mbarrier wait is bounded (sm100_ptx.cuh).
// No TMA multicast anywhere: each CTA loads its own tiles.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "sm100_ptx.cuh"
#include "tc_kernels.h"

namespace llk_b200 {

namespace {

constexpr int kThreads = 192;
constexpr int kStages = 4;
constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kMmaN = 256;
constexpr int kUmmaK = 16;
constexpr uint32_t kABytes = kBM * kBK * 2;        // 16 KB
constexpr uint32_t kSlabBytes = 64 * kBK * 2;      // 8 KB: 64 n x 64 k
constexpr uint32_t kBBytes = 4 * kSlabBytes;       // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;  // 48 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

struct __align__(8) SharedTail {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    tc_swiglu_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b0,
                     const __grid_constant__ CUtensorMap tm_b1, const TcParams p) {
  constexpr int kMode = MODE & ~TC_FAST_MATH;
  constexpr bool kFast = (MODE & TC_FAST_MATH) != 0;
  constexpr bool kSwiglu = (kMode == TC_SWIGLU_BF16 || kMode == TC_SWIGLU_F32);
  constexpr int kTileN = kSwiglu ? 128 : 256;  // output columns per tile

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzle atoms.
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SharedTail *st = reinterpret_cast<SharedTail *>(smem + kStages * kStageBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
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
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b0);
    if (kSwiglu) tma_prefetch_desc(&tm_b1);
  }
  if (warp == 1) {
    tmem_alloc(&st->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  pdl_wait();  // the previous kernel's writes are visible from here on
  const uint32_t tmem_base = st->tmem_base;
  volatile int *abort = &st->abort;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile % p.m_tiles) * kBM;
        const int n0 = (tile / p.m_tiles) * kTileN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&st->empty[stage], phase ^ 1u, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + stage * kStageBytes;
          uint8_t *sb = sa + kABytes;
          mbar_arrive_expect_tx(&st->full[stage], kStageBytes);
          const int k0 = kb * kBK;
          tma_load_2d(sa, &tm_a, &st->full[stage], k0, m0);
          if (kSwiglu) {
            tma_load_weight_slab(sb + 0 * kSlabBytes, &tm_b0, &st->full[stage], n0, k0, p.slab_major);
            tma_load_weight_slab(sb + 1 * kSlabBytes, &tm_b0, &st->full[stage], n0 + 64, k0, p.slab_major);
            tma_load_weight_slab(sb + 2 * kSlabBytes, &tm_b1, &st->full[stage], n0, k0, p.slab_major);
            tma_load_weight_slab(sb + 3 * kSlabBytes, &tm_b1, &st->full[stage], n0 + 64, k0, p.slab_major);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tma_load_weight_slab(sb + j * kSlabBytes, &tm_b0, &st->full[stage], n0 + 64 * j, k0, p.slab_major);
          }
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let the loads already in flight land before the CTA exits: wait
        // (bounded) on the full barrier of each of the last stages issued.
        uint32_t n = issued < kStages ? issued : kStages;
        for (uint32_t i = 0; i < n; ++i) {
          uint32_t idx = issued - 1 - i;
          int dummy = 0;
          mbar_wait_bounded(&st->full[idx % kStages], (idx / kStages) & 1u, &dummy, 1, 100000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t idesc = make_idesc_bf16_f32(kBM, kMmaN, false, true);
      const uint32_t smem_base = smem_u32(smem);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      int local = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++local) {
        const uint32_t acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&st->tmem_empty[acc], acc_phase ^ 1u, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kMmaN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&st->full[stage], phase, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_base + stage * kStageBytes;
          const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            // A: K-major, advance 16 elements (32 bytes) inside the swizzle atom.
            const uint64_t a_desc = make_smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            // B: MN-major, advance 16 k-rows = two 8-row groups (2 KB).
            const uint64_t b_desc = make_smem_desc_sw128(b_addr + kk * 2048, p.b_lbo, p.b_sbo);
            tc_mma_bf16(d_tmem, a_desc, b_desc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&st->empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&st->tmem_full[acc]);
      }
      // Every MMA this thread issued has finished before TMEM is released.
      tc_commit(&st->mma_done);
      int dummy = 0;
      mbar_wait_bounded(&st->mma_done, 0, &dummy, 1, 100000000ull);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      const uint32_t acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_bounded(&st->tmem_full[acc], acc_phase, abort, LLK_ERR_TIMEOUT, kWaitLimitNs)) break;
      tc_fence_after();
      const int m0 = (tile % p.m_tiles) * kBM;
      const int n0 = (tile / p.m_tiles) * kTileN;
      const int row = m0 + row_in_tile;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kMmaN;
      if (kSwiglu) {
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(t_row + c, g);
          tmem_ld_32x32b_x32(t_row + 128 + c, u);
          tmem_ld_wait();
          const int col = n0 + c;
          if (row < p.M && col < p.N) {
            float y[32];
            silu_mul_block<kFast, 32>(g, u, y);
            if (kMode == TC_SWIGLU_BF16) {
              uint16_t *dst = reinterpret_cast<uint16_t *>(p.y) + (int64_t)row * p.ldy + col;
              if (p.vec_ok && col + 32 <= p.N) {
                uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll
                for (int v = 0; v < 4; ++v)
                  d4[v] = make_uint4(pack_bf16x2(y[8 * v + 0], y[8 * v + 1]), pack_bf16x2(y[8 * v + 2], y[8 * v + 3]),
                                     pack_bf16x2(y[8 * v + 4], y[8 * v + 5]), pack_bf16x2(y[8 * v + 6], y[8 * v + 7]));
              } else {
                uint16_t *d16 = dst;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (col + j < p.N) d16[j] = static_cast<uint16_t>(pack_bf16x2(y[j], 0.f));
              }
            } else {
              float *dst = reinterpret_cast<float *>(p.y) + (int64_t)row * p.ldy + col;
              if (p.vec_ok && col + 32 <= p.N) {
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
      } else {
#pragma unroll 1
        for (int c = 0; c < 256; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c, r);
          tmem_ld_wait();
          const int col = n0 + c;
          if (row < p.M && col < p.N) {
            float *dst = reinterpret_cast<float *>(p.y) + (int64_t)row * p.ldy + col;
            if (p.vec_ok && col + 32 <= p.N) {
              float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                float4 o = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                       __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                if (kMode == TC_MATMUL_F32_ACC) {
                  float4 c4 = d4[v];
                  o.x += c4.x;
                  o.y += c4.y;
                  o.z += c4.z;
                  o.w += c4.w;
                }
                d4[v] = o;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (col + j < p.N) {
                  float o = __uint_as_float(r[j]);
                  if (kMode == TC_MATMUL_F32_ACC) o += dst[j];
                  dst[j] = o;
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&st->tmem_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && st->abort != 0 && p.status != nullptr) atomicExch(p.status, st->abort);
}

}  // namespace

int tc_smem_bytes() { return kStages * kStageBytes + static_cast<int>(sizeof(SharedTail)) + 1024; }
int tc_threads() { return kThreads; }
int tc_tile_n(int mode) {
  const int base = mode & ~TC_FAST_MATH;
  return (base == TC_SWIGLU_BF16 || base == TC_SWIGLU_F32) ? 128 : 256;
}

template <int MODE>
static cudaError_t launch_mode(const CUtensorMap &a, const CUtensorMap &b0, const CUtensorMap &b1, const TcParams &p,
                               int grid, cudaStream_t stream) {
  auto kern = tc_swiglu_kernel<MODE>;
  const int smem = tc_smem_bytes();
  static std::atomic<uint64_t> attr_set{0};  // bit per device: smem attribute done
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_set.load(std::memory_order_relaxed) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  // Programmatic stream serialisation: CTAs may start and set up while the
  // previous kernel finishes (the kernel waits for it: pdl_wait).
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, b0, b1, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t tc_launch(int mode, const CUtensorMap &a, const CUtensorMap &b0, const CUtensorMap &b1, const TcParams &p,
                      int grid, cudaStream_t stream) {
  switch (mode) {
    case TC_SWIGLU_BF16:
      return launch_mode<TC_SWIGLU_BF16>(a, b0, b1, p, grid, stream);
    case TC_SWIGLU_F32:
      return launch_mode<TC_SWIGLU_F32>(a, b0, b1, p, grid, stream);
    case TC_SWIGLU_BF16 | TC_FAST_MATH:
      return launch_mode<TC_SWIGLU_BF16 | TC_FAST_MATH>(a, b0, b1, p, grid, stream);
    case TC_SWIGLU_F32 | TC_FAST_MATH:
      return launch_mode<TC_SWIGLU_F32 | TC_FAST_MATH>(a, b0, b1, p, grid, stream);
    case TC_MATMUL_F32:
      return launch_mode<TC_MATMUL_F32>(a, b0, b1, p, grid, stream);
    case TC_MATMUL_F32_ACC:
      return launch_mode<TC_MATMUL_F32_ACC>(a, b0, b1, p, grid, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace llk_b200
