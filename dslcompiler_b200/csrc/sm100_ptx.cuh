// sm100_ptx.cuh -- thin inline-PTX wrappers for the sm_100a features the
// SwiGLU / micro.mma kernels use: mbarriers, TMA tiled loads (no multicast),
// tcgen05 MMA / commit / TMEM alloc / TMEM loads, and a bounded mbarrier wait
// that reports a timeout instead of spinning forever.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "llk_b200.h"

namespace llk_b200 {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------- programmatic dependent launch
// Kernels launched with programmatic stream serialisation start their CTAs
// while the previous kernel in the stream is still finishing: they set up
// (barriers, TMEM, descriptor prefetch) and then wait here, before their
// first global-memory access, until that kernel has completed and its writes
// are visible.  Without a programmatic dependency the wait returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel's CTAs launch (onto SMs as this kernel's CTAs leave).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase of `bar` with the given parity to complete.  Gives up
// after `limit_ns` of wall time or as soon as another role in the CTA has
// raised *abort; on giving up it records `code` in *abort and returns false.
// No wait in these kernels can spin forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, volatile int *abort,
                                                  int code, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*abort != 0) return false;
      if (global_timer_ns() - t0 > limit_ns) {
        *abort = code;
        return false;
      }
    }
  }
}

// 16-byte global -> shared copy through L2 (cp.async, no TMA), and the wait
// for all of the thread's copies.
__device__ __forceinline__ void cp_async_16(void *smem_dst, const void *gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// ------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load into this CTA's shared memory; completion is signalled as
// transaction bytes on `bar`.  c0 is the innermost coordinate (elements);
// callers keep c0 * element size a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int32_t c0,
                                            int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 3-D tiled load (c0 innermost).  Used for slab-major packed weights.
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int32_t c0,
                                            int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Loads the 64-column x 64-k weight slab whose first column is n (a
// multiple of 64) and first row k: from a row-major [K, N] tensor map
// (2-D, {N, K}) or from slab-major packed weights (3-D, {64, K, N/64}).
__device__ __forceinline__ void tma_load_weight_slab(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int n,
                                                     int k, bool slab_major) {
  if (slab_major) {
    tma_load_3d(smem_dst, map, bar, 0, k, n >> 6);
  } else {
    tma_load_2d(smem_dst, map, bar, n, k);
  }
}

// --------------------------------------------------------------- tcgen05
// Shared-memory matrix descriptor (tcgen05 format): start address >> 4 in
// bits 0-13, leading-dimension byte offset >> 4 in 16-29, stride-dimension
// byte offset >> 4 in 32-45, descriptor version 1 in bit 46, swizzle mode in
// bits 61-63 (2 = 128-byte swizzle).  Base offset 0: every operand tile
// starts on a 1024-byte boundary.
__host__ __device__ __forceinline__ uint64_t make_smem_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes,
                                                                  uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor for tcgen05.mma kind::f16 with bf16 A/B and f32
// accumulation: D format f32 (bits 4-5 = 1), A format bf16 (bits 7-9 = 1),
// B format bf16 (bits 10-12 = 1), A major (bit 15), B major (bit 16;
// 1 = MN-major), N >> 3 (bits 17-22), M >> 4 (bits 24-28).
__host__ __device__ __forceinline__ constexpr uint32_t make_idesc_bf16_f32(uint32_t M, uint32_t N, bool a_mn_major,
                                                                           bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((N >> 3) << 17) | ((M >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t *smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]; issued by a single thread.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 op issued so far by this thread
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (base lane + t), columns col .. col+31.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Global int load with acquire semantics at GPU scope (for counters other
// CTAs release with a fence + atomic).
__device__ __forceinline__ int ld_acquire_gpu(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(lo), "f"(hi));
  return r;
}

// SiLU(g) * u = g / (1 + e^-g) * u with CUDA's fast exp and fast division
// (__fdividef: reciprocal approximation and a multiply, 2 ulp; it gives 0 for
// the divisors above 2^126 that e^-g reaches for g < -87, where SiLU(g)
// underflows anyway).  The IEEE-rounded '/' made each element cost ~10x
// more, enough to make the epilogue slower than a tile's MMAs (measured on
// B200: 24 us against 22 us per tile at K = 4096; 5 us with __fdividef).
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

// Correctly rounded reciprocal of b in [1, 2^126) by Markstein's method
// (P. Markstein, "IA-64 and Elementary Functions", 2000, ch. 8): the
// hardware's approximate reciprocal, then two residual corrections
// e = 1 - b*y, y = y + e*y, each one FMA.  The result equals the IEEE
// division 1.0f / b for every such b: checked against __frcp_rn over all
// 2^30 floats of the range on a B200 (llk_diag_reciprocal_check).  No check
// of the range here; rcp_rn_ge1 adds it.
__device__ __forceinline__ float rcp_rn_markstein(float b) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
  float e = fmaf(-b, y, 1.0f);
  y = fmaf(e, y, y);
  e = fmaf(-b, y, 1.0f);
  return fmaf(e, y, y);
}

// 1 / b correctly rounded for b >= 1: Markstein's method in its range, CUDA's
// correctly rounded reciprocal where the result would be denormal or zero.
__device__ __forceinline__ float rcp_rn_ge1(float b) {
  if (!(b < 0x1p126f)) return __frcp_rn(b);
  return rcp_rn_markstein(b);
}

// The strict epilogue of the fused lowering (the reference's math.exp /
// arith.divf sequence, lib/Transforms/FuseDoubleContraction.cpp:189-196):
// sigmoid = 1 / (1 + exp(-g)) with CUDA's accurate expf and the reciprocal
// correctly rounded (the same value as the IEEE division), silu = g *
// sigmoid, r = silu * u -- the same operations in the same order.
__device__ __forceinline__ float silu_mul_strict(float g, float u) {
  const float sigmoid = rcp_rn_ge1(1.0f + expf(-g));
  return (g * sigmoid) * u;
}

// y[j] = SiLU(g[j]) * u[j] for a block of N elements (bit patterns of f32,
// as tcgen05.ld returns them), strict or fast.  The strict block checks the
// reciprocal's range outside its unrolled loop and redoes the rare elements
// with 1 + e^-g >= 2^126 (g < -87) afterwards, so the common path stays
// straight-line code: a full '/' made each tile's epilogue slower than its
// MMAs, and a branch per element still cost half the epilogue's throughput
// (measured on B200: 12 -> 5.6 us per 256 x 128 tile).
template <bool kFast, int N>
__device__ __forceinline__ void silu_mul_block(const uint32_t (&gb)[N], const uint32_t (&ub)[N], float (&y)[N]) {
  float g[N], u[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    g[j] = __uint_as_float(gb[j]);
    u[j] = __uint_as_float(ub[j]);
  }
  if constexpr (kFast) {
#pragma unroll
    for (int j = 0; j < N; ++j) y[j] = silu_mul(g[j], u[j]);
  } else {
    float x[N];
    bool rare = false;
#pragma unroll
    for (int j = 0; j < N; ++j) {
      x[j] = 1.0f + expf(-g[j]);
      rare |= !(x[j] < 0x1p126f);
    }
#pragma unroll
    for (int j = 0; j < N; ++j) y[j] = (g[j] * rcp_rn_markstein(x[j])) * u[j];
    if (rare) {
#pragma unroll
      for (int j = 0; j < N; ++j)
        if (!(x[j] < 0x1p126f)) y[j] = (g[j] * __frcp_rn(x[j])) * u[j];
    }
  }
}

template <bool kFast, int N>
__device__ __forceinline__ void silu_mul_block(const float (&g)[N], const float (&u)[N], float (&y)[N]) {
  uint32_t gb[N], ub[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    gb[j] = __float_as_uint(g[j]);
    ub[j] = __float_as_uint(u[j]);
  }
  silu_mul_block<kFast, N>(gb, ub, y);
}

// Epilogue by math mode: kFast = bounded/unsafe fast (silu_mul), else strict.
template <bool kFast>
__device__ __forceinline__ float silu_mul_mode(float g, float u) {
  if constexpr (kFast) {
    return silu_mul(g, u);
  } else {
    return silu_mul_strict(g, u);
  }
}

// ----------------------------------------------------- CTA pairs (2-SM MMA)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t map_shared_rank(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

// 32-bit load from shared memory anywhere in the cluster (shared::cluster address).
__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}

__device__ __forceinline__ float4 ld_shared_cluster_v4f32(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier anywhere in the cluster (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA tiled loads of the 2-SM form: the destination is this CTA's shared
// memory, the completion barrier may be in either CTA of the pair (here:
// always the pair leader's).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const CUtensorMap *map, uint32_t bar_cluster,
                                                 int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void *smem_dst, const CUtensorMap *map, uint32_t bar_cluster,
                                                 int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_weight_slab_pair(void *smem_dst, const CUtensorMap *map,
                                                          uint32_t bar_cluster, int n, int k, bool slab_major) {
  if (slab_major) {
    tma_load_3d_pair(smem_dst, map, bar_cluster, 0, k, n >> 6);
  } else {
    tma_load_2d_pair(smem_dst, map, bar_cluster, n, k);
  }
}

// L2 eviction-priority policies for the cache-hinted loads below
// (createpolicy.fractional with fraction 1.0: every line the load touches).
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Pair loads with an L2 cache policy.
__device__ __forceinline__ void tma_load_2d_pair_hint(void *smem_dst, const CUtensorMap *map, uint32_t bar_cluster,
                                                      int32_t c0, int32_t c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair_hint(void *smem_dst, const CUtensorMap *map, uint32_t bar_cluster,
                                                      int32_t c0, int32_t c1, int32_t c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_weight_slab_pair_hint(void *smem_dst, const CUtensorMap *map,
                                                               uint32_t bar_cluster, int n, int k, bool slab_major,
                                                               uint64_t policy) {
  if (slab_major) {
    tma_load_3d_pair_hint(smem_dst, map, bar_cluster, 0, k, n >> 6, policy);
  } else {
    tma_load_2d_pair_hint(smem_dst, map, bar_cluster, n, k, policy);
  }
}

// TMA tensor store shared -> global (bulk-group completion), and the
// group bookkeeping around it.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t smem_src, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_src), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N committed groups still READ shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Generic-proxy shared-memory writes become visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// TMEM allocation for a CTA pair: issued by the same warp in both CTAs,
// with the same shared-memory slot offset.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D (+)= A * B over the CTA pair (M = 256: 128 rows of A from each CTA's
// shared memory; B's N columns split in halves between the CTAs); issued by
// one thread of the pair leader.  All output lanes enabled.
__device__ __forceinline__ void tc_mma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z)
      : "memory");
}

// Arrive once on the barrier at this shared-memory offset in every CTA of
// `cta_mask` when all tcgen05 ops issued so far by this thread completed.
__device__ __forceinline__ void tc_commit_pair_mc(uint64_t *bar, uint16_t cta_mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                   "r"(smem_u32(bar)),
               "h"(cta_mask)
               : "memory");
}



// Wait on a barrier that other CTAs of the cluster arrive on, with
// cluster-scope acquire (makes their shared::cluster stores visible).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t *bar, uint32_t parity, volatile int *abort,
                                                          int code, uint64_t limit_ns) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*abort != 0) return false;
      if (global_timer_ns() - t0 > limit_ns) {
        *abort = code;
        return false;
      }
    }
  }
}

// 32-bit store into another CTA's shared memory (shared::cluster address).
__device__ __forceinline__ void st_shared_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

}  // namespace llk_b200
