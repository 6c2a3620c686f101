// rope_attention.cu -- the llk.rope and llk.attention ops on sm_100a.
//
// Both ops are f32 in the reference (include/LLK/Dialect/LLKOps.td:69-131)
// and lowered by lib/Conversion/LLKToLinalg/LLKToLinalg.cpp:162-615; these
// kernels compute the same results on the GPU.
//
// RoPE (x [B,H,L,D] f32, position_ids [L] i64, theta):
//   freq[i] = theta^(-2i/D) (f64), angle[p,i] = pos[p] * freq[i] (f64),
//   c, s = cos / sin of the angle rounded to f32,
//   y[2i] = x[2i]*c - x[2i+1]*s,  y[2i+1] = x[2i+1]*c + x[2i]*s  (f32, each
//   product and sum rounded on its own, as the unfused arith ops are).
// HBM-bound: a small kernel builds the (cos, sin) table [L][D/2] once per
// call (it stays in L2), then a grid-stride kernel streams x -> y with
// 16-byte loads and stores, several in flight per thread.
//
// Attention (q [B,H,Lq,D], k/v [B,H,Lk,D] f32, scale, causal):
//   O = init + softmax(scale * Q K^T, masked where k > q when causal) V.
// The reference materialises the [Lq, Lk] scores and runs a 3-pass stable
// softmax; this kernel keeps a 64-row query tile on chip and sweeps 64-row
// key tiles with the online (running max / running sum) form of the same
// softmax -- identical in exact arithmetic, f32 rounding aside.  f32 inputs
// and f32 accumulation on the CUDA cores (the op is f32; tensor-core tf32
// would drop 13 mantissa bits of every product).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "attention_kernels.h"
#include "sm100_ptx.cuh"

namespace llk_b200 {

namespace {

// ------------------------------------------------------------------- RoPE
constexpr int kRopeThreads = 256;

template <bool kFast>
__device__ __forceinline__ void sincos_mode(float a, float *s, float *c) {
  if constexpr (kFast) {
    *s = __sinf(a);
    *c = __cosf(a);
  } else {
    *s = sinf(a);
    *c = cosf(a);
  }
}

// Rotation of one (even, odd) pair with unfused f32 multiplies and adds.
__device__ __forceinline__ float2 rotate(float e, float o, float c, float s) {
  return make_float2(__fsub_rn(__fmul_rn(e, c), __fmul_rn(o, s)), __fadd_rn(__fmul_rn(o, c), __fmul_rn(e, s)));
}

// The (cos, sin) table [L][D/2] (float2), built once per call: the
// frequencies and angles in f64, the trig of the f32 angle.
template <bool kFast>
__global__ void __launch_bounds__(kRopeThreads) rope_table_kernel(const int64_t *__restrict__ pos,
                                                                 float2 *__restrict__ table, int64_t L, int D,
                                                                 double theta) {
  const int half = D / 2;
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < L * half;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p = e / half;
    const int i = static_cast<int>(e % half);
    const double freq = pow(theta, (-2.0 * static_cast<double>(i)) / static_cast<double>(D));
    const double angle = static_cast<double>(pos[p]) * freq;
    float s, c;
    sincos_mode<kFast>(static_cast<float>(angle), &s, &c);
    table[e] = make_float2(c, s);
  }
}

// Streams x -> y with 16-byte accesses (D % 4 == 0; two pairs per access,
// their (cos, sin) one 16-byte table load from L2), kUnroll accesses in
// flight per thread; grid-stride over the whole tensor.
constexpr int kUnroll = 4;
__global__ void __launch_bounds__(kRopeThreads) rope_apply4_kernel(const float4 *__restrict__ x,
                                                                  const float4 *__restrict__ table,
                                                                  float4 *__restrict__ y, int64_t n4, int64_t L,
                                                                  int D) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int q4 = D / 4;  // accesses per row
  for (int64_t v0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v0 < n4; v0 += kUnroll * stride) {
    float4 a[kUnroll], cs[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = v0 + u * stride;
      if (v < n4) {
        a[u] = __ldcs(x + v);
        const int64_t row = v / q4;  // (b, h, p) row
        const int64_t p = row % L;
        cs[u] = table[p * q4 + (v - row * q4)];  // pairs 2j, 2j+1 of the row: (c0, s0, c1, s1)
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = v0 + u * stride;
      if (v < n4) {
        const float2 r0 = rotate(a[u].x, a[u].y, cs[u].x, cs[u].y), r1 = rotate(a[u].z, a[u].w, cs[u].z, cs[u].w);
        __stcs(y + v, make_float4(r0.x, r0.y, r1.x, r1.y));
      }
    }
  }
}

// D % 4 == 2: one pair per 8-byte access.
__global__ void __launch_bounds__(kRopeThreads) rope_apply2_kernel(const float2 *__restrict__ x,
                                                                  const float2 *__restrict__ table,
                                                                  float2 *__restrict__ y, int64_t n2, int64_t L,
                                                                  int D) {
  pdl_launch_dependents();
  pdl_wait();
  const int half = D / 2;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < n2;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = v / half;
    const int64_t p = row % L;
    const float2 cs = table[p * half + (v - row * half)];
    const float2 a = x[v];
    y[v] = rotate(a.x, a.y, cs.x, cs.y);
  }
}

// -------------------------------------------------------------- attention
constexpr int kBQ = 64;         // query rows per CTA
constexpr int kBK = 64;         // key rows per tile
constexpr int kAttnThreads = 256;
constexpr int kPad = 4;         // shared-memory row padding (floats)

template <bool kFast>
__device__ __forceinline__ float exp_mode(float v) {
  if constexpr (kFast) {
    return __expf(v);
  } else {
    return expf(v);
  }
}

// Query tile and head of this CTA.  The grid is one-dimensional over
// (query tile, head) with the LAST query tiles first: under a causal mask a
// tile's work grows with its index, so the heaviest CTAs start in the first
// wave and the light ones fill the end (longest-first order).
__device__ __forceinline__ void tile_of_block(int64_t Lq, int64_t &bh, int64_t &q0) {
  const int64_t n_qt = (Lq + kBQ - 1) / kBQ;
  const int64_t BH = static_cast<int64_t>(gridDim.x) / n_qt;
  const int64_t i = blockIdx.x;
  bh = i % BH;
  q0 = (n_qt - 1 - i / BH) * kBQ;
}

// Thread layout: ty = tid / 16 owns query rows 4*ty .. 4*ty+3 of the tile;
// tx = tid % 16 owns key columns 4*tx .. 4*tx+3 of the score tile and output
// columns {4*tx + 64*j .. +3} (j < DP/64).  The 16 threads of a row group are
// 16 consecutive lanes of one warp, so row reductions are warp shuffles.
// Shared memory (floats): Qt [DP][BQ+pad], Kt [DP][BK+pad] (both d-major),
// V [BK][DP+pad], Pt [BK][BQ+pad].
template <int DP, bool kFast>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                     float *__restrict__ o, int64_t Lq, int64_t Lk, int D, float scale, int causal) {
  extern __shared__ __align__(16) float sm[];
  float *Qt = sm;
  float *Kt = Qt + DP * (kBQ + kPad);
  float *Vs = Kt + DP * (kBK + kPad);
  float *Pt = Vs + kBK * (DP + kPad);
  constexpr int kOC = DP / 64;  // output float4 groups per thread

  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;
  int64_t bh, q0;
  tile_of_block(Lq, bh, q0);
  const float *qb = q + bh * Lq * D;
  const float *kb = k + bh * Lk * D;
  const float *vb = v + bh * Lk * D;
  float *ob = o + bh * Lq * D;

  pdl_launch_dependents();
  pdl_wait();
  // Q tile, transposed: Qt[d][r] (zero past Lq / D).
  for (int e = tid; e < kBQ * DP; e += kAttnThreads) {
    const int r = e / DP, d = e % DP;
    const int64_t qi = q0 + r;
    Qt[d * (kBQ + kPad) + r] = (qi < Lq && d < D) ? qb[qi * D + d] : 0.f;
  }

  float m[4], l[4], acc[4][kOC][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kOC; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[i][j][c] = 0.f;
  }

  // With the causal mask, key tiles past the tile's last query row carry no weight.
  int64_t k_end = Lk;
  if (causal) {
    const int64_t last_q = (q0 + kBQ - 1 < Lq - 1 ? q0 + kBQ - 1 : Lq - 1);
    k_end = last_q + 1 < Lk ? last_q + 1 : Lk;
  }
  for (int64_t k0 = 0; k0 < k_end; k0 += kBK) {
    __syncthreads();  // the previous tile's Kt / Vs / Pt are no longer read
    for (int e = tid; e < kBK * DP; e += kAttnThreads) {
      const int r = e / DP, d = e % DP;
      const int64_t ki = k0 + r;
      const bool in = ki < Lk && d < D;
      Kt[d * (kBK + kPad) + r] = in ? kb[ki * D + d] : 0.f;
      Vs[r * (DP + kPad) + d] = in ? vb[ki * D + d] : 0.f;
    }
    __syncthreads();
    // S = Q K^T for this thread's 4 x 4 block, the sum over d in order.
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < DP; ++d) {
      const float4 a = *reinterpret_cast<const float4 *>(&Qt[d * (kBQ + kPad) + 4 * ty]);
      const float4 b = *reinterpret_cast<const float4 *>(&Kt[d * (kBK + kPad) + 4 * tx]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(av[i], bv[j], s[i][j]);
    }
    // scale, mask, running max / sum per row (16 lanes share a row group)
    float p[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t qi = q0 + 4 * ty + i;
      float rmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t ki = k0 + 4 * tx + j;
        float sv = s[i][j] * scale;
        if (ki >= Lk || (causal && ki > qi)) sv = -INFINITY;
        s[i][j] = sv;
        rmax = fmaxf(rmax, sv);
      }
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
      const float m_new = fmaxf(m[i], rmax);
      // a row with no unmasked key yet keeps m = -inf: its weights are 0
      const float corr = (m_new == -INFINITY) ? 1.f : exp_mode<kFast>(m[i] - m_new);
      float rsum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        p[i][j] = (s[i][j] == -INFINITY) ? 0.f : exp_mode<kFast>(s[i][j] - m_new);
        rsum += p[i][j];
      }
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) rsum += __shfl_xor_sync(0xffffffffu, rsum, off);
      l[i] = l[i] * corr + rsum;
      m[i] = m_new;
#pragma unroll
      for (int jj = 0; jj < kOC; ++jj)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[i][jj][c] *= corr;
    }
    // P^T to shared memory: Pt[key][row]
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4 *>(&Pt[(4 * tx + j) * (kBQ + kPad) + 4 * ty]) =
          make_float4(p[0][j], p[1][j], p[2][j], p[3][j]);
    __syncthreads();
    // O += P V
#pragma unroll 4
    for (int kk = 0; kk < kBK; ++kk) {
      const float4 pr = *reinterpret_cast<const float4 *>(&Pt[kk * (kBQ + kPad) + 4 * ty]);
      const float pv[4] = {pr.x, pr.y, pr.z, pr.w};
#pragma unroll
      for (int jj = 0; jj < kOC; ++jj) {
        const float4 vv = *reinterpret_cast<const float4 *>(&Vs[kk * (DP + kPad) + 64 * jj + 4 * tx]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[i][jj][0] = fmaf(pv[i], vv.x, acc[i][jj][0]);
          acc[i][jj][1] = fmaf(pv[i], vv.y, acc[i][jj][1]);
          acc[i][jj][2] = fmaf(pv[i], vv.z, acc[i][jj][2]);
          acc[i][jj][3] = fmaf(pv[i], vv.w, acc[i][jj][3]);
        }
      }
    }
  }
  // O = init + acc / l
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t qi = q0 + 4 * ty + i;
    if (qi >= Lq || l[i] == 0.f) continue;  // no key (Lk = 0): O keeps its initial value
    const float inv = 1.f / l[i];
#pragma unroll
    for (int jj = 0; jj < kOC; ++jj) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int d = 64 * jj + 4 * tx + c;
        if (d < D) ob[qi * D + d] += acc[i][jj][c] * inv;
      }
    }
  }
}

// One warp per query row, for head dimensions above 256: scores in three
// passes over the keys (max, sum, weighted V) -- the reference's order.
template <bool kFast>
__global__ void attention_rows_kernel(const float *__restrict__ q, const float *__restrict__ k,
                                      const float *__restrict__ v, float *__restrict__ o, int64_t Lq, int64_t Lk,
                                      int D, float scale, int causal) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int64_t bh = blockIdx.y;
  pdl_launch_dependents();
  pdl_wait();
  if (row >= Lq) return;
  const float *qr = q + (bh * Lq + row) * D;
  const float *kb = k + bh * Lk * D;
  const float *vb = v + bh * Lk * D;
  float *orow = o + (bh * Lq + row) * D;
  const int64_t kn = causal ? (row + 1 < Lk ? row + 1 : Lk) : Lk;
  auto score = [&](int64_t j) {
    float s = 0.f;
    for (int d = lane; d < D; d += 32) s = fmaf(qr[d], kb[j * D + d], s);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    return s * scale;
  };
  float mx = -INFINITY;
  for (int64_t j = 0; j < kn; ++j) mx = fmaxf(mx, score(j));
  float den = 0.f;
  for (int64_t j = 0; j < kn; ++j) den += exp_mode<kFast>(score(j) - mx);
  if (den == 0.f) return;  // no key (Lk = 0): O keeps its initial value
  for (int d0 = 0; d0 < D; d0 += 32) {
    const int d = d0 + lane;
    float val = 0.f;
    for (int64_t j = 0; j < kn; ++j) {
      const float w = exp_mode<kFast>(score(j) - mx) / den;
      if (d < D) val = fmaf(w, vb[j * D + d], val);
    }
    if (d < D) orow[d] += val;
  }
}

// ---- double-buffered variant (D % 4 == 0): Q, K, V tiles row-major in
// shared memory, K / V tiles copied with cp.async 16-byte chunks two tiles
// ahead of use, so the next key tile streams in while this one computes.
// Thread layout as above, except that thread tx owns key columns tx + 16 j
// (j < 4): consecutive lanes read consecutive K rows, conflict-free.
__device__ __forceinline__ void cp_async16(float *smem_dst, const float *gsrc, bool in) {
  const uint32_t d = smem_u32(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gsrc), "r"(in ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int DP, bool kFast>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_db_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                        float *__restrict__ o, int64_t Lq, int64_t Lk, int D, float scale, int causal) {
  extern __shared__ __align__(16) float sm[];
  constexpr int kLd = DP + kPad;  // row stride of Q / K / V tiles
  float *Qs = sm;                              // [BQ][kLd]
  float *KV = Qs + kBQ * kLd;                  // 2 stages x ([BK][kLd] K, [BK][kLd] V)
  float *Pt = KV + 2 * 2 * kBK * kLd;          // [BK][BQ+pad]
  constexpr int kOC = DP / 64;
  constexpr int kChunks = DP / 4;              // 16-byte chunks per row

  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;
  int64_t bh, q0;
  tile_of_block(Lq, bh, q0);
  const float *qb = q + bh * Lq * D;
  const float *kb = k + bh * Lk * D;
  const float *vb = v + bh * Lk * D;
  float *ob = o + bh * Lq * D;

  int64_t k_end = Lk;
  if (causal) {
    const int64_t last_q = (q0 + kBQ - 1 < Lq - 1 ? q0 + kBQ - 1 : Lq - 1);
    k_end = last_q + 1 < Lk ? last_q + 1 : Lk;
  }
  const int n_tiles = static_cast<int>((k_end + kBK - 1) / kBK);

  // chunk (row, c) of a tile: rows past the end / chunks past D read as zero
  auto load_rows = [&](float *dst, const float *src, int64_t row0, int64_t nrows) {
    for (int e = tid; e < kBK * kChunks; e += kAttnThreads) {
      const int r = e / kChunks, c = e % kChunks;
      const bool in = row0 + r < nrows && 4 * c < D;
      const float *g = in ? src + (row0 + r) * D + 4 * c : src;
      cp_async16(dst + r * kLd + 4 * c, g, in);
    }
  };
  auto load_tile = [&](int t) {
    float *Ks = KV + (t & 1) * 2 * kBK * kLd;
    load_rows(Ks, kb, static_cast<int64_t>(t) * kBK, Lk);
    load_rows(Ks + kBK * kLd, vb, static_cast<int64_t>(t) * kBK, Lk);
  };

  pdl_launch_dependents();
  pdl_wait();
  load_rows(Qs, qb, q0, Lq);
  if (n_tiles > 0) load_tile(0);
  cp_async_commit();

  float m[4], l[4], acc[4][kOC][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kOC; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[i][j][c] = 0.f;
  }

  for (int t = 0; t < n_tiles; ++t) {
    // issue tile t+1 (its buffer was last read by tile t-1, finished at the
    // barrier that ended iteration t-1), then wait for tile t
    if (t + 1 < n_tiles) load_tile(t + 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const float *Ks = KV + (t & 1) * 2 * kBK * kLd;
    const float *Vs = Ks + kBK * kLd;
    const int64_t k0 = static_cast<int64_t>(t) * kBK;
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
    // operands of step d + 4 are loaded while step d computes (registers
    // double-buffered: the shared-memory latency overlaps the FMAs)
    float4 a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4 *>(&Qs[(4 * ty + i) * kLd]);
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4 *>(&Ks[(tx + 16 * j) * kLd]);
#pragma unroll 4
    for (int d = 0; d < DP; d += 4) {
      float4 an[4], bn[4];
      const int dn = d + 4 < DP ? d + 4 : d;
#pragma unroll
      for (int i = 0; i < 4; ++i) an[i] = *reinterpret_cast<const float4 *>(&Qs[(4 * ty + i) * kLd + dn]);
#pragma unroll
      for (int j = 0; j < 4; ++j) bn[j] = *reinterpret_cast<const float4 *>(&Ks[(tx + 16 * j) * kLd + dn]);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(a[i].x, b[j].x, s[i][j]);
          s[i][j] = fmaf(a[i].y, b[j].y, s[i][j]);
          s[i][j] = fmaf(a[i].z, b[j].z, s[i][j]);
          s[i][j] = fmaf(a[i].w, b[j].w, s[i][j]);
        }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = an[i];
        b[i] = bn[i];
      }
    }
    float p[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t qi = q0 + 4 * ty + i;
      float rmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t ki = k0 + tx + 16 * j;
        float sv = s[i][j] * scale;
        if (ki >= Lk || (causal && ki > qi)) sv = -INFINITY;
        s[i][j] = sv;
        rmax = fmaxf(rmax, sv);
      }
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
      const float m_new = fmaxf(m[i], rmax);
      const float corr = (m_new == -INFINITY) ? 1.f : exp_mode<kFast>(m[i] - m_new);
      float rsum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        p[i][j] = (s[i][j] == -INFINITY) ? 0.f : exp_mode<kFast>(s[i][j] - m_new);
        rsum += p[i][j];
      }
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) rsum += __shfl_xor_sync(0xffffffffu, rsum, off);
      l[i] = l[i] * corr + rsum;
      m[i] = m_new;
#pragma unroll
      for (int jj = 0; jj < kOC; ++jj)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[i][jj][c] *= corr;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4 *>(&Pt[(tx + 16 * j) * (kBQ + kPad) + 4 * ty]) =
          make_float4(p[0][j], p[1][j], p[2][j], p[3][j]);
    __syncthreads();
    float4 pr = *reinterpret_cast<const float4 *>(&Pt[4 * ty]);
    float4 vr[kOC];
#pragma unroll
    for (int jj = 0; jj < kOC; ++jj) vr[jj] = *reinterpret_cast<const float4 *>(&Vs[64 * jj + 4 * tx]);
#pragma unroll 8
    for (int kk = 0; kk < kBK; ++kk) {
      const int kn = kk + 1 < kBK ? kk + 1 : kk;
      const float4 prn = *reinterpret_cast<const float4 *>(&Pt[kn * (kBQ + kPad) + 4 * ty]);
      float4 vrn[kOC];
#pragma unroll
      for (int jj = 0; jj < kOC; ++jj) vrn[jj] = *reinterpret_cast<const float4 *>(&Vs[kn * kLd + 64 * jj + 4 * tx]);
      const float pv[4] = {pr.x, pr.y, pr.z, pr.w};
#pragma unroll
      for (int jj = 0; jj < kOC; ++jj) {
        const float4 vv = vr[jj];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[i][jj][0] = fmaf(pv[i], vv.x, acc[i][jj][0]);
          acc[i][jj][1] = fmaf(pv[i], vv.y, acc[i][jj][1]);
          acc[i][jj][2] = fmaf(pv[i], vv.z, acc[i][jj][2]);
          acc[i][jj][3] = fmaf(pv[i], vv.w, acc[i][jj][3]);
        }
      }
      pr = prn;
#pragma unroll
      for (int jj = 0; jj < kOC; ++jj) vr[jj] = vrn[jj];
    }
    __syncthreads();  // Pt and this stage's K / V are free for the next loads
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t qi = q0 + 4 * ty + i;
    if (qi >= Lq || l[i] == 0.f) continue;  // no key (Lk = 0): O keeps its initial value
    const float inv = 1.f / l[i];
#pragma unroll
    for (int jj = 0; jj < kOC; ++jj) {
      const int d = 64 * jj + 4 * tx;
      if (d < D) {
        float4 *dst = reinterpret_cast<float4 *>(ob + qi * D + d);
        float4 cur = *dst;
        cur.x += acc[i][jj][0] * inv;
        cur.y += acc[i][jj][1] * inv;
        cur.z += acc[i][jj][2] * inv;
        cur.w += acc[i][jj][3] * inv;
        *dst = cur;
      }
    }
  }
}

template <int DP>
int attention_db_smem_bytes() {
  return ((kBQ + 4 * kBK) * (DP + kPad) + kBK * (kBQ + kPad)) * static_cast<int>(sizeof(float));
}

template <int DP>
int attention_smem_bytes() {
  return (DP * (kBQ + kPad) + DP * (kBK + kPad) + kBK * (DP + kPad) + kBK * (kBQ + kPad)) *
         static_cast<int>(sizeof(float));
}

template <int DP, bool kFast>
cudaError_t launch_attention_dp(const float *q, const float *k, const float *v, float *o, int64_t BH, int64_t Lq,
                                int64_t Lk, int D, float scale, int causal, cudaStream_t stream) {
  // rows of 16-byte chunks (D % 4 == 0, 16-byte aligned tensors): the
  // double-buffered kernel; otherwise the synchronous one
  const bool db = (D % 4) == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(k) & 15) == 0 && (reinterpret_cast<uintptr_t>(v) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(o) & 15) == 0;
  auto kern = db ? attention_db_kernel<DP, kFast> : attention_kernel<DP, kFast>;
  const int smem = db ? attention_db_smem_bytes<DP>() : attention_smem_bytes<DP>();
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(static_cast<unsigned>((Lq + kBQ - 1) / kBQ * BH));  // see tile_of_block
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, q, k, v, o, Lq, Lk, D, scale, causal);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <bool kFast>
cudaError_t launch_attention_mode(const float *q, const float *k, const float *v, float *o, int64_t BH, int64_t Lq,
                                  int64_t Lk, int D, float scale, int causal, cudaStream_t stream) {
  if (D <= 64) return launch_attention_dp<64, kFast>(q, k, v, o, BH, Lq, Lk, D, scale, causal, stream);
  if (D <= 128) return launch_attention_dp<128, kFast>(q, k, v, o, BH, Lq, Lk, D, scale, causal, stream);
  const dim3 block(256);
  const dim3 grid(static_cast<unsigned>((Lq + 7) / 8), static_cast<unsigned>(BH));
  attention_rows_kernel<kFast><<<grid, block, 0, stream>>>(q, k, v, o, Lq, Lk, D, scale, causal);
  return cudaGetLastError();
}

}  // namespace

bool rope_supported(int64_t B, int64_t H, int64_t L, int64_t D) {
  return B >= 0 && H >= 0 && L >= 0 && D >= 2 && D % 2 == 0 && D <= (int64_t(1) << 20);
}

size_t rope_table_bytes(int64_t L, int64_t D) { return static_cast<size_t>(L) * static_cast<size_t>(D / 2) * 8; }

cudaError_t rope_launch(const float *x, const int64_t *pos, float *y, int64_t B, int64_t H, int64_t L, int64_t D,
                        double theta, int fast_math, void *table, int sm_count, cudaStream_t stream) {
  if (B == 0 || H == 0 || L == 0) return cudaSuccess;
  if (!rope_supported(B, H, L, D)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(kRopeThreads);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int64_t pairs = L * (D / 2);
  int64_t tb = (pairs + kRopeThreads - 1) / kRopeThreads;
  cfg.gridDim = dim3(static_cast<unsigned>(tb < 4 * sm_count ? tb : 4 * sm_count));
  float2 *tab = static_cast<float2 *>(table);
  cudaError_t e = fast_math ? cudaLaunchKernelEx(&cfg, rope_table_kernel<true>, pos, tab, L, static_cast<int>(D), theta)
                            : cudaLaunchKernelEx(&cfg, rope_table_kernel<false>, pos, tab, L, static_cast<int>(D),
                                                 theta);
  if (e != cudaSuccess) return e;
  // Streaming: 8 CTAs of 256 threads per SM, grid-stride.
  const int64_t n = B * H * L * D;
  if ((D & 3) == 0) {
    const int64_t n4 = n / 4;
    const int64_t need = (n4 + kRopeThreads * kUnroll - 1) / (kRopeThreads * kUnroll);
    cfg.gridDim = dim3(static_cast<unsigned>(need < 8 * sm_count ? need : 8 * sm_count));
    e = cudaLaunchKernelEx(&cfg, rope_apply4_kernel, reinterpret_cast<const float4 *>(x),
                           reinterpret_cast<const float4 *>(table), reinterpret_cast<float4 *>(y), n4, L,
                           static_cast<int>(D));
  } else {
    const int64_t n2 = n / 2;
    const int64_t need = (n2 + kRopeThreads - 1) / kRopeThreads;
    cfg.gridDim = dim3(static_cast<unsigned>(need < 8 * sm_count ? need : 8 * sm_count));
    e = cudaLaunchKernelEx(&cfg, rope_apply2_kernel, reinterpret_cast<const float2 *>(x),
                           reinterpret_cast<const float2 *>(table), reinterpret_cast<float2 *>(y), n2, L,
                           static_cast<int>(D));
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

bool attention_supported(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D) {
  // grid: (Lq / 64) x B x H CTAs in one dimension (D <= 128), or (Lq / 8)
  // x (B x H) in two
  return B >= 0 && H >= 0 && Lq >= 0 && Lk >= 0 && D >= 1 && D <= 4096 && B * H <= 65535 &&
         (Lq + 63) / 64 * B * H <= INT32_MAX && (Lq + 7) / 8 <= INT32_MAX;
}

cudaError_t attention_launch(const float *q, const float *k, const float *v, float *o, int64_t B, int64_t H,
                             int64_t Lq, int64_t Lk, int64_t D, float scale, int causal, int fast_math,
                             cudaStream_t stream) {
  if (B == 0 || H == 0 || Lq == 0) return cudaSuccess;
  if (!attention_supported(B, H, Lq, Lk, D)) return cudaErrorInvalidValue;
  return fast_math ? launch_attention_mode<true>(q, k, v, o, B * H, Lq, Lk, static_cast<int>(D), scale, causal, stream)
                   : launch_attention_mode<false>(q, k, v, o, B * H, Lq, Lk, static_cast<int>(D), scale, causal,
                                                  stream);
}

}  // namespace llk_b200
