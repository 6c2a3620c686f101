/*
 * swiglu_oracle.c -- CPU restatement of DSLCompiler's fused SwiGLU and
 * matmul arithmetic.  TEST INFRASTRUCTURE ONLY: the checker that the CUDA
 * path is compared against.  Nothing in the product (the dslcompiler_b200
 * package and its shared library) links, loads or calls this file.
 *
 * Built with -ffp-contract=off so every multiply and add rounds separately,
 * in the same order as the reference's scalar C++ loops; the functions that
 * restate those loops are bit-exact against the reference compiled from its
 * own sources (oracle/_ref, see oracle/Makefile).
 *
 * Reference citations are paths inside the DSLCompiler project.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* bf16 <-> f32, round-to-nearest-even.
 * Follows test/Execution/swiglu_reference.cpp:19-32 (bits += 0x8000 + lsb). */
float oracle_bf16_to_f32(uint16_t h) {
  uint32_t bits = (uint32_t)h << 16;
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

uint16_t oracle_f32_to_bf16(float f) {
  uint32_t bits;
  memcpy(&bits, &f, sizeof bits);
  bits += 0x8000u + ((bits >> 16) & 1u);
  return (uint16_t)(bits >> 16);
}

void oracle_f32_to_bf16_array(const float *src, uint16_t *dst, int64_t n) {
  for (int64_t i = 0; i < n; i++) dst[i] = oracle_f32_to_bf16(src[i]);
}

void oracle_bf16_to_f32_array(const uint16_t *src, float *dst, int64_t n) {
  for (int64_t i = 0; i < n; i++) dst[i] = oracle_bf16_to_f32(src[i]);
}

/* Naive FP32 SwiGLU exactly as the reference's test oracle computes it:
 * gate and up as separate k-ordered f32 dot products, then
 * silu = g / (1 + exp(-g)), y = silu * up.
 * Follows test/Execution/swiglu_reference.cpp:38-71. */
void oracle_swiglu_naive_f32(const float *x, const float *wg, const float *wu,
                             float *y, int64_t M, int64_t N, int64_t K) {
  for (int64_t m = 0; m < M; m++) {
    for (int64_t n = 0; n < N; n++) {
      float sg = 0.0f, su = 0.0f;
      for (int64_t k = 0; k < K; k++) sg += x[m * K + k] * wg[k * N + n];
      for (int64_t k = 0; k < K; k++) su += x[m * K + k] * wu[k * N + n];
      float silu = sg / (1.0f + expf(-sg));
      y[m * N + n] = silu * su;
    }
  }
}

/* FP64 ground truth.  Follows test/Execution/swiglu_reference.cpp:77-99. */
void oracle_swiglu_fp64(const double *x, const double *wg, const double *wu,
                        double *y, int64_t M, int64_t N, int64_t K) {
  for (int64_t m = 0; m < M; m++) {
    for (int64_t n = 0; n < N; n++) {
      double sg = 0.0, su = 0.0;
      for (int64_t k = 0; k < K; k++) {
        sg += x[m * K + k] * wg[k * N + n];
        su += x[m * K + k] * wu[k * N + n];
      }
      double silu = sg / (1.0 + exp(-sg));
      y[m * N + n] = silu * su;
    }
  }
}

/* FP64 SwiGLU on bf16 inputs with arbitrary row strides (elements), for
 * the error reference at sampled points of large shapes: computes only the
 * (row, col) pairs listed.  Same math as oracle_swiglu_fp64. */
void oracle_swiglu_fp64_points(const uint16_t *x, int64_t ldx,
                               const uint16_t *wg, const uint16_t *wu,
                               int64_t ldw, int64_t K, const int64_t *rows,
                               const int64_t *cols, int64_t npts,
                               double *out) {
  for (int64_t p = 0; p < npts; p++) {
    int64_t m = rows[p], n = cols[p];
    double sg = 0.0, su = 0.0;
    for (int64_t k = 0; k < K; k++) {
      double xv = oracle_bf16_to_f32(x[m * ldx + k]);
      sg += xv * oracle_bf16_to_f32(wg[k * ldw + n]);
      su += xv * oracle_bf16_to_f32(wu[k * ldw + n]);
    }
    out[p] = sg / (1.0 + exp(-sg)) * su;
  }
}

/* The production (fused) semantics: one pass over K with two f32
 * accumulators g += f32(x)*f32(wg), u += f32(x)*f32(wu), then the epilogue
 * sigmoid = 1/(1+exp(-g)), silu = g*sigmoid, r = silu*u, optionally
 * truncated to bf16 (RNE).
 * Follows lib/Transforms/FuseDoubleContraction.cpp:119-173 (accumulation)
 * and :179-199 (epilogue).
 * Inputs are bf16 bit patterns with row strides in elements; the output is
 * written as f32 (y_f32 != NULL) and/or bf16 (y_bf16 != NULL). */
void oracle_swiglu_fused(const uint16_t *x, int64_t ldx, const uint16_t *wg,
                         const uint16_t *wu, int64_t ldw, int64_t M, int64_t N,
                         int64_t K, float *y_f32, uint16_t *y_bf16,
                         int64_t ldy) {
  float *g = (float *)calloc((size_t)(N > 0 ? N : 1), sizeof(float));
  float *u = (float *)calloc((size_t)(N > 0 ? N : 1), sizeof(float));
  for (int64_t m = 0; m < M; m++) {
    memset(g, 0, sizeof(float) * (size_t)N);
    memset(u, 0, sizeof(float) * (size_t)N);
    for (int64_t k = 0; k < K; k++) {
      float xv = oracle_bf16_to_f32(x[m * ldx + k]);
      const uint16_t *rg = wg + k * ldw, *ru = wu + k * ldw;
      for (int64_t n = 0; n < N; n++) {
        g[n] = g[n] + xv * oracle_bf16_to_f32(rg[n]);
        u[n] = u[n] + xv * oracle_bf16_to_f32(ru[n]);
      }
    }
    for (int64_t n = 0; n < N; n++) {
      float sig = 1.0f / (1.0f + expf(-g[n]));
      float r = (g[n] * sig) * u[n];
      if (y_f32) y_f32[m * ldy + n] = r;
      if (y_bf16) y_bf16[m * ldy + n] = oracle_f32_to_bf16(r);
    }
  }
  free(g);
  free(u);
}

/* C = A * B with bf16 operands, f32 k-ordered accumulation and f32 output:
 * the contract of micro.mma (acc += lhs x rhs, lhs [M,K], rhs [K,N]) as
 * verified in lib/Dialect/Micro/MicroOps.cpp:246-291, with the linalg.matmul
 * accumulation of lib/Conversion/LLKToLinalg/LLKToLinalg.cpp:104-116.
 * c is read as the initial accumulator when accumulate != 0. */
void oracle_matmul(const uint16_t *a, int64_t lda, const uint16_t *b,
                   int64_t ldb, float *c, int64_t ldc, int64_t M, int64_t N,
                   int64_t K, int accumulate) {
  float *acc = (float *)calloc((size_t)(N > 0 ? N : 1), sizeof(float));
  for (int64_t m = 0; m < M; m++) {
    for (int64_t n = 0; n < N; n++) acc[n] = accumulate ? c[m * ldc + n] : 0.0f;
    for (int64_t k = 0; k < K; k++) {
      float av = oracle_bf16_to_f32(a[m * lda + k]);
      const uint16_t *rb = b + k * ldb;
      for (int64_t n = 0; n < N; n++) acc[n] = acc[n] + av * oracle_bf16_to_f32(rb[n]);
    }
    for (int64_t n = 0; n < N; n++) c[m * ldc + n] = acc[n];
  }
  free(acc);
}

/* Block-major weight packing: for each k-block of BK rows, BK full-N rows,
 * zero-padded past K.  Follows runtime/PackedWeights.cpp:5-33 (bf16 only). */
void oracle_pack_weights_kblock(const uint16_t *w, int64_t K, int64_t N,
                                int64_t ldw, int64_t BK, uint16_t *out) {
  int64_t kblocks = (K + BK - 1) / BK;
  memset(out, 0, sizeof(uint16_t) * (size_t)(kblocks * BK * N));
  for (int64_t k = 0; k < K; k++)
    memcpy(out + k * N, w + k * ldw, sizeof(uint16_t) * (size_t)N);
}

/* BKxBN tile-major packing (tiles ordered k-block major, then n-block;
 * row-major inside a tile, zero-padded).
 * Follows test/Execution/packed_vs_unpacked.cpp:31-51. */
void oracle_pack_weights_tiled(const float *w, int64_t K, int64_t N,
                               int64_t BK, int64_t BN, float *out) {
  int64_t kb_n = (K + BK - 1) / BK, nb_n = (N + BN - 1) / BN;
  for (int64_t kb = 0; kb < kb_n; kb++)
    for (int64_t nb = 0; nb < nb_n; nb++)
      for (int64_t ko = 0; ko < BK; ko++)
        for (int64_t no = 0; no < BN; no++) {
          int64_t k = kb * BK + ko, n = nb * BN + no;
          out[(kb * nb_n + nb) * BK * BN + ko * BN + no] =
              (k < K && n < N) ? w[k * N + n] : 0.0f;
        }
}

/* M-bucket classifier: {1}, [2,4], [5,16], [17,64], >=65.
 * Follows lib/Transforms/Common/ScheduleLoader.cpp:19-29. */
int oracle_classify_m(int64_t M) {
  if (M == 1) return 0;
  if (M <= 4) return 1;
  if (M <= 16) return 2;
  if (M <= 64) return 3;
  return 4;
}
