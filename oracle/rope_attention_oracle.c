/*
 * rope_attention_oracle.c -- CPU restatement of the reference's llk.rope and
 * llk.attention ops.  TEST INFRASTRUCTURE ONLY: the checker of the GPU
 * kernels, never part of the product.  Compiled with -ffp-contract=off so
 * every f32 product and sum is rounded on its own, as the MLIR arith ops are.
 *
 *   oracle_rope_f32        the LLKToLinalg lowering of llk.rope
 *                          (lib/Conversion/LLKToLinalg/LLKToLinalg.cpp:162-324):
 *                          freq = pow(theta, (-2 i) / D) and angle = pos * freq
 *                          in f64, cos / sin of the angle rounded to f32,
 *                          then even*c - odd*s and odd*c + even*s in f32;
 *   oracle_rope_fp64       the FP64 reference of test/Execution/rope_correctness.cpp:14-35;
 *   oracle_attention_f32   the lowering of llk.attention (LLKToLinalg.cpp:330-608):
 *                          S = sum_d q*k (f32, in d order), S*scale, causal
 *                          -inf where k > q, row max, sum of exp(s - max),
 *                          w = exp(s - max) / sum, O = init + sum_k w*v (in k order);
 *   oracle_attention_fp64  the FP64 reference of test/Execution/attention_correctness.cpp:15-60.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

void oracle_rope_f32(const float *x, const int64_t *pos, float *y, int64_t B, int64_t H, int64_t L, int64_t D,
                     double theta) {
  const int64_t half = D / 2;
  float *cs = (float *)malloc(sizeof(float) * 2 * (size_t)(L * half > 0 ? L * half : 1));
  for (int64_t p = 0; p < L; ++p) {
    for (int64_t i = 0; i < half; ++i) {
      const double freq = pow(theta, (-2.0 * (double)i) / (double)D);
      const double angle = (double)pos[p] * freq;
      const float a = (float)angle;
      cs[2 * (p * half + i)] = cosf(a);
      cs[2 * (p * half + i) + 1] = sinf(a);
    }
  }
  for (int64_t bh = 0; bh < B * H; ++bh) {
    for (int64_t p = 0; p < L; ++p) {
      const float *xr = x + (bh * L + p) * D;
      float *yr = y + (bh * L + p) * D;
      for (int64_t i = 0; i < half; ++i) {
        const float c = cs[2 * (p * half + i)], s = cs[2 * (p * half + i) + 1];
        const float e = xr[2 * i], o = xr[2 * i + 1];
        const float t1 = e * c, t2 = o * s, t3 = o * c, t4 = e * s;
        yr[2 * i] = t1 - t2;
        yr[2 * i + 1] = t3 + t4;
      }
    }
  }
  free(cs);
}

void oracle_rope_fp64(const double *x, const int64_t *pos, double *y, int64_t B, int64_t H, int64_t L, int64_t D,
                      double theta) {
  for (int64_t bh = 0; bh < B * H; ++bh) {
    for (int64_t p = 0; p < L; ++p) {
      for (int64_t i = 0; i < D / 2; ++i) {
        const double freq = pow(theta, -2.0 * (double)i / (double)D);
        const double angle = (double)pos[p] * freq;
        const double c = cos(angle), s = sin(angle);
        const int64_t base = (bh * L + p) * D;
        const double e = x[base + 2 * i], o = x[base + 2 * i + 1];
        y[base + 2 * i] = e * c - o * s;
        y[base + 2 * i + 1] = o * c + e * s;
      }
    }
  }
}

void oracle_attention_f32(const float *q, const float *k, const float *v, float *o, int64_t B, int64_t H, int64_t Lq,
                          int64_t Lk, int64_t D, float scale, int causal) {
  float *s = (float *)malloc(sizeof(float) * (size_t)(Lk > 0 ? Lk : 1));
  for (int64_t bh = 0; bh < B * H; ++bh) {
    for (int64_t i = 0; i < Lq; ++i) {
      const float *qr = q + (bh * Lq + i) * D;
      float mx = -INFINITY;
      for (int64_t j = 0; j < Lk; ++j) {
        const float *kr = k + (bh * Lk + j) * D;
        float acc = 0.0f;
        for (int64_t d = 0; d < D; ++d) {
          const float prod = qr[d] * kr[d];
          acc = prod + acc;
        }
        float sv = acc * scale;
        if (causal && j > i) sv = -INFINITY;
        s[j] = sv;
        mx = fmaxf(sv, mx);
      }
      float den = 0.0f;
      for (int64_t j = 0; j < Lk; ++j) den = expf(s[j] - mx) + den;
      float *orow = o + (bh * Lq + i) * D;
      for (int64_t j = 0; j < Lk; ++j) {
        const float w = expf(s[j] - mx) / den;
        const float *vr = v + (bh * Lk + j) * D;
        for (int64_t d = 0; d < D; ++d) {
          const float prod = w * vr[d];
          orow[d] = prod + orow[d];
        }
      }
    }
  }
  free(s);
}

void oracle_attention_fp64(const double *q, const double *k, const double *v, double *o, int64_t B, int64_t H,
                           int64_t Lq, int64_t Lk, int64_t D, double scale, int causal) {
  double *sc = (double *)malloc(sizeof(double) * (size_t)(Lk > 0 ? Lk : 1));
  for (int64_t bh = 0; bh < B * H; ++bh) {
    for (int64_t i = 0; i < Lq; ++i) {
      double mx = -INFINITY;
      for (int64_t j = 0; j < Lk; ++j) {
        double dot = 0.0;
        for (int64_t d = 0; d < D; ++d) dot += q[(bh * Lq + i) * D + d] * k[(bh * Lk + j) * D + d];
        dot *= scale;
        if (causal && j > i) dot = -INFINITY;
        sc[j] = dot;
        if (dot > mx) mx = dot;
      }
      double sum = 0.0;
      for (int64_t j = 0; j < Lk; ++j) {
        sc[j] = (causal && j > i) ? 0.0 : exp(sc[j] - mx);
        sum += sc[j];
      }
      for (int64_t d = 0; d < D; ++d) {
        double val = 0.0;
        for (int64_t j = 0; j < Lk; ++j) val += (sc[j] / sum) * v[(bh * Lk + j) * D + d];
        o[(bh * Lq + i) * D + d] = val;
      }
    }
  }
  free(sc);
}
