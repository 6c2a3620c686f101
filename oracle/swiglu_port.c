/*
 * swiglu_port.c -- multi-threaded CPU restatement of the reference's fused
 * SwiGLU schedule, used only as the timed CPU baseline and as a fast checker
 * for shapes the scalar oracle cannot finish in seconds.  TEST/BENCH
 * INFRASTRUCTURE ONLY: never linked into the product library.
 *
 * What it restates:
 *   - the fused semantics of lib/Transforms/FuseDoubleContraction.cpp:119-199
 *     (one pass over K, two f32 accumulators, epilogue g*sigmoid(g)*u);
 *   - the tiling of lib/Transforms/TileAndVectorize.cpp:53-57 and the
 *     bucket-4 entry of schedules/schedule_db.json (BM=32, BN=64, BK=64),
 *     with M x N tiles handed out by an atomic counter the way
 *     runtime/ThreadPool.cpp:48-63 hands out parallelFor tiles.
 * The K loop walks k in ascending order for every output element, so the
 * f32 accumulation order matches the scalar oracle; with FMA contraction
 * enabled (as the reference's AVX2 JIT uses) results agree to rounding.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define PORT_BM 32
#define PORT_BN 64
#define PORT_BK 64

static inline float bf2f(uint16_t h) {
  union { uint32_t u; float f; } v;
  v.u = (uint32_t)h << 16;
  return v.f;
}

static inline uint16_t f2bf(float f) {
  union { uint32_t u; float f; } v;
  v.f = f;
  v.u += 0x8000u + ((v.u >> 16) & 1u);
  return (uint16_t)(v.u >> 16);
}

typedef struct {
  const uint16_t *x, *wg, *wu;
  int64_t ldx, ldw, ldy, M, N, K;
  float *y_f32;
  uint16_t *y_bf16;
  int mode; /* 0 = swiglu, 1 = matmul (wg only, y = acc) */
  atomic_long next;
  int64_t tiles_n, tiles_total;
} port_job;

static void run_tile(port_job *j, int64_t t) {
  int64_t m0 = (t / j->tiles_n) * PORT_BM, n0 = (t % j->tiles_n) * PORT_BN;
  int64_t bm = j->M - m0 < PORT_BM ? j->M - m0 : PORT_BM;
  int64_t bn = j->N - n0 < PORT_BN ? j->N - n0 : PORT_BN;
  float g[PORT_BM][PORT_BN], u[PORT_BM][PORT_BN];
  float wgf[PORT_BK][PORT_BN], wuf[PORT_BK][PORT_BN];
  memset(g, 0, sizeof g);
  memset(u, 0, sizeof u);
  for (int64_t k0 = 0; k0 < j->K; k0 += PORT_BK) {
    int64_t bk = j->K - k0 < PORT_BK ? j->K - k0 : PORT_BK;
    for (int64_t kk = 0; kk < bk; kk++) {
      const uint16_t *rg = j->wg + (k0 + kk) * j->ldw + n0;
      for (int64_t nn = 0; nn < bn; nn++) wgf[kk][nn] = bf2f(rg[nn]);
      for (int64_t nn = bn; nn < PORT_BN; nn++) wgf[kk][nn] = 0.0f;
      if (j->mode == 0) {
        const uint16_t *ru = j->wu + (k0 + kk) * j->ldw + n0;
        for (int64_t nn = 0; nn < bn; nn++) wuf[kk][nn] = bf2f(ru[nn]);
        for (int64_t nn = bn; nn < PORT_BN; nn++) wuf[kk][nn] = 0.0f;
      }
    }
    for (int64_t mm = 0; mm < bm; mm++) {
      const uint16_t *xr = j->x + (m0 + mm) * j->ldx + k0;
      float *gr = g[mm], *ur = u[mm];
      for (int64_t kk = 0; kk < bk; kk++) {
        float xv = bf2f(xr[kk]);
        const float *a = wgf[kk], *b = wuf[kk];
        for (int nn = 0; nn < PORT_BN; nn++) gr[nn] += xv * a[nn];
        if (j->mode == 0)
          for (int nn = 0; nn < PORT_BN; nn++) ur[nn] += xv * b[nn];
      }
    }
  }
  for (int64_t mm = 0; mm < bm; mm++)
    for (int64_t nn = 0; nn < bn; nn++) {
      float r;
      if (j->mode == 0) {
        float sig = 1.0f / (1.0f + expf(-g[mm][nn]));
        r = (g[mm][nn] * sig) * u[mm][nn];
      } else {
        r = g[mm][nn];
      }
      int64_t o = (m0 + mm) * j->ldy + n0 + nn;
      if (j->y_f32) j->y_f32[o] = r;
      if (j->y_bf16) j->y_bf16[o] = f2bf(r);
    }
}

static void *worker(void *arg) {
  port_job *j = (port_job *)arg;
  for (;;) {
    long t = atomic_fetch_add(&j->next, 1);
    if (t >= j->tiles_total) break;
    run_tile(j, t);
  }
  return NULL;
}

static int run_job(port_job *j, int threads) {
  j->tiles_n = (j->N + PORT_BN - 1) / PORT_BN;
  j->tiles_total = ((j->M + PORT_BM - 1) / PORT_BM) * j->tiles_n;
  atomic_init(&j->next, 0);
  if (threads < 1) threads = 1;
  pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
  int started = 0;
  for (int i = 1; i < threads; i++)
    if (pthread_create(&tids[i], NULL, worker, j) == 0) started++;
    else break;
  worker(j); /* the caller participates, as ThreadPool::parallelFor does */
  for (int i = 1; i <= started; i++) pthread_join(tids[i], NULL);
  free(tids);
  return 0;
}

/* Fused SwiGLU on bf16 inputs; y as f32 and/or bf16 (row stride ldy). */
int port_swiglu(const uint16_t *x, int64_t ldx, const uint16_t *wg,
                const uint16_t *wu, int64_t ldw, int64_t M, int64_t N,
                int64_t K, float *y_f32, uint16_t *y_bf16, int64_t ldy,
                int threads) {
  port_job j;
  memset(&j, 0, sizeof j);
  j.x = x; j.wg = wg; j.wu = wu; j.ldx = ldx; j.ldw = ldw; j.ldy = ldy;
  j.M = M; j.N = N; j.K = K; j.y_f32 = y_f32; j.y_bf16 = y_bf16; j.mode = 0;
  return run_job(&j, threads);
}

/* C[M,N] (f32) = A[M,K] * B[K,N], bf16 operands. */
int port_matmul(const uint16_t *a, int64_t lda, const uint16_t *b, int64_t ldb,
                float *c, int64_t ldc, int64_t M, int64_t N, int64_t K,
                int threads) {
  port_job j;
  memset(&j, 0, sizeof j);
  j.x = a; j.wg = b; j.wu = b; j.ldx = lda; j.ldw = ldb; j.ldy = ldc;
  j.M = M; j.N = N; j.K = K; j.y_f32 = c; j.mode = 1;
  return run_job(&j, threads);
}
