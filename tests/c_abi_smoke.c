/* Compiled and linked as plain C11 by tests/test_capi.py (and run there when
 * a GPU is present): the header is valid C, every entry point links, and a
 * host-buffer llk_swiglu call works from C with the reference's struct
 * layouts.  Prints "ok <status>" and exits 0 when the call returns. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "llk_b200.h"

int main(void) {
  enum { M = 64, K = 256, N = 512 };
  static uint16_t x[M * K], wg[K * N], wu[K * N], y[M * N];
  /* bf16 0.0625 and 0.125 */
  for (int i = 0; i < M * K; ++i) x[i] = 0x3D80;
  for (int i = 0; i < K * N; ++i) wg[i] = wu[i] = 0x3E00;
  Tensor2D tx = {x, M, K, K, 1}, tg = {wg, K, N, N, 1}, tu = {wu, K, N, N, 1}, ty = {y, M, N, N, 1};
  KernelContext ctx;
  memset(&ctx, 0, sizeof ctx);
  llk_swiglu(&tx, &tg, &tu, &ty, &ctx);
  int st = llk_last_status();
  if (sizeof(Tensor2D) != 40 || sizeof(MemRef2D) != 56 || sizeof(KernelContext) != 16) return 3;
  printf("ok %d %s y0=0x%04x\n", st, llk_status_string(st), (unsigned)y[0]);
  /* g = u = 256 * 0.0625 * 0.125 = 2, y = 2 / (1 + e^-2) * 2 = 3.523 -> bf16 0x4061 */
  if (st == LLK_OK && y[0] != 0x4061) return 2;
  return st == LLK_OK || st == LLK_ERR_DEVICE ? 0 : 1;
}
