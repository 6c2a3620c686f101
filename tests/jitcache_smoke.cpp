// Compiled and linked as C++17 by tests/test_capi.py: the JitCache-shaped
// header over the C ABI.  Without a GPU it exercises the plan levels and the
// L4 miss path; with one (argv[1] == "gpu") it also packs a pair, inserts it,
// looks it up, evicts it while a reference is held and runs the packed op.
// Prints "ok" and exits 0 on success; a failing check exits with its line.
#include <cstdio>
#include <cstring>
#include <vector>

#include "llk_b200_jitcache.hpp"

#define CHECK(c)                                    \
  do {                                              \
    if (!(c)) {                                     \
      std::printf("fail line %d: %s\n", __LINE__, #c); \
      return __LINE__;                              \
    }                                               \
  } while (0)

int main(int argc, char **argv) {
  const bool gpu = argc > 1 && std::strcmp(argv[1], "gpu") == 0;
  llk_b200::JitCache cache;
  cache.clear();
  const llk_kernel_key key = llk_b200::make_kernel_key(LLK_OP_FUSED_SWIGLU, 4, 11008, 4096);
  CHECK(!cache.lookupObjectCode(key));                  // L3 miss
  auto plan = cache.lookupOrCompile(key, 2048);         // built and cached
  CHECK(plan && plan->variant == LLK_VARIANT_TC && plan->block_m == 256);
  auto again = cache.lookupObjectCode(key);             // L3 hit
  CHECK(again && std::memcmp(&*again, &*plan, sizeof(*plan)) == 0);
  llk_launch_plan tuned = *plan;
  tuned.sched = 0;
  CHECK(cache.insertObjectCode(key, tuned));
  CHECK(cache.lookupObjectCode(key)->sched == 0);
  CHECK(!cache.lookupIR("x") && !cache.lookupOptimizedMLIR("x"));
  llk_b200::CacheStats s = cache.getStats();
  CHECK(s.hits[2] == 2 && s.misses[2] == 2);           // find miss + build miss; two find hits
  llk_weight_key wk;
  std::memset(&wk, 0, sizeof wk);
  wk.weight_ptr = &wk;
  CHECK(!cache.lookupPackedWeights(wk));                // L4 miss
  CHECK(cache.getStats().misses[3] == 1);
  if (gpu) {
    enum { K = 256, N = 512, M = 64 };
    std::vector<uint16_t> wg(K * N, 0x3E00), wu(K * N, 0x3E00), x(M * K, 0x3D80), y(M * N, 0);
    Tensor2D tg = {wg.data(), K, N, N, 1}, tu = {wu.data(), K, N, N, 1};
    llk_packed_weights *pw = nullptr;
    CHECK(llk_pack_weights(&tg, &tu, nullptr, &pw) == LLK_OK);
    CHECK(llk_weight_key_for(&tg, &tu, &wk) == LLK_OK && wk.BK == 64 && wk.BN == 64);
    CHECK(cache.insertPackedWeights(wk, pw));
    llk_packed_weights_free(pw);                        // the cache's reference keeps it alive
    llk_b200::PackedWeightsRef ref = cache.lookupPackedWeights(wk);
    CHECK(ref && ref.get() == pw);
    cache.setMaxEntries(4, 0);                          // evicted; our reference remains
    CHECK(!cache.lookupPackedWeights(wk) && cache.getStats().evictions[3] == 1);
    llk_packed_layout lay;
    CHECK(llk_packed_weights_layout(ref.get(), &lay) == LLK_OK && lay.box_n == 64 && lay.slab_stride_bytes == K * 128);
    Tensor2D tx = {x.data(), M, K, K, 1}, ty = {y.data(), M, N, N, 1};
    CHECK(llk_swiglu_packed(&tx, ref.get(), &ty, nullptr, nullptr) == LLK_OK);
    CHECK(llk_synchronize(-1, nullptr) == LLK_OK);
    CHECK(y[0] == 0x4061);                              // 2 / (1 + e^-2) * 2 in bf16
    cache.setMaxEntries(4, 64);
  }
  cache.clear();
  CHECK(cache.size() == 0);
  std::printf("ok\n");
  return 0;
}
