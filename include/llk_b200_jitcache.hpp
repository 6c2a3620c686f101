/* llk_b200_jitcache.hpp -- C++ face of the B200 library's caches with the
 * method names of the reference's llk::JitCache
 * (include/LLK/Runtime/JitCache.h:77-163), header-only over the C ABI of
 * llk_b200.h.
 *
 *   reference                                  here
 *   lookupOrCompile(KernelKey, ModuleOp)       lookupOrCompile(key, M): the
 *                                              built-in launch plan, cached
 *   lookupObjectCode / insertObjectCode (L3)   launch plans keyed by
 *                                              KernelKey (llk_kernel_key)
 *   lookupPackedWeights / insertPackedWeights  device-resident packed pairs
 *   (L4, WeightKey -> serialised blob)         keyed by WeightKey
 *                                              (llk_weight_key)
 *   lookupIR / lookupOptimizedMLIR (L1, L2)    none: the kernels are compiled
 *                                              ahead of time (always miss)
 *   setMaxEntries(level, n), getStats(),       same, levels numbered as the
 *   clear(), size()                            reference's (1..4)
 *
 * The caches are process-wide (one per library, like one JitCache shared by
 * the process); JitCache objects are thin handles onto them.  Thread-safe.
 */
#ifndef LLK_B200_JITCACHE_HPP
#define LLK_B200_JITCACHE_HPP

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <optional>
#include <string>
#include <utility>

#include "llk_b200.h"

namespace llk_b200 {

/* Aggregate statistics per level, index 0..3 = levels 1..4
 * (JitCache.h:66-71). */
struct CacheStats {
  size_t hits[4]{};
  size_t misses[4]{};
  size_t evictions[4]{};
};

/* One reference to a packed pair; released on destruction. */
class PackedWeightsRef {
 public:
  PackedWeightsRef() = default;
  explicit PackedWeightsRef(llk_packed_weights *pw) : pw_(pw) {}
  PackedWeightsRef(const PackedWeightsRef &) = delete;
  PackedWeightsRef &operator=(const PackedWeightsRef &) = delete;
  PackedWeightsRef(PackedWeightsRef &&o) noexcept : pw_(std::exchange(o.pw_, nullptr)) {}
  PackedWeightsRef &operator=(PackedWeightsRef &&o) noexcept {
    if (this != &o) {
      reset();
      pw_ = std::exchange(o.pw_, nullptr);
    }
    return *this;
  }
  ~PackedWeightsRef() { reset(); }

  llk_packed_weights *get() const { return pw_; }
  explicit operator bool() const { return pw_ != nullptr; }
  void reset() {
    if (pw_) llk_packed_weights_free(pw_);
    pw_ = nullptr;
  }

 private:
  llk_packed_weights *pw_ = nullptr;
};

class JitCache {
 public:
  using Plan = llk_launch_plan;

  /* The plan a key resolves to for M rows; built and cached on a miss. */
  std::optional<Plan> lookupOrCompile(const llk_kernel_key &key, int64_t M) {
    Plan p;
    if (llk_plan_lookup(&key, M, &p) != LLK_OK) return std::nullopt;
    return p;
  }

  /* L3 */
  std::optional<Plan> lookupObjectCode(const llk_kernel_key &key) {
    Plan p;
    if (llk_plan_find(&key, &p) != LLK_OK) return std::nullopt;
    return p;
  }
  bool insertObjectCode(const llk_kernel_key &key, const Plan &plan) {
    return llk_plan_insert(&key, &plan) == LLK_OK;
  }

  /* L2 / L1: no ahead-of-time counterpart; always a miss. */
  std::optional<std::string> lookupOptimizedMLIR(const std::string &) { return std::nullopt; }
  void insertOptimizedMLIR(const std::string &, std::string) {}
  std::optional<std::string> lookupIR(const std::string &) { return std::nullopt; }
  void insertIR(const std::string &, std::string) {}

  /* L4 */
  PackedWeightsRef lookupPackedWeights(const llk_weight_key &key) {
    llk_packed_weights *pw = nullptr;
    if (llk_lookup_packed_weights(&key, &pw) != LLK_OK) return PackedWeightsRef();
    return PackedWeightsRef(pw);
  }
  /* The cache takes its own reference; `pw` stays the caller's. */
  bool insertPackedWeights(const llk_weight_key &key, llk_packed_weights *pw) {
    return llk_insert_packed_weights(&key, pw) == LLK_OK;
  }

  /* Management (level 1-indexed, as the reference's). */
  void evictLRU(size_t level, size_t max_entries) {
    /* trims to max_entries and keeps that bound, like setMaxEntries */
    setMaxEntries(level, max_entries);
  }
  void setMaxEntries(size_t level, size_t max_entries) {
    llk_cache_level_set_max_entries(static_cast<int>(level), static_cast<uint64_t>(max_entries));
  }
  CacheStats getStats() const {
    CacheStats s;
    for (int level = 1; level <= 4; ++level) {
      uint64_t h = 0, m = 0, e = 0;
      llk_cache_level_stats(level, &h, &m, &e, nullptr);
      s.hits[level - 1] = static_cast<size_t>(h);
      s.misses[level - 1] = static_cast<size_t>(m);
      s.evictions[level - 1] = static_cast<size_t>(e);
    }
    return s;
  }
  void clear() {
    llk_cache_level_clear(3);
    llk_cache_level_clear(4);
  }
  size_t size() const {
    uint64_t n3 = 0, n4 = 0;
    llk_cache_level_stats(3, nullptr, nullptr, nullptr, &n3);
    llk_cache_level_stats(4, nullptr, nullptr, nullptr, &n4);
    return static_cast<size_t>(n3 + n4);
  }
};

/* KernelKey with the field defaults of KernelKey.h:45-58 for this backend
 * (isa = SM100A, strict math, library compiler_version), value-initialised
 * so the whole-struct comparison sees zero padding. */
inline llk_kernel_key make_kernel_key(int operation, int64_t M_bucket, int64_t N, int64_t K,
                                      int output_type = LLK_DTYPE_BF16, int variant = LLK_VARIANT_TC) {
  llk_kernel_key k;
  std::memset(&k, 0, sizeof(k));
  k.operation = static_cast<uint8_t>(operation);
  k.input_type = LLK_DTYPE_BF16;
  k.output_type = static_cast<uint8_t>(output_type);
  k.M_bucket = M_bucket;
  k.N = N;
  k.K = K;
  k.isa = LLK_ISA_SM100A;
  k.thread_count = static_cast<uint16_t>(variant);
  k.compiler_version = llk_version();
  k.schedule_version = 1;
  return k;
}

}  // namespace llk_b200

#endif /* LLK_B200_JITCACHE_HPP */
