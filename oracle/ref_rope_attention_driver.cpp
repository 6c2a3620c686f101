// ref_rope_attention_driver.cpp -- runs the DSLCompiler reference's own FP64
// RoPE and attention references on inputs given as files.  TEST
// INFRASTRUCTURE ONLY.
//
// test/Execution/rope_correctness.cpp (ropeReferenceFP64, lines 14-35) and
// test/Execution/attention_correctness.cpp (attentionRefFP64, lines 15-60),
// with their gtest cases, are compiled where they lie in the reference tree
// by including them into this translation unit (oracle/Makefile passes the
// reference root as an include path).  Nothing is copied.
//
// Usage:
//   ref_rope_attention_driver gtest [flags]
//   ref_rope_attention_driver rope B H L D theta x pos y        (x, y f64; pos i64)
//   ref_rope_attention_driver attention B H Lq Lk D scale causal q k v o   (f64)
#include "test/Execution/rope_correctness.cpp"
#include "test/Execution/attention_correctness.cpp"

#include <cstdio>
#include <cstdlib>
#include <string>

template <typename T>
static bool readFile(const char *path, std::vector<T> &v, size_t n) {
  v.resize(n);
  FILE *f = std::fopen(path, "rb");
  if (!f) return false;
  size_t got = n ? std::fread(v.data(), sizeof(T), n, f) : 0;
  std::fclose(f);
  return got == n;
}

template <typename T>
static bool writeFile(const char *path, const std::vector<T> &v) {
  FILE *f = std::fopen(path, "wb");
  if (!f) return false;
  size_t put = v.empty() ? 0 : std::fwrite(v.data(), sizeof(T), v.size(), f);
  std::fclose(f);
  return put == v.size();
}

int main(int argc, char **argv) {
  if (argc >= 2 && std::string(argv[1]) == "gtest") {
    int gargc = argc - 1;
    testing::InitGoogleTest(&gargc, argv + 1);
    return RUN_ALL_TESTS();
  }
  if (argc == 10 && std::string(argv[1]) == "rope") {
    const int64_t B = std::atoll(argv[2]), H = std::atoll(argv[3]), L = std::atoll(argv[4]), D = std::atoll(argv[5]);
    const double theta = std::atof(argv[6]);
    std::vector<double> x, y(B * H * L * D);
    std::vector<int64_t> pos;
    if (!readFile(argv[7], x, B * H * L * D) || !readFile(argv[8], pos, L)) return 2;
    ropeReferenceFP64(x.data(), pos.data(), y.data(), B, H, L, D, theta);
    return writeFile(argv[9], y) ? 0 : 2;
  }
  if (argc == 13 && std::string(argv[1]) == "attention") {
    const int64_t B = std::atoll(argv[2]), H = std::atoll(argv[3]), Lq = std::atoll(argv[4]),
                  Lk = std::atoll(argv[5]), D = std::atoll(argv[6]);
    const double scale = std::atof(argv[7]);
    const bool causal = std::atoi(argv[8]) != 0;
    std::vector<double> q, k, v, o(B * H * Lq * D);
    if (!readFile(argv[9], q, B * H * Lq * D) || !readFile(argv[10], k, B * H * Lk * D) ||
        !readFile(argv[11], v, B * H * Lk * D))
      return 2;
    attentionRefFP64(q.data(), k.data(), v.data(), o.data(), B, H, Lq, Lk, D, scale, causal);
    return writeFile(argv[12], o) ? 0 : 2;
  }
  std::fprintf(stderr, "usage: ref_rope_attention_driver gtest | rope ... | attention ...\n");
  return 1;
}
