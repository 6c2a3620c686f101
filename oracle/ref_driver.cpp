// ref_driver.cpp -- runs the DSLCompiler reference's own C++ SwiGLU oracle
// on inputs given as files.  TEST INFRASTRUCTURE ONLY.
//
// The reference's test/Execution/swiglu_reference.cpp (its naive FP32
// swiglu_reference, lines 38-71, and FP64 swiglu_reference_fp64, lines
// 77-99, plus its gtest cases) is compiled where it lies in the reference
// tree by including it into this translation unit (oracle/Makefile passes
// the reference root as an include path).  Nothing is copied.
//
// Usage:
//   ref_driver gtest [gtest flags]          run the reference's own tests
//   ref_driver swiglu M N K x wg wu y32 y64 read f32 inputs (raw little-
//                                           endian files), write the
//                                           reference's f32 and f64 outputs
//   ref_driver time M N K reps              time the reference's naive f32
//                                           swiglu_reference (one thread) on
//                                           seeded inputs: prints the best
//                                           seconds per call
#include "test/Execution/swiglu_reference.cpp"

#include <cstdio>
#include <chrono>
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
  if (argc == 10 && std::string(argv[1]) == "swiglu") {
    int64_t M = std::atoll(argv[2]), N = std::atoll(argv[3]),
            K = std::atoll(argv[4]);
    std::vector<float> x, wg, wu;
    if (!readFile(argv[5], x, M * K) || !readFile(argv[6], wg, K * N) ||
        !readFile(argv[7], wu, K * N)) {
      std::fprintf(stderr, "ref_driver: cannot read inputs\n");
      return 2;
    }
    std::vector<float> y(M * N);
    swiglu_reference(x.data(), wg.data(), wu.data(), y.data(), M, N, K);
    std::vector<double> xd(x.begin(), x.end()), wgd(wg.begin(), wg.end()),
        wud(wu.begin(), wu.end()), yd(M * N);
    swiglu_reference_fp64(xd.data(), wgd.data(), wud.data(), yd.data(), M, N,
                          K);
    if (!writeFile(argv[8], y) || !writeFile(argv[9], yd)) {
      std::fprintf(stderr, "ref_driver: cannot write outputs\n");
      return 2;
    }
    return 0;
  }
  if (argc == 6 && std::string(argv[1]) == "time") {
    int64_t M = std::atoll(argv[2]), N = std::atoll(argv[3]),
            K = std::atoll(argv[4]);
    const int reps = std::atoi(argv[5]);
    if (M <= 0 || N <= 0 || K <= 0 || reps <= 0) return 1;
    std::vector<float> x(M * K), wg(K * N), wu(K * N), y(M * N);
    uint32_t st = 12345u;  // LCG in [-1, 1): the timing does not depend on values
    auto rnd = [&st]() {
      st = st * 1664525u + 1013904223u;
      return static_cast<float>(st >> 8) / 8388608.0f - 1.0f;
    };
    for (auto &v : x) v = rnd();
    for (auto &v : wg) v = rnd() * 0.02f;
    for (auto &v : wu) v = rnd() * 0.02f;
    double best = 1e30;
    for (int r = 0; r < reps; ++r) {
      auto t0 = std::chrono::steady_clock::now();
      swiglu_reference(x.data(), wg.data(), wu.data(), y.data(), M, N, K);
      double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      if (dt < best) best = dt;
    }
    std::printf("%.9f %g\n", best, static_cast<double>(y[0]));
    return 0;
  }
  std::fprintf(stderr,
               "usage: ref_driver gtest | ref_driver swiglu M N K x wg wu "
               "y32 y64 | ref_driver time M N K reps\n");
  return 1;
}
