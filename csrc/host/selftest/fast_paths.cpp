// Exhaustive check of the host fast paths (csrc/host/fast_scalar.h) against
// the scalar rules of csrc/common/ngl_scalar.h: q823_from_f32 and eb_code
// (both forms, scale 1 and 2e-3) over all 2^32 float bit patterns, q823_to_f32 over all
// 2^32 int32 values, stochastic rounding on 10^8 random (value, seed,
// counter), absmax folds with NaN / inf / signed zeros, u64 -> f32 on 10^8
// values of every magnitude.  Prints "fast paths ok" and exits 0 when every result matches.
//
//   g++ -std=c++17 -O2 -ffp-contract=off -pthread -Icsrc csrc/host/selftest/fast_paths.cpp -o fp && ./fp
#include <atomic>
#include <cstdio>
#include <cstring>
#include <limits>
#include <random>
#include <thread>
#include <vector>

#include "../fast_scalar.h"

using namespace ngl;

namespace {
std::atomic<uint64_t> g_bad{0};

float f_of(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

void check_range(uint64_t lo, uint64_t hi) {
  uint64_t bad = 0;
  for (uint64_t k = lo; k < hi; ++k) {
    const uint32_t u = (uint32_t)k;
    const float x = f_of(u);
    bad += host::fast::q823_from_f32(x) != ngl::q823_from_f32(x);
    bad += host::fast::eb_code(x, 1.0f) != ngl::eb_code(x, 1.0f);
    bad += host::fast::eb_code(x, 2e-3f) != ngl::eb_code(x, 2e-3f);
    bad += host::fast::eb_code_bf(x, 1.0f) != ngl::eb_code(x, 1.0f);
    bad += host::fast::eb_code_bf(x, 2e-3f) != ngl::eb_code(x, 2e-3f);
    const float a = host::fast::q823_to_f32((int32_t)u), b = ngl::q823_to_f32((int32_t)u);
    bad += std::memcmp(&a, &b, 4) != 0;
  }
  g_bad += bad;
}
}  // namespace

int main() {
  const unsigned nt = std::max(1u, std::thread::hardware_concurrency());
  const uint64_t total = 1ull << 32;
  std::vector<std::thread> ts;
  for (unsigned t = 0; t < nt; ++t) ts.emplace_back(check_range, total * t / nt, total * (t + 1) / nt);
  for (auto& t : ts) t.join();
  std::mt19937_64 rng(7);
  uint64_t bad = 0;
  for (int i = 0; i < 100000000; ++i) {
    const uint64_t w = rng();
    // values around the INT4/INT8 code range, with exact integers and halves
    const float v = (i & 3) == 0 ? (float)((int)(w % 33) - 16) * 0.5f : f_of((uint32_t)(w >> 32)) ;
    const uint64_t seed = rng(), counter = rng();
    bad += host::fast::stochastic_round(v, seed, counter) != ngl::compat_stochastic_round(v, seed, counter);
  }
  // absmax against the maxNum fold, with NaN, inf and signed zeros mixed in
  for (int t = 0; t < 20000; ++t) {
    float v[64];
    for (float& x : v) {
      const uint64_t w = rng();
      x = (w & 7) == 0 ? f_of((uint32_t)(w >> 32)) : (float)(int)(w % 2001 - 1000) * 1e-3f;
      // quiet NaNs only: glibc's fmaxf returns NaN for a signaling one (the
      // fold then loses its maximum), Rust's max and the comparison skip it
      if (x != x) x = std::numeric_limits<float>::quiet_NaN();
    }
    float m = 0.0f;
    for (float x : v) m = ngl::f_max(m, ngl::f_abs(x));
    const float a = host::fast::absmax(v, 64);
    bad += std::memcmp(&a, &m, 4) != 0;
  }
  for (int i = 0; i < 100000000; ++i) {
    const uint64_t x = rng() >> (i % 64);
    const float a = host::fast::u64_to_f32(x), b = ngl::u64_to_f32(x);
    bad += std::memcmp(&a, &b, 4) != 0;
  }
  g_bad += bad;
  if (g_bad != 0) {
    std::printf("fast paths differ on %llu inputs\n", (unsigned long long)g_bad.load());
    return 1;
  }
  std::printf("fast paths ok\n");
  return 0;
}
