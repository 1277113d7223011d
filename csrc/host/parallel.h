// Block-parallel loops of the host library on plain std::threads (no OpenMP
// runtime next to torch's).  The thread count is NGL_HOST_THREADS, else
// OMP_NUM_THREADS (the variable torch's CPU ops follow), else the hardware
// count.  Callers give each thread a contiguous range of independent work,
// so results do not depend on the thread count.
#pragma once
#include <algorithm>
#include <cstddef>
#include <cstdlib>
#include <thread>
#include <vector>

namespace ngl {
namespace host {

inline size_t host_threads() {
  for (const char* var : {"NGL_HOST_THREADS", "OMP_NUM_THREADS"}) {
    if (const char* v = std::getenv(var)) {
      const long t = std::strtol(v, nullptr, 10);
      if (t > 0) return (size_t)t;
    }
  }
  return std::max<size_t>(1, std::thread::hardware_concurrency());
}

// fn(begin, end) over [0, n) in up to host_threads() contiguous ranges of at
// least min_per_thread items; runs inline when one range suffices.
template <typename F>
void parallel_for(size_t n, size_t min_per_thread, F&& fn) {
  const size_t t = std::min(host_threads(), n / std::max<size_t>(1, min_per_thread));
  if (t <= 1) {
    fn((size_t)0, n);
    return;
  }
  std::vector<std::thread> ts;
  ts.reserve(t - 1);
  for (size_t k = 1; k < t; ++k) ts.emplace_back([&fn, n, t, k] { fn(n * k / t, n * (k + 1) / t); });
  fn((size_t)0, n / t);
  for (auto& th : ts) th.join();
}

}  // namespace host
}  // namespace ngl
