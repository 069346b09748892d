// Minimal fork-join helper for the data loaders: a dynamic work counter shared by
// `threads` std::threads; the first exception thrown by a worker is rethrown.
#pragma once
#include <algorithm>
#include <atomic>
#include <exception>
#include <mutex>
#include <thread>
#include <vector>

namespace ddd {

template <class F>
void parallel_for(int64_t n, int threads, F&& fn) {
  if (n <= 0) return;
  int t = threads > 0 ? threads : static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  t = static_cast<int>(std::min<int64_t>(t, n));
  if (t <= 1) {
    for (int64_t i = 0; i < n; ++i) fn(i);
    return;
  }
  std::atomic<int64_t> next{0};
  std::exception_ptr err;
  std::mutex mu;
  auto work = [&] {
    for (;;) {
      const int64_t i = next.fetch_add(1);
      if (i >= n) return;
      try {
        fn(i);
      } catch (...) {
        std::lock_guard<std::mutex> g(mu);
        if (!err) err = std::current_exception();
        next.store(n);
        return;
      }
    }
  };
  std::vector<std::thread> pool;
  pool.reserve(t - 1);
  for (int k = 1; k < t; ++k) pool.emplace_back(work);
  work();
  for (auto& th : pool) th.join();
  if (err) std::rethrow_exception(err);
}

}  // namespace ddd
