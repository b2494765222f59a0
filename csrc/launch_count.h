// Host-side count of kernels launched by this library (one shared object for
// every translation unit: the static local of an inline function).
#pragma once
#include <atomic>

namespace g2b {
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> c{0};
  return c;
}
inline void count_launches(int n) { launch_counter().fetch_add(n, std::memory_order_relaxed); }
}  // namespace g2b
