// Host-side count of kernels launched by this library (one shared object for
// every translation unit: the static local of an inline function).
#pragma once
#include <cuda_runtime.h>

#include <atomic>

namespace g2b {
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> c{0};
  return c;
}
inline void count_launches(int n) { launch_counter().fetch_add(n, std::memory_order_relaxed); }

// The error of the last failed launch on this host thread (cudaSuccess if
// none), kept for the host-side message: the launchers consume the error
// with cudaGetLastError so that it does not leak into unrelated calls.
inline cudaError_t& last_launch_error() {
  static thread_local cudaError_t e = cudaSuccess;
  return e;
}
// true if the launch just issued succeeded; records the error otherwise.
inline bool launch_succeeded() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) last_launch_error() = e;
  return e == cudaSuccess;
}
}  // namespace g2b
