// Allocation-free bias-gradient column sum; see noalloc.h for the contract
// (no counterpart in the reference; the scratch array and its limits).
#include "noalloc.h"

#include <cuda_bf16.h>
#include <stdio.h>

#include <mutex>

namespace {

constexpr int kRows = 128;      // rows summed into one partial
constexpr int kMaxDevices = 64;

// The one scratch array (1 MiB per device that loads the library).
static __device__ __align__(256) float g2b_noalloc_scratch[G2B_NOALLOC_SCRATCH_FLOATS];

std::mutex g_mu;
float* g_scratch[kMaxDevices] = {};

// Stage 1: part[chunk, c] = sum of rows [chunk*128, chunk*128+128) of column
// c. Block = 32 groups of 8 columns x 8 row lanes; lanes are combined in a
// fixed order through shared memory, so the result is deterministic.
__global__ void __launch_bounds__(256) noalloc_partial_kernel(const __nv_bfloat16* __restrict__ dy,
                                                              int64_t ld, int M, int C,
                                                              float* __restrict__ part) {
  __shared__ float red[8][32 * 8 + 4];
  const int cg = blockIdx.x * 32 + threadIdx.x;
  const int r0 = blockIdx.y * kRows;
  const int r1 = min(M, r0 + kRows);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (cg * 8 < C) {
    for (int r = r0 + threadIdx.y; r < r1; r += 8) {
      const uint4 w = *reinterpret_cast<const uint4*>(dy + (int64_t)r * ld + cg * 8);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[j]));
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[threadIdx.y][threadIdx.x * 8 + j] = acc[j];
  __syncthreads();
  const int t = threadIdx.y * 32 + threadIdx.x;
  const int col = blockIdx.x * 256 + t;
  if (col < C) {
    float s = 0.f;
#pragma unroll
    for (int y = 0; y < 8; ++y) s += red[y][t];
    part[(int64_t)blockIdx.y * C + col] = s;
  }
}

// Stage 2: out[c] (+)= sum over chunks of part[chunk, c], in chunk order.
__global__ void __launch_bounds__(256) noalloc_final_kernel(const float* __restrict__ part,
                                                            int chunks, int C,
                                                            float* __restrict__ out,
                                                            int accumulate) {
  __shared__ float red[8][33];
  const int c = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (c < C)
    for (int k = threadIdx.y; k < chunks; k += 8) s += part[(int64_t)k * C + c];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < C) {
    float t = 0.f;
#pragma unroll
    for (int y = 0; y < 8; ++y) t += red[y][threadIdx.x];
    out[c] = accumulate ? out[c] + t : t;
  }
}

// Device address of the scratch array on the current device (looked up once
// per device with that device current).
float* scratch_for_current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g2b_noalloc_scratch) != cudaSuccess || p == nullptr) return nullptr;
    g_scratch[dev] = static_cast<float*>(p);
  }
  return g_scratch[dev];
}

}  // namespace

extern "C" int g2b_bias_grad_noalloc(const void* dy, int64_t ld, int M, int C, float* out,
                                     int accumulate, cudaStream_t stream) {
  if (dy == nullptr || out == nullptr || M <= 0 || C <= 0 || C % 8 != 0 || ld % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(dy) & 15) != 0)
    return G2B_NOALLOC_ERR_ARGS;
  const int chunks = (M + kRows - 1) / kRows;
  if ((int64_t)chunks * C > (int64_t)G2B_NOALLOC_SCRATCH_FLOATS) {
    fprintf(stderr,
            "g2b_bias_grad_noalloc: M=%d, C=%d needs %lld scratch floats; the fixed scratch "
            "holds %d (ceil(M/128) * C must not exceed it)\n",
            M, C, (long long)chunks * C, G2B_NOALLOC_SCRATCH_FLOATS);
    return G2B_NOALLOC_ERR_TOO_LARGE;
  }
  float* part = scratch_for_current_device();
  if (part == nullptr) return G2B_NOALLOC_ERR_SETUP;
  noalloc_partial_kernel<<<dim3((C + 255) / 256, chunks), dim3(32, 8), 0, stream>>>(
      static_cast<const __nv_bfloat16*>(dy), ld, M, C, part);
  noalloc_final_kernel<<<(C + 31) / 32, dim3(32, 8), 0, stream>>>(part, chunks, C, out,
                                                                  accumulate);
  return cudaGetLastError() == cudaSuccess ? 0 : G2B_NOALLOC_ERR_LAUNCH;
}
