// Fused peer-memory all-reduce over NVLink 5 / NVSwitch (sm_100a).
//
// Replaces the DDP bucket all-reduce of the reference
// (src/transformer_internals/parallel/data_parallel.py:98-152: SUM all-reduce
// of 25 MB reverse-order buckets, then divide by p) with one kernel per bucket
// that does the reduce-scatter, the 1/p scale and the all-gather itself:
//
//   1. every CTA j of every rank raises "arrived" flag j on all peers
//      (st.release.sys through the peer mapping), then waits (bounded) until
//      all peers' CTA j have arrived: the gradients each peer produced before
//      this launch are complete;
//   2. CTA j of rank r owns part j of slice r of the bucket: it loads that part
//      from every peer's buffer (P2P loads over NVLink, fp32 accumulate),
//      scales by 1/p and stores the result into every peer's buffer (P2P
//      stores): reduce-scatter + all-gather with no staging copy;
//   3. every CTA raises "done" on all peers and waits for all peers' "done",
//      so on exit this rank's buffer holds the final reduced bucket.
//
// Bytes each rank moves: (p-1)/p * S loaded + (p-1)/p * S stored, the ring
// optimum. All waits are bounded by a wall-clock budget; on expiry the kernel
// records ERR_TIMEOUT_PEER and returns without touching peer data.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <string.h>

#include "comm.cuh"
#include "common.cuh"

namespace g2b {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until (int)(*flag - epoch) >= 0. Returns false on timeout.
__device__ bool wait_flag(const uint32_t* flag, uint32_t epoch, int64_t budget) {
  if ((int32_t)(ld_acquire_sys(flag) - epoch) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if ((int32_t)(ld_acquire_sys(flag) - epoch) >= 0) return true;
    if ((int64_t)(globaltimer_ns() - t0) > budget) return false;
    __nanosleep(64);
  }
}

__device__ __forceinline__ uint32_t* flag_slot(uint32_t* base, int phase, int src_rank, int blk) {
  return base + ((phase * kCommMaxRanks + src_rank) * kCommMaxBlocks + blk);
}

// Arrive/wait handshake of one CTA against the same CTA index on every peer.
__device__ bool handshake(const CommArgs& a, uint32_t epoch, int phase, int* fail) {
  const int j = blockIdx.x;
  if (threadIdx.x < a.world) {
    const int q = threadIdx.x;
    st_release_sys(flag_slot(a.peer_flags[q], phase, a.rank, j), epoch);
  }
  if (threadIdx.x < a.world) {
    const int q = threadIdx.x;
    const uint32_t* f = flag_slot(a.peer_flags[a.rank], phase, q, j);
    if (!wait_flag(f, epoch, a.wait_budget_ns)) {
      *fail = 1;
      report_error(a.err, ERR_TIMEOUT_PEER);
      // the first give-up on this rank, for the host to read back
      uint32_t* rec = a.peer_flags[a.rank] + kCommTimeoutWord;
      if (atomicCAS(rec, 0u, 1u) == 0u) {
        rec[1] = (uint32_t)phase;
        rec[2] = (uint32_t)j;
        rec[3] = (uint32_t)q;
        rec[4] = epoch;
        rec[5] = ld_acquire_sys(f);
        rec[6] = (uint32_t)a.rank;
        __threadfence_system();
      }
    }
  }
  __syncthreads();
  return *fail == 0;
}

// The launch's epoch: the caller's, or (epoch 0) this rank's device counter
// + 1. The counter advances when the launch's last CTA finishes, so the next
// launch on the stream reads the new value whichever path launched it (a
// captured graph replays launches with their recorded arguments).
__device__ __forceinline__ uint32_t* epoch_words(const CommArgs& a) {
  return a.peer_flags[a.rank] + kCommEpochWord;
}
__device__ __forceinline__ uint32_t launch_epoch(const CommArgs& a) {
  if (a.epoch) return a.epoch;
  return *reinterpret_cast<volatile uint32_t*>(epoch_words(a)) + 1;
}
// Thread 0 of every CTA, after the CTA's last use of the epoch (also on the
// error path, so a failed launch cannot leave the next one with its epoch).
__device__ __forceinline__ void launch_done(const CommArgs& a, uint32_t epoch) {
  if (a.epoch || threadIdx.x != 0) return;
  uint32_t* w = epoch_words(a);
  __threadfence();
  if (atomicAdd(w + 1, 1u) == gridDim.x - 1) {
    w[1] = 0;
    w[0] = epoch;
    __threadfence();
  }
}

template <typename T>
struct Vec;
template <>
struct Vec<float> {
  static constexpr int N = 4;  // elements per 16-byte vector
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
};

__device__ __forceinline__ void acc_vec(float* acc, const uint4& w, float) {
  acc[0] += __uint_as_float(w.x);
  acc[1] += __uint_as_float(w.y);
  acc[2] += __uint_as_float(w.z);
  acc[3] += __uint_as_float(w.w);
}
__device__ __forceinline__ void acc_vec(float* acc, const uint4& w, __nv_bfloat16) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(ws[i]);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}
__device__ __forceinline__ uint4 pack_vec(const float* acc, float) {
  return make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(acc[2]),
                    __float_as_uint(acc[3]));
}
__device__ __forceinline__ uint4 pack_vec(const float* acc, __nv_bfloat16) {
  return make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                    pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
}

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16(x);
}

// The data path of one launch (between the arrive and done handshakes).
template <typename T, int W>
__device__ __forceinline__ void allreduce_p2p_body(const CommArgs& a) {
  constexpr int VN = Vec<T>::N;
  // Vectorised part: slices of whole 16-byte vectors; the scalar tail (< VN
  // elements per rank boundary) is handled by rank 0's last CTA.
  const int64_t nvec = a.n / VN;
  const int64_t per_rank = (nvec + W - 1) / W;
  const int64_t s0 = min(nvec, per_rank * a.rank), s1 = min(nvec, s0 + per_rank);
  const int64_t per_blk = (s1 - s0 + gridDim.x - 1) / gridDim.x;
  const int64_t b0 = min(s1, s0 + per_blk * blockIdx.x), b1 = min(s1, b0 + per_blk);
  const T zero_tag{};
  // U vectors per thread per iteration, every peer's loads issued before any
  // sum: U x W = 8 sixteen-byte loads in flight per thread, so a few CTAs
  // already cover NVLink latency and the kernel holds few SMs while it
  // overlaps the backward.
  constexpr int U = W >= 8 ? 1 : 8 / W;
  const int64_t span = (int64_t)blockDim.x * U;
  for (int64_t v0 = b0 + threadIdx.x; v0 < b1; v0 += span) {
    uint4 w[U][W];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + (int64_t)u * blockDim.x;
      if (v < b1) {
#pragma unroll
        for (int q = 0; q < W; ++q)
          w[u][q] = __ldcg(reinterpret_cast<const uint4*>(
                               reinterpret_cast<const T*>(a.peer_bufs[q]) + a.offset) + v);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + (int64_t)u * blockDim.x;
      if (v < b1) {
        float acc[VN];
#pragma unroll
        for (int i = 0; i < VN; ++i) acc[i] = 0.f;
#pragma unroll
        for (int q = 0; q < W; ++q) acc_vec(acc, w[u][q], zero_tag);
#pragma unroll
        for (int i = 0; i < VN; ++i) acc[i] *= a.scale;
        const uint4 out = pack_vec(acc, zero_tag);
#pragma unroll
        for (int q = 0; q < W; ++q) {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.peer_bufs[q]) + a.offset) + v;
          __stcg(dst, out);
        }
      }
    }
  }
  if (a.rank == 0 && blockIdx.x == gridDim.x - 1) {
    for (int64_t e = nvec * VN + threadIdx.x; e < a.n; e += blockDim.x) {
      float acc = 0.f;
      for (int q = 0; q < W; ++q) {
        const T* src = reinterpret_cast<const T*>(a.peer_bufs[q]) + a.offset + e;
        acc += to_f32(__ldcg(src));
      }
      for (int q = 0; q < W; ++q)
        reinterpret_cast<T*>(a.peer_bufs[q])[a.offset + e] = from_f32<T>(acc * a.scale);
    }
  }
  __threadfence_system();
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, (unsigned long long)(a.count >= 0 ? a.count : a.n) * sizeof(T));
}

template <typename T, int W, int NT>
__global__ void __launch_bounds__(NT, NT == 128 ? 6 : 1) allreduce_p2p_kernel(const CommArgs a) {
  __shared__ int fail;
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) {
    fail = 0;
    s_epoch = launch_epoch(a);
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  if (handshake(a, epoch, 0, &fail)) allreduce_p2p_body<T, W>(a);
  if (!fail) handshake(a, epoch, 1, &fail);
  launch_done(a, epoch);
}


// ------------------------------------------------------ multimem (NVLS) --
__device__ __forceinline__ uint4 mc_ld_reduce(const uint4* p, float) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p)
               : "memory");
  return r;
}
__device__ __forceinline__ uint4 mc_ld_reduce(const uint4* p, __nv_bfloat16) {
  uint4 r;
  asm volatile(
      "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p)
      : "memory");
  return r;
}
__device__ __forceinline__ void mc_st(uint4* p, const uint4& v, float) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void mc_st(uint4* p, const uint4& v, __nv_bfloat16) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(p),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

template <typename T, int NT>
__device__ __forceinline__ void allreduce_mc_body(const CommArgs& a) {
  constexpr int VN = Vec<T>::N;
  const T tag{};
  const int64_t nvec = a.n / VN;  // the launch requires n % VN == 0
  const int64_t s0 = nvec * a.rank / a.world, s1 = nvec * (a.rank + 1) / a.world;
  const int64_t per_blk = (s1 - s0 + gridDim.x - 1) / gridDim.x;
  const int64_t b0 = min(s1, s0 + per_blk * blockIdx.x), b1 = min(s1, b0 + per_blk);
  uint4* mc = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.mc_base) + a.offset);
  // U switch reductions in flight per thread before the first store
  constexpr int U = 8;
  for (int64_t v0 = b0 + threadIdx.x; v0 < b1; v0 += (int64_t)NT * U) {
    uint4 w[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + (int64_t)u * NT;
      if (v < b1) w[u] = mc_ld_reduce(mc + v, tag);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + (int64_t)u * NT;
      if (v < b1) {
        float acc[VN];
#pragma unroll
        for (int i = 0; i < VN; ++i) acc[i] = 0.f;
        acc_vec(acc, w[u], tag);
#pragma unroll
        for (int i = 0; i < VN; ++i) acc[i] *= a.scale;
        mc_st(mc + v, pack_vec(acc, tag), tag);
      }
    }
  }
  // the stores went out through the multicast alias; peers read the result
  // through their own addresses after the handshake
  asm volatile("fence.proxy.alias;" ::: "memory");
  __threadfence_system();
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, (unsigned long long)(a.count >= 0 ? a.count : a.n) * sizeof(T));
}

template <typename T, int NT>
__global__ void __launch_bounds__(NT, 1) allreduce_mc_kernel(const CommArgs a) {
  __shared__ int fail;
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) {
    fail = 0;
    s_epoch = launch_epoch(a);
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  if (handshake(a, epoch, 0, &fail)) allreduce_mc_body<T, NT>(a);
  if (!fail) handshake(a, epoch, 1, &fail);
  launch_done(a, epoch);
}

template <typename T, int NT>
void launch_allreduce_nt(const CommArgs& a, cudaStream_t s) {
  switch (a.world) {
    case 1: allreduce_p2p_kernel<T, 1, NT><<<a.nblocks, NT, 0, s>>>(a); break;
    case 2: allreduce_p2p_kernel<T, 2, NT><<<a.nblocks, NT, 0, s>>>(a); break;
    case 3: allreduce_p2p_kernel<T, 3, NT><<<a.nblocks, NT, 0, s>>>(a); break;
    case 4: allreduce_p2p_kernel<T, 4, NT><<<a.nblocks, NT, 0, s>>>(a); break;
    case 5: allreduce_p2p_kernel<T, 5, NT><<<a.nblocks, NT, 0, s>>>(a); break;
    case 6: allreduce_p2p_kernel<T, 6, NT><<<a.nblocks, NT, 0, s>>>(a); break;
    case 7: allreduce_p2p_kernel<T, 7, NT><<<a.nblocks, NT, 0, s>>>(a); break;
    default: allreduce_p2p_kernel<T, 8, NT><<<a.nblocks, NT, 0, s>>>(a); break;
  }
}

template <typename T>
void launch_allreduce(const CommArgs& a, cudaStream_t s) {
  if (a.threads == 128)
    launch_allreduce_nt<T, 128>(a, s);
  else
    launch_allreduce_nt<T, 512>(a, s);
}

__global__ void flag_wait_test_kernel(uint32_t* flag, uint32_t value, int64_t budget,
                                      uint32_t* err) {
  if (!wait_flag(flag, value, budget)) report_error(err, ERR_TIMEOUT_PEER);
}

}  // namespace

int comm_allreduce_launch(const CommArgs& a, cudaStream_t s) {
  if (a.world < 1 || a.world > kCommMaxRanks || a.nblocks < 1 || a.nblocks > kCommMaxBlocks)
    return -1;
  if (a.threads != 128 && a.threads != 512) return -3;
  if (a.n <= 0) return 0;
  const int esz = a.dtype == 0 ? 4 : 2;
  if ((a.offset * esz) % 16) return -2;  // bucket starts must be 16-byte aligned
  if (a.dtype == 0)
    launch_allreduce<float>(a, s);
  else
    launch_allreduce<__nv_bfloat16>(a, s);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int comm_allreduce_mc_launch(const CommArgs& a, cudaStream_t s) {
  if (a.world < 1 || a.world > kCommMaxRanks || a.nblocks < 1 || a.nblocks > kCommMaxBlocks)
    return -1;
  if (!a.mc_base) return -4;
  if (a.n <= 0) return 0;
  const int esz = a.dtype == 0 ? 4 : 2;
  // whole 16-byte vectors, 16-byte aligned: multimem.v4 moves exactly one
  if ((a.offset * esz) % 16 || (a.n * esz) % 16 || (reinterpret_cast<uintptr_t>(a.mc_base) % 16))
    return -2;
  if (a.dtype == 0)
    allreduce_mc_kernel<float, 512><<<a.nblocks, 512, 0, s>>>(a);
  else
    allreduce_mc_kernel<__nv_bfloat16, 512><<<a.nblocks, 512, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int comm_flag_wait_test_launch(uint32_t* flag, uint32_t value, int64_t budget_ns, uint32_t* err,
                               cudaStream_t s) {
  flag_wait_test_kernel<<<1, 1, 0, s>>>(flag, value, budget_ns, err);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

std::string comm_ipc_handle(void* ptr) {
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return std::string();
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void* comm_ipc_open(const std::string& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) return nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return nullptr;
  return p;
}

void comm_ipc_close(void* ptr) {
  if (ptr) cudaIpcCloseMemHandle(ptr);
}

void* comm_symm_alloc(int64_t bytes) {
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return nullptr;
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess) {
    cudaFree(p);
    return nullptr;
  }
  return p;
}

void comm_symm_free(void* p) {
  if (p) cudaFree(p);
}

int comm_enable_peer(int peer) {
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return 0;
  }
  return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace g2b
