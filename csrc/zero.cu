// ZeRO-2 over NVLink 5 peer memory, fused with the sharded AdamW (sm_100a).
//
// Replaces the reference's ZeRO-2 step (src/transformer_internals/parallel/
// zero.py:393-486: reduce_scatter of the flat gradient, divide by p, sharded
// global-norm clip with a 4-byte all_reduce, AdamW on the owned slice in
// torch's single-tensor order, all_gather of the updated slices) with two
// kernels:
//
//   zero_rs_kernel        (one launch per gradient bucket, on a communication
//                          stream while backward continues): every rank
//                          reduces ITS slice of the bucket by loading it from
//                          every peer's gradient buffer (P2P loads over
//                          NVLink, fixed rank order), scales by 1/p, writes
//                          the averaged slice into its local gradient shard
//                          and leaves per-CTA partial sums of squares.
//   zero_adamw_ag_kernel  (once per step): exchanges the local sum of squares
//                          with every peer through one 64-bit {epoch, value}
//                          word per (CTA, rank) -- value and flag in a single
//                          release store -- so every rank and every CTA forms
//                          the same global norm and clip coefficient; runs
//                          AdamW on the owned slices; stores the updated bf16
//                          parameters straight into every peer's parameter
//                          buffer (P2P stores: the all-gather); finishes with
//                          a done handshake so no rank reads its parameters
//                          before every peer has written them.
//
// Slices: bucket b = flat elements [lo, hi) (64-element aligned); rank r owns
// [lo + r*s, min(hi, lo + (r+1)*s)) with s = ceil((hi-lo)/p) rounded up to 64,
// stored at shard offset off_b = sum of the earlier buckets' s. All waits are
// bounded; on expiry a kernel records ERR_TIMEOUT_PEER and returns.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "comm.cuh"
#include "common.cuh"
#include "zero.cuh"

namespace g2b {
namespace {

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t* zflag(uint32_t* base, int phase, int src, int blk) {
  return base + ((phase * kCommMaxRanks + src) * kZeroMaxBlocks + blk);
}

// CTA j raises its flag on every peer, then waits (bounded) for every peer's
// CTA j. Threads [0, world) do the work; the result is CTA-uniform.
__device__ bool zero_handshake(const ZeroArgs& a, int phase, int* fail) {
  const int j = blockIdx.x;
  if (threadIdx.x < a.world)
    st_release_sys_u32(zflag(a.peer_flags[threadIdx.x], phase, a.rank, j), a.epoch);
  if (threadIdx.x < a.world) {
    const uint32_t* f = zflag(a.peer_flags[a.rank], phase, threadIdx.x, j);
    if ((int32_t)(ld_acquire_sys_u32(f) - a.epoch) < 0) {
      const uint64_t t0 = globaltimer_ns();
      while ((int32_t)(ld_acquire_sys_u32(f) - a.epoch) < 0) {
        if ((int64_t)(globaltimer_ns() - t0) > a.wait_budget_ns) {
          *fail = 1;
          report_error(a.err, ERR_TIMEOUT_PEER);
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  return *fail == 0;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0) {
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  }
  return t;  // valid in thread 0
}

struct Slice {
  int64_t f0, n, off;  // flat start, elements owned, shard offset
};
__device__ __forceinline__ Slice my_slice(const ZeroArgs& a, int b) {
  const int64_t lo = a.buckets[4 * b], hi = a.buckets[4 * b + 1];
  const int64_t s = a.buckets[4 * b + 2], off = a.buckets[4 * b + 3];
  const int64_t f0 = lo + (int64_t)a.rank * s;
  int64_t n = min(hi, f0 + s) - f0;
  if (n < 0) n = 0;
  return {f0, n, off};
}

// The reduce-scatter and the parameter gather overlap backward / the
// previous block's compute on a side stream: 128-thread CTAs with at most 80
// registers a thread and 4 bytes of shared memory, so one fits on an SM next
// to a resident persistent GEMM or attention CTA.
constexpr int kZeroThreads = 128;

// Four gradient elements of rank q at vector v of the slice: fp32, or (BF16)
// the rank's bf16 copy.
template <bool BF16>
__device__ __forceinline__ float4 rs_load(const ZeroArgs& a, int q, int64_t f0, int64_t v) {
  if (BF16) {
    const uint2 w = __ldcg(reinterpret_cast<const uint2*>(a.peer_grad16[q] + f0) + v);
    const float2 lo = unpack_bf16x2(w.x), hi = unpack_bf16x2(w.y);
    return make_float4(lo.x, lo.y, hi.x, hi.y);
  }
  return __ldcg(reinterpret_cast<const float4*>(a.peer_grad[q] + f0) + v);
}

template <bool BF16>
__global__ void __launch_bounds__(kZeroThreads, 6) zero_rs_kernel(const ZeroArgs a) {
  __shared__ int fail;
  __shared__ float red[16];
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!zero_handshake(a, 0, &fail)) return;
  const Slice sl = my_slice(a, a.bucket);
  const int64_t nv = sl.n / 4;
  const int64_t per = (nv + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = min(nv, per * blockIdx.x), v1 = min(nv, v0 + per);
  float ss = 0.f;
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    // every rank's load is issued before the first sum (rank order kept)
    float4 w[kCommMaxRanks];
#pragma unroll
    for (int q = 0; q < kCommMaxRanks; ++q)
      if (q < a.world) w[q] = rs_load<BF16>(a, q, sl.f0, v);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < kCommMaxRanks; ++q) {
      if (q >= a.world) break;
      acc.x += w[q].x;
      acc.y += w[q].y;
      acc.z += w[q].z;
      acc.w += w[q].w;
    }
    acc.x *= a.scale;
    acc.y *= a.scale;
    acc.z *= a.scale;
    acc.w *= a.scale;
    reinterpret_cast<float4*>(a.gsh + sl.off)[v] = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  const float t = block_sum(ss, red);
  if (threadIdx.x == 0 && a.sumsq_parts)
    a.sumsq_parts[(int64_t)a.bucket * a.rs_blocks + blockIdx.x] = t;
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, (unsigned long long)(a.buckets[4 * a.bucket + 1] -
                                                   a.buckets[4 * a.bucket]) * (BF16 ? 2ull : 4ull));
  if (a.done_handshake) {
    __syncthreads();
    zero_handshake(a, 1, &fail);
  }
}

__global__ void __launch_bounds__(kZeroThreads, 6) zero_ag_kernel(const ZeroArgs a) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!zero_handshake(a, 0, &fail)) return;
  const int64_t nv = a.ag_span / 8;
  const int64_t sv = a.ag_slice / 8;
  // slice q of the unit comes from rank q; kAgLoads independent 16-byte peer
  // loads in flight per thread
  constexpr int kAgLoads = 8;
  const int64_t span = (int64_t)gridDim.x * blockDim.x;
  for (int q = 0; q < a.world; ++q) {
    const uint4* src = reinterpret_cast<const uint4*>(a.peer_shard[q] + a.ag_offset);
    uint4* dst = reinterpret_cast<uint4*>(a.gather_dst) + (int64_t)q * sv;
    const int64_t n = min(sv, nv - (int64_t)q * sv);
    for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < n;
         i0 += span * kAgLoads) {
      uint4 w[kAgLoads];
#pragma unroll
      for (int u = 0; u < kAgLoads; ++u)
        if (i0 + u * span < n) w[u] = __ldcg(src + i0 + u * span);
#pragma unroll
      for (int u = 0; u < kAgLoads; ++u)
        if (i0 + u * span < n) dst[i0 + u * span] = w[u];
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, (unsigned long long)a.ag_span * 2ull);
}

__device__ __forceinline__ bool zero_in_decay(int64_t e, const int64_t* __restrict__ r, int nr) {
  int lo = 0, hi = nr;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(r + 2 * mid) <= e) lo = mid; else hi = mid;
  }
  return nr > 0 && e >= __ldg(r + 2 * lo) && e < __ldg(r + 2 * lo + 1);
}

__global__ void __launch_bounds__(512) zero_adamw_ag_kernel(const ZeroArgs a) {
  __shared__ int fail;
  __shared__ float red[16];
  __shared__ float peer_ss[kCommMaxRanks];
  __shared__ float s_clip;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  // 1. this rank's sum of squares, fixed order over (bucket, rs CTA)
  float ss = 0.f;
  const int nparts = a.nb * a.rs_blocks;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) ss += a.sumsq_parts[i];
  const float local = block_sum(ss, red);
  // 2. exchange with every peer: one {epoch, value} word per (CTA, source rank)
  const int j = blockIdx.x;
  const int par = a.epoch & 1;
  if (threadIdx.x == 0) red[0] = local;
  __syncthreads();
  if (threadIdx.x < a.world) {
    const unsigned long long word =
        ((unsigned long long)a.epoch << 32) | (unsigned long long)__float_as_uint(red[0]);
    st_release_sys_u64(a.peer_norm[threadIdx.x] + ((par * kZeroMaxBlocks + j) * kCommMaxRanks + a.rank),
                       word);
    const unsigned long long* slot =
        a.peer_norm[a.rank] + ((par * kZeroMaxBlocks + j) * kCommMaxRanks + threadIdx.x);
    unsigned long long w = ld_acquire_sys_u64(slot);
    if ((uint32_t)(w >> 32) != a.epoch) {
      const uint64_t t0 = globaltimer_ns();
      while ((uint32_t)((w = ld_acquire_sys_u64(slot)) >> 32) != a.epoch) {
        if ((int64_t)(globaltimer_ns() - t0) > a.wait_budget_ns) {
          fail = 1;
          report_error(a.err, ERR_TIMEOUT_PEER);
          break;
        }
        __nanosleep(32);
      }
    }
    peer_ss[threadIdx.x] = __uint_as_float((uint32_t)w);
  }
  __syncthreads();
  if (fail) return;
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int q = 0; q < a.world; ++q) tot += peer_ss[q];  // same order on every rank
    const float norm = sqrtf(tot);
    float c = 1.f;
    if (a.max_norm > 0.f) c = fminf(a.max_norm / (norm + 1e-6f), 1.f);
    s_clip = c;
    if (j == 0 && a.norm_out) a.norm_out[0] = norm;
  }
  __syncthreads();
  // 3. AdamW on the owned slices (torch single-tensor order) + bf16 all-gather
  const float lr = a.hp[0], b1 = a.hp[1], b2 = a.hp[2], eps = a.hp[3], wd = a.hp[4];
  const float bc1 = a.hp[5], bc2s = a.hp[6];
  const float gs = a.hp[7] * s_clip;
  const float step_size = lr / bc1;
  for (int b = 0; b < a.nb; ++b) {
    const Slice sl = my_slice(a, b);
    const int64_t n8 = sl.n / 8;  // slices are multiples of 64 elements
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n8;
         v += (int64_t)gridDim.x * blockDim.x) {
      const int64_t s0 = sl.off + 8 * v;
      const bool decay = zero_in_decay(sl.f0 + 8 * v, a.decay_ranges, a.nr);
      float p[8], g[8], m[8], q[8];
      *reinterpret_cast<float4*>(p) = reinterpret_cast<const float4*>(a.master + s0)[0];
      *reinterpret_cast<float4*>(p + 4) = reinterpret_cast<const float4*>(a.master + s0)[1];
      *reinterpret_cast<float4*>(g) = reinterpret_cast<const float4*>(a.gsh + s0)[0];
      *reinterpret_cast<float4*>(g + 4) = reinterpret_cast<const float4*>(a.gsh + s0)[1];
      *reinterpret_cast<float4*>(m) = reinterpret_cast<const float4*>(a.exp_avg + s0)[0];
      *reinterpret_cast<float4*>(m + 4) = reinterpret_cast<const float4*>(a.exp_avg + s0)[1];
      *reinterpret_cast<float4*>(q) = reinterpret_cast<const float4*>(a.exp_avg_sq + s0)[0];
      *reinterpret_cast<float4*>(q + 4) = reinterpret_cast<const float4*>(a.exp_avg_sq + s0)[1];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float gk = g[k] * gs;
        if (decay) p[k] *= (1.f - lr * wd);
        m[k] += (gk - m[k]) * (1.f - b1);
        q[k] = q[k] * b2 + (1.f - b2) * gk * gk;
        const float denom = sqrtf(q[k]) / bc2s + eps;
        p[k] += -step_size * (m[k] / denom);
      }
      reinterpret_cast<float4*>(a.master + s0)[0] = *reinterpret_cast<float4*>(p);
      reinterpret_cast<float4*>(a.master + s0)[1] = *reinterpret_cast<float4*>(p + 4);
      reinterpret_cast<float4*>(a.exp_avg + s0)[0] = *reinterpret_cast<float4*>(m);
      reinterpret_cast<float4*>(a.exp_avg + s0)[1] = *reinterpret_cast<float4*>(m + 4);
      reinterpret_cast<float4*>(a.exp_avg_sq + s0)[0] = *reinterpret_cast<float4*>(q);
      reinterpret_cast<float4*>(a.exp_avg_sq + s0)[1] = *reinterpret_cast<float4*>(q + 4);
      const uint4 w = make_uint4(pack_bf16x2(p[0], p[1]), pack_bf16x2(p[2], p[3]),
                                 pack_bf16x2(p[4], p[5]), pack_bf16x2(p[6], p[7]));
      for (int r = 0; r < a.world; ++r)
        reinterpret_cast<uint4*>(a.peer_shadow[r] + sl.f0)[v] = w;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter) {
    // all-gather payload in the reference convention (output buffer, bf16)
    // plus the 4-byte norm all-reduce
    int64_t tot = 0;
    for (int b = 0; b < a.nb; ++b) tot += a.buckets[4 * b + 1] - a.buckets[4 * b];
    atomicAdd(a.byte_counter, (unsigned long long)tot * 2ull + 4ull);
  }
  zero_handshake(a, 1, &fail);
}

}  // namespace

int zero_rs_launch(const ZeroArgs& a, cudaStream_t s) {
  if (a.world < 1 || a.world > kCommMaxRanks || a.rs_blocks < 1 || a.rs_blocks > kZeroMaxBlocks ||
      a.bucket < 0 || a.bucket >= a.nb)
    return -1;
  if (a.peer_grad16)
    zero_rs_kernel<true><<<a.rs_blocks, kZeroThreads, 0, s>>>(a);
  else
    zero_rs_kernel<false><<<a.rs_blocks, kZeroThreads, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int zero_ag_launch(const ZeroArgs& a, int nblocks, cudaStream_t s) {
  if (a.world < 1 || a.world > kCommMaxRanks || nblocks < 1 || nblocks > kZeroMaxBlocks ||
      a.ag_slice <= 0 || a.ag_slice % 64 || a.ag_span % 64 || a.ag_offset % 8 ||
      (a.ag_span + a.ag_slice - 1) / a.ag_slice > a.world)
    return -1;
  zero_ag_kernel<<<nblocks, kZeroThreads, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int zero_adamw_ag_launch(const ZeroArgs& a, int nblocks, cudaStream_t s) {
  if (a.world < 1 || a.world > kCommMaxRanks || nblocks < 1 || nblocks > kZeroMaxBlocks) return -1;
  zero_adamw_ag_kernel<<<nblocks, 512, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

}  // namespace g2b
