// Incremental (KV-cached) decoding kernels, head_dim 64.
//
// The cache is preallocated: K and V are [B, Hkv, Tmax, 64] bf16 and a device
// vector lens[B] holds how many positions of each sequence are cached. One
// decode step reads lens from device memory, so a whole step (embedding,
// layers, head, argmax) can be captured once in a CUDA graph and replayed.
//
//   decode_embed      x[b] = wte[tok[b]] + wpe[lens[b]]                (fp32)
//   decode_attn       per (split, kv head, b): append this step's k/v at
//                     position lens[b] and attend the group's query heads
//                     over positions [split*64, split*64+64) of 0..lens[b]
//                     (the new position is read from the projection, not the
//                     cache, so no intra-kernel ordering is needed); writes a
//                     partial (max, sum, o) per split
//   decode_combine    merges the splits of each (b, h) into the bf16 output
//   decode_argmax     greedy next token, history append, lens[b] += 1
//
// Query heads are grouped per kv head (grouped-query / multi-query attention
// without repeating K/V). Scores are kept in the log2 domain.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <float.h>
#include <stdint.h>

#include "launch_count.h"

namespace g2b {
namespace {

constexpr int kChunk = 64;     // positions per split
constexpr int kMaxGroup = 16;  // query heads per kv head

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

__global__ void decode_embed_kernel(const int64_t* tok, const int* lens, const __nv_bfloat16* wte,
                                    const __nv_bfloat16* wpe, float* x, int C) {
  const int b = blockIdx.x;
  const int64_t t = tok[b];
  const int pos = lens[b];
  for (int c = threadIdx.x; c < C; c += blockDim.x)
    x[(int64_t)b * C + c] = bf(wte[t * C + c]) + bf(wpe[(int64_t)pos * C + c]);
}

struct DecodeArgs {
  const __nv_bfloat16* qkv;  // [B, ld] : q (H*64) | k (Hkv*64) | v (Hkv*64)
  int64_t ld;
  __nv_bfloat16* kc;         // [B, Hkv, Tmax, 64]
  __nv_bfloat16* vc;
  const int* lens;           // [B]
  float* part_o;             // [B, H, S, 64]
  float* part_ml;            // [B, H, S, 2]
  __nv_bfloat16* out;        // [B, H*64] (row stride ld_out)
  int64_t ld_out;
  int B, H, Hkv, Tmax, S;
  float scale_log2;          // softmax scale * log2(e)
};

__global__ void __launch_bounds__(128) decode_attn_kernel(const DecodeArgs a) {
  __shared__ float q_s[kMaxGroup][64];
  __shared__ float p_s[kMaxGroup][kChunk];
  __shared__ float red[4][kMaxGroup][64];
  __shared__ float ml_s[kMaxGroup][2];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = a.H / a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = a.lens[b];
  const int p_end = len + 1;  // the new token sits at position len
  const int p0 = split * kChunk;
  const int p1 = min(p0 + kChunk, p_end);
  const __nv_bfloat16* row = a.qkv + (int64_t)b * a.ld;
  const __nv_bfloat16* k_new = row + a.H * 64 + kvh * 64;
  const __nv_bfloat16* v_new = row + (a.H + a.Hkv) * 64 + kvh * 64;
  const int64_t cache_base = ((int64_t)b * a.Hkv + kvh) * a.Tmax * 64;
  const int64_t ml_base = ((int64_t)b * a.H + kvh * G) * a.S + split;

  if (split == len / kChunk && len < a.Tmax) {
    // append this step's key and value (read back only by later launches)
    if (threadIdx.x < 64)
      a.kc[cache_base + (int64_t)len * 64 + threadIdx.x] = k_new[threadIdx.x];
    else
      a.vc[cache_base + (int64_t)len * 64 + threadIdx.x - 64] = v_new[threadIdx.x - 64];
  }
  if (p0 >= p1) {
    // empty split: contributes nothing
    if (threadIdx.x < G) {
      a.part_ml[(ml_base + (int64_t)threadIdx.x * a.S) * 2 + 0] = -FLT_MAX;
      a.part_ml[(ml_base + (int64_t)threadIdx.x * a.S) * 2 + 1] = 0.f;
    }
    return;
  }
  for (int i = threadIdx.x; i < G * 64; i += blockDim.x)
    q_s[i / 64][i % 64] = bf(row[(kvh * G + i / 64) * 64 + (i % 64)]) * a.scale_log2;
  __syncthreads();

  // scores: warp w takes positions p0+w, p0+w+4, ...; lane l owns dims 2l, 2l+1
  for (int p = p0 + warp; p < p1; p += 4) {
    const __nv_bfloat162 k2 = (p == len) ? reinterpret_cast<const __nv_bfloat162*>(k_new)[lane]
                                         : reinterpret_cast<const __nv_bfloat162*>(
                                               a.kc + cache_base + (int64_t)p * 64)[lane];
    const float2 kf = __bfloat1622float2(k2);
    for (int g = 0; g < G; ++g) {
      float s = q_s[g][2 * lane] * kf.x + q_s[g][2 * lane + 1] * kf.y;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (lane == 0) p_s[g][p - p0] = s;
    }
  }
  __syncthreads();
  // per head: chunk max, probabilities, sum
  const int n = p1 - p0;
  for (int g = warp; g < G; g += 4) {
    const float s0 = lane < n ? p_s[g][lane] : -FLT_MAX;
    const float s1 = lane + 32 < n ? p_s[g][lane + 32] : -FLT_MAX;
    float m = fmaxf(s0, s1);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float e0 = lane < n ? exp2f(s0 - m) : 0.f;
    const float e1 = lane + 32 < n ? exp2f(s1 - m) : 0.f;
    if (lane < n) p_s[g][lane] = e0;
    if (lane + 32 < n) p_s[g][lane + 32] = e1;
    float l = e0 + e1;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (lane == 0) {
      ml_s[g][0] = m;
      ml_s[g][1] = l;
    }
  }
  __syncthreads();
  // P V: warp w takes positions p0+w, p0+w+4, ...
  float acc[kMaxGroup][2];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) acc[g][0] = acc[g][1] = 0.f;
  for (int p = p0 + warp; p < p1; p += 4) {
    const __nv_bfloat162 v2 = (p == len) ? reinterpret_cast<const __nv_bfloat162*>(v_new)[lane]
                                         : reinterpret_cast<const __nv_bfloat162*>(
                                               a.vc + cache_base + (int64_t)p * 64)[lane];
    const float2 vf = __bfloat1622float2(v2);
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      if (g < G) {
        const float pr = p_s[g][p - p0];
        acc[g][0] = fmaf(pr, vf.x, acc[g][0]);
        acc[g][1] = fmaf(pr, vf.y, acc[g][1]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g < G) {
      red[warp][g][2 * lane] = acc[g][0];
      red[warp][g][2 * lane + 1] = acc[g][1];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * 64; i += blockDim.x) {
    const int g = i / 64, d = i % 64;
    const float o = red[0][g][d] + red[1][g][d] + red[2][g][d] + red[3][g][d];
    a.part_o[(ml_base + (int64_t)g * a.S) * 64 + d] = o;
  }
  if (threadIdx.x < G) {
    a.part_ml[(ml_base + (int64_t)threadIdx.x * a.S) * 2 + 0] = ml_s[threadIdx.x][0];
    a.part_ml[(ml_base + (int64_t)threadIdx.x * a.S) * 2 + 1] = ml_s[threadIdx.x][1];
  }
}

// Restructured form of decode_attn_kernel (same append, same per-split
// partials, so decode_combine is shared). Selected with decode_set_impl(2);
// the default stays decode_attn_kernel until this one has been A/B-tested on
// a GPU. A warp covers four positions at once: 8 lanes a position, each lane
// one 16-byte vector (8 dims) of the key or value row, so a score needs a
// 3-step shuffle tree (5 steps for one position a warp before) and every
// load moves 16 bytes (4 before). Query groups of up to kMaxGroupV2 heads.
constexpr int kMaxGroupV2 = 4;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& w, float* f) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[i]));
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__global__ void __launch_bounds__(128) decode_attn_v2_kernel(const DecodeArgs a) {
  __shared__ __align__(16) float q_s[kMaxGroupV2][64];
  __shared__ float p_s[kMaxGroupV2][kChunk];
  __shared__ float red[4][kMaxGroupV2][64];
  __shared__ float ml_s[kMaxGroupV2][2];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = a.H / a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane >> 3;      // position slot of this lane within the warp
  const int d0 = (lane & 7) * 8;  // this lane's 8 dims
  const int len = a.lens[b];
  const int p_end = len + 1;
  const int p0 = split * kChunk;
  const int p1 = min(p0 + kChunk, p_end);
  const __nv_bfloat16* row = a.qkv + (int64_t)b * a.ld;
  const __nv_bfloat16* k_new = row + a.H * 64 + kvh * 64;
  const __nv_bfloat16* v_new = row + (a.H + a.Hkv) * 64 + kvh * 64;
  const int64_t cache_base = ((int64_t)b * a.Hkv + kvh) * a.Tmax * 64;
  const int64_t ml_base = ((int64_t)b * a.H + kvh * G) * a.S + split;

  if (split == len / kChunk && len < a.Tmax) {
    if (threadIdx.x < 64)
      a.kc[cache_base + (int64_t)len * 64 + threadIdx.x] = k_new[threadIdx.x];
    else
      a.vc[cache_base + (int64_t)len * 64 + threadIdx.x - 64] = v_new[threadIdx.x - 64];
  }
  if (p0 >= p1) {
    if (threadIdx.x < G) {
      a.part_ml[(ml_base + (int64_t)threadIdx.x * a.S) * 2 + 0] = -FLT_MAX;
      a.part_ml[(ml_base + (int64_t)threadIdx.x * a.S) * 2 + 1] = 0.f;
    }
    return;
  }
  for (int i = threadIdx.x; i < G * 64; i += blockDim.x)
    q_s[i / 64][i % 64] = bf(row[(kvh * G + i / 64) * 64 + (i % 64)]) * a.scale_log2;
  __syncthreads();

  // scores: warp w, iteration t -> positions p0 + 16 t + 4 w + sub
  for (int pb = p0 + warp * 4; pb < p1; pb += 16) {
    const int p = pb + sub;
    const bool valid = p < p1;
    uint4 kw = make_uint4(0u, 0u, 0u, 0u);
    if (valid)
      kw = (p == len) ? *reinterpret_cast<const uint4*>(k_new + d0)
                      : *reinterpret_cast<const uint4*>(a.kc + cache_base + (int64_t)p * 64 + d0);
    float kf[8];
    bf16x8_to_f32(kw, kf);
#pragma unroll
    for (int g = 0; g < kMaxGroupV2; ++g) {
      if (g < G) {
        const float4 qa = *reinterpret_cast<const float4*>(&q_s[g][d0]);
        const float4 qb = *reinterpret_cast<const float4*>(&q_s[g][d0 + 4]);
        float s = qa.x * kf[0] + qa.y * kf[1] + qa.z * kf[2] + qa.w * kf[3] + qb.x * kf[4] +
                  qb.y * kf[5] + qb.z * kf[6] + qb.w * kf[7];
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (valid && (lane & 7) == 0) p_s[g][p - p0] = s;
      }
    }
  }
  __syncthreads();
  const int n = p1 - p0;
  for (int g = warp; g < G; g += 4) {
    const float s0 = lane < n ? p_s[g][lane] : -FLT_MAX;
    const float s1 = lane + 32 < n ? p_s[g][lane + 32] : -FLT_MAX;
    float m = fmaxf(s0, s1);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float e0 = lane < n ? exp2f(s0 - m) : 0.f;
    const float e1 = lane + 32 < n ? exp2f(s1 - m) : 0.f;
    if (lane < n) p_s[g][lane] = e0;
    if (lane + 32 < n) p_s[g][lane + 32] = e1;
    float l = e0 + e1;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (lane == 0) {
      ml_s[g][0] = m;
      ml_s[g][1] = l;
    }
  }
  __syncthreads();
  // P V: the same position slots; each lane accumulates its 8 value dims
  float acc[kMaxGroupV2][8];
#pragma unroll
  for (int g = 0; g < kMaxGroupV2; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[g][i] = 0.f;
  for (int pb = p0 + warp * 4; pb < p1; pb += 16) {
    const int p = pb + sub;
    if (p < p1) {
      const uint4 vw = (p == len) ? *reinterpret_cast<const uint4*>(v_new + d0)
                                  : *reinterpret_cast<const uint4*>(a.vc + cache_base + (int64_t)p * 64 + d0);
      float vf[8];
      bf16x8_to_f32(vw, vf);
#pragma unroll
      for (int g = 0; g < kMaxGroupV2; ++g) {
        if (g < G) {
          const float pr = p_s[g][p - p0];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[g][i] = fmaf(pr, vf[i], acc[g][i]);
        }
      }
    }
  }
  // the warp's four position slots hold the same dims: fold them
#pragma unroll
  for (int g = 0; g < kMaxGroupV2; ++g) {
    if (g < G) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        acc[g][i] += __shfl_xor_sync(0xffffffffu, acc[g][i], 8);
        acc[g][i] += __shfl_xor_sync(0xffffffffu, acc[g][i], 16);
      }
      if (sub == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) red[warp][g][d0 + i] = acc[g][i];
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * 64; i += blockDim.x) {
    const int g = i / 64, d = i % 64;
    const float o = red[0][g][d] + red[1][g][d] + red[2][g][d] + red[3][g][d];
    a.part_o[(ml_base + (int64_t)g * a.S) * 64 + d] = o;
  }
  if (threadIdx.x < G) {
    a.part_ml[(ml_base + (int64_t)threadIdx.x * a.S) * 2 + 0] = ml_s[threadIdx.x][0];
    a.part_ml[(ml_base + (int64_t)threadIdx.x * a.S) * 2 + 1] = ml_s[threadIdx.x][1];
  }
}

int g_decode_impl = 1;

__global__ void decode_combine_kernel(const DecodeArgs a) {
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;  // 64 threads
  const int64_t base = ((int64_t)b * a.H + h) * a.S;
  float m = -FLT_MAX;
  for (int s = 0; s < a.S; ++s) m = fmaxf(m, a.part_ml[(base + s) * 2]);
  float l = 0.f, o = 0.f;
  for (int s = 0; s < a.S; ++s) {
    const float ls = a.part_ml[(base + s) * 2 + 1];
    if (ls == 0.f) continue;
    const float w = exp2f(a.part_ml[(base + s) * 2] - m);
    l = fmaf(ls, w, l);
    o = fmaf(a.part_o[(base + s) * 64 + d], w, o);
  }
  a.out[(int64_t)b * a.ld_out + h * 64 + d] = __float2bfloat16(l > 0.f ? o / l : 0.f);
}

// Greedy next token of row b; appends it to the history and advances lens[b].
__global__ void __launch_bounds__(1024) decode_argmax_kernel(const __nv_bfloat16* logits, int64_t ld,
                                                             int V, int64_t* tok, int* lens,
                                                             int64_t* hist, int Tmax) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int b = blockIdx.x;
  const __nv_bfloat16* row = logits + (int64_t)b * ld;
  float best = -FLT_MAX;
  int bi = 0;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = bf(row[i]);
    if (v > best) {  // strictly greater: the lowest index wins ties within a thread
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -FLT_MAX;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      const int pos = lens[b] + 1;  // position of the new token
      tok[b] = bi;
      if (pos < Tmax) hist[(int64_t)b * Tmax + pos] = bi;
      lens[b] = pos;
    }
  }
}

}  // namespace

int decode_embed_launch(const int64_t* tok, const int* lens, const void* wte, const void* wpe, float* x,
                        int B, int C, cudaStream_t s) {
  decode_embed_kernel<<<B, 256, 0, s>>>(tok, lens, reinterpret_cast<const __nv_bfloat16*>(wte),
                                        reinterpret_cast<const __nv_bfloat16*>(wpe), x, C);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int decode_attn_launch(const void* qkv, int64_t ld, void* kc, void* vc, const int* lens, float* part_o,
                       float* part_ml, void* out, int64_t ld_out, int B, int H, int Hkv, int Tmax,
                       float scale, cudaStream_t s) {
  if (Hkv <= 0 || H % Hkv || H / Hkv > kMaxGroup || B <= 0 || Tmax <= 0) return -1;
  DecodeArgs a;
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv);
  a.ld = ld;
  a.kc = reinterpret_cast<__nv_bfloat16*>(kc);
  a.vc = reinterpret_cast<__nv_bfloat16*>(vc);
  a.lens = lens;
  a.part_o = part_o;
  a.part_ml = part_ml;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.ld_out = ld_out;
  a.B = B;
  a.H = H;
  a.Hkv = Hkv;
  a.Tmax = Tmax;
  a.S = (Tmax + kChunk - 1) / kChunk;
  a.scale_log2 = scale * 1.4426950408889634f;
  // the restructured kernel reads 16-byte vectors of the projection row
  const bool v2 = g_decode_impl == 2 && H / Hkv <= kMaxGroupV2 && ld % 8 == 0 &&
                  (reinterpret_cast<uintptr_t>(qkv) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(kc) & 15) == 0 && (reinterpret_cast<uintptr_t>(vc) & 15) == 0;
  if (v2)
    decode_attn_v2_kernel<<<dim3(a.S, Hkv, B), 128, 0, s>>>(a);
  else
    decode_attn_kernel<<<dim3(a.S, Hkv, B), 128, 0, s>>>(a);
  decode_combine_kernel<<<dim3(H, B), 64, 0, s>>>(a);
  count_launches(2);
  return launch_succeeded() ? 0 : -11;
}

void decode_set_impl(int impl) { g_decode_impl = impl == 2 ? 2 : 1; }
int decode_get_impl() { return g_decode_impl; }

int decode_partials_numel(int B, int H, int Tmax) {
  return B * H * ((Tmax + kChunk - 1) / kChunk) * 64;
}

int decode_argmax_launch(const void* logits, int64_t ld, int V, int64_t* tok, int* lens, int64_t* hist,
                         int Tmax, int B, cudaStream_t s) {
  decode_argmax_kernel<<<B, 1024, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(logits), ld, V, tok,
                                          lens, hist, Tmax);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

}  // namespace g2b
