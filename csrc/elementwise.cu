// Memory-bound kernels of the GPT-2 training step (sm_100a).
//
// Reference ops covered (src/transformer_internals/...):
//   model.py:382,384,473   nn.LayerNorm (eps 1e-5)        -> layernorm_fwd / _bwd
//   model.py:561-564       wte[idx] + wpe[pos]             -> embedding_fwd / _bwd
//   model.py:593-598       F.cross_entropy(ignore -100)    -> cross_entropy_fwd_bwd
//   zero.py:158-186        AdamW (torch single-tensor order) -> adamw
//   zero.py:194-233        global grad norm + clip coef    -> sumsq / clip_coef
// Every reduction is deterministic (fixed order, no float atomics); the
// token-embedding scatter has an fp32-atomic form for callers that give it no
// workspace and a deterministic two-pass form (emb_det_*) for those that do.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "elementwise.cuh"

namespace g2b {
namespace {

// Store an 8-byte chunk of an output row into every peer copy (RowPush).
__device__ __forceinline__ void push_store(const RowPush& push, const __nv_bfloat16* local_ptr,
                                           uint2 v) {
  const int64_t off = reinterpret_cast<const char*>(local_ptr) -
                      reinterpret_cast<const char*>(push.local);
  for (int j = 0; j < push.n; ++j)
    *reinterpret_cast<uint2*>(reinterpret_cast<char*>(push.bases[j]) + off) = v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}

int grid_for(int64_t work, int per_block, int cap = 148 * 16) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (int)g;
}

// --------------------------------------------------------------- LayerNorm ---
constexpr int LN_MAXV_CAP = 16;  // float4 per lane -> C <= 2048

// Smallest compiled float4-per-lane count covering C (keeps registers tight).
template <typename F>
int ln_dispatch(int C, F&& f) {
  const int need = (C / 4 + 31) / 32;
  if (need <= 1) return f(std::integral_constant<int, 1>{});
  if (need <= 2) return f(std::integral_constant<int, 2>{});
  if (need <= 4) return f(std::integral_constant<int, 4>{});
  if (need <= 6) return f(std::integral_constant<int, 6>{});
  if (need <= 8) return f(std::integral_constant<int, 8>{});
  if (need <= 10) return f(std::integral_constant<int, 10>{});
  if (need <= 13) return f(std::integral_constant<int, 13>{});
  return f(std::integral_constant<int, 16>{});
}

template <int LN_MAXV, bool PUSH>
__global__ void __launch_bounds__(256) ln_fwd_kernel(const float* __restrict__ x, int64_t ldx,
                                                     const __nv_bfloat16* __restrict__ g,
                                                     const __nv_bfloat16* __restrict__ bta,
                                                     __nv_bfloat16* __restrict__ y, int64_t ldy,
                                                     float* __restrict__ mean,
                                                     float* __restrict__ rstd, int M, int C,
                                                     float eps, const RowPush push) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int C4 = C >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (int64_t)row * ldx);
  float4 v[LN_MAXV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int c = lane + 32 * i;
    if (c < C4) {
      v[i] = xr[c];
      s += v[i].x + v[i].y + v[i].z + v[i].w;
    }
  }
  const float mu = warp_sum(s) / C;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int c = lane + 32 * i;
    if (c < C4) {
      const float a = v[i].x - mu, b = v[i].y - mu, cc = v[i].z - mu, d = v[i].w - mu;
      q += a * a + b * b + cc * cc + d * d;
    }
  }
  const float var = warp_sum(q) / C;
  const float rs = rsqrtf(var + eps);
  __nv_bfloat16* yr = y + (int64_t)row * ldy;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int c = lane + 32 * i;
    if (c < C4) {
      const uint2 gw = *reinterpret_cast<const uint2*>(g + 4 * c);
      const uint2 bw = *reinterpret_cast<const uint2*>(bta + 4 * c);
      const float2 g01 = unpack_bf16x2(gw.x), g23 = unpack_bf16x2(gw.y);
      const float2 b01 = unpack_bf16x2(bw.x), b23 = unpack_bf16x2(bw.y);
      uint2 o;
      o.x = pack_bf16x2((v[i].x - mu) * rs * g01.x + b01.x, (v[i].y - mu) * rs * g01.y + b01.y);
      o.y = pack_bf16x2((v[i].z - mu) * rs * g23.x + b23.x, (v[i].w - mu) * rs * g23.y + b23.y);
      *reinterpret_cast<uint2*>(yr + 4 * c) = o;
      if (PUSH) push_store(push, yr + 4 * c, o);
    }
  }
  if (lane == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
  if (PUSH) __threadfence_system();  // pushed rows visible before any later signal
}

// LayerNorm backward, one warp per row, CTAs in clusters of LNB_CLUSTER.
//
// Per row: dx = rstd * (g*dy - mean(g*dy) - xhat * mean(g*dy*xhat)), written
// to (or added into) the fp32 residual gradient together with its bf16 copy.
// The column sums dgamma = sum dy*xhat, dbeta = sum dy and (optionally)
// dsum = sum dres_out -- the bias gradient of the projection whose output fed
// this residual stream -- are accumulated per warp in shared memory, reduced
// across the CTA's 8 warps, then across the cluster's CTAs through
// distributed shared memory, so each cluster writes ONE partial row
// [3][C]; ln_param_reduce_kernel adds the per-cluster rows in fixed order.
// Every load of a row (x, dy and the old dres) is issued before its two
// reductions, so a warp keeps ~3 row-loads in flight.
constexpr int LNB_WARPS = 8;
constexpr int LNB_CLUSTER = 8;
constexpr int LNB_NSUM = 3;  // dgamma, dbeta, dsum

template <int LN_MAXV, bool PUSH>
__global__ void __cluster_dims__(LNB_CLUSTER, 1, 1) __launch_bounds__(256) ln_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, const float* __restrict__ x,
    const float* __restrict__ mean, const float* __restrict__ rstd,
    const __nv_bfloat16* __restrict__ g, float* __restrict__ dres,
    __nv_bfloat16* __restrict__ dres_bf16, float* __restrict__ partials, int M, int C,
    int accumulate, int with_dsum, const RowPush push) {
  extern __shared__ float4 sacc[];  // [LNB_WARPS][LNB_NSUM][C/4]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C4 = C >> 2;
  const int nsum4 = LNB_NSUM * C4;
  float4* my = sacc + warp * nsum4;
  for (int c = lane; c < nsum4; c += 32) my[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  uint2 gw[LN_MAXV];
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int c = lane + 32 * i;
    gw[i] = c < C4 ? *reinterpret_cast<const uint2*>(g + 4 * c) : make_uint2(0, 0);
  }
  const int rpc = (M + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * rpc, r1 = min(M, r0 + rpc);
  for (int row = r0 + warp; row < r1; row += LNB_WARPS) {
    const float mu = __ldg(mean + row), rs = __ldg(rstd + row);
    const float4* xr = reinterpret_cast<const float4*>(x + (int64_t)row * C);
    const __nv_bfloat16* dyr = dy + (int64_t)row * C;
    float4* dr = reinterpret_cast<float4*>(dres + (int64_t)row * C);
    float4 xv[LN_MAXV], ov[LN_MAXV];
    uint2 dw[LN_MAXV];
#pragma unroll
    for (int i = 0; i < LN_MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < C4) {
        xv[i] = __ldcs(xr + c);
        dw[i] = __ldcs(reinterpret_cast<const uint2*>(dyr + 4 * c));
        ov[i] = accumulate ? __ldcs(dr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < LN_MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < C4) {
        const float2 d01 = unpack_bf16x2(dw[i].x), d23 = unpack_bf16x2(dw[i].y);
        const float2 g01 = unpack_bf16x2(gw[i].x), g23 = unpack_bf16x2(gw[i].y);
        // xv becomes xhat, dw is kept; gy is recomputed below from dw and gw
        xv[i] = make_float4((xv[i].x - mu) * rs, (xv[i].y - mu) * rs, (xv[i].z - mu) * rs,
                            (xv[i].w - mu) * rs);
        const float gy0 = d01.x * g01.x, gy1 = d01.y * g01.y, gy2 = d23.x * g23.x,
                    gy3 = d23.y * g23.y;
        s1 += gy0 + gy1 + gy2 + gy3;
        s2 += gy0 * xv[i].x + gy1 * xv[i].y + gy2 * xv[i].z + gy3 * xv[i].w;
      }
    }
    s1 = warp_sum(s1) / C;
    s2 = warp_sum(s2) / C;
    __nv_bfloat16* db16 = dres_bf16 ? dres_bf16 + (int64_t)row * C : nullptr;
#pragma unroll
    for (int i = 0; i < LN_MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < C4) {
        const float2 d01 = unpack_bf16x2(dw[i].x), d23 = unpack_bf16x2(dw[i].y);
        const float2 g01 = unpack_bf16x2(gw[i].x), g23 = unpack_bf16x2(gw[i].y);
        const float4 xh = xv[i];
        float4 d = make_float4(rs * (d01.x * g01.x - s1 - xh.x * s2),
                               rs * (d01.y * g01.y - s1 - xh.y * s2),
                               rs * (d23.x * g23.x - s1 - xh.z * s2),
                               rs * (d23.y * g23.y - s1 - xh.w * s2));
        d.x += ov[i].x;
        d.y += ov[i].y;
        d.z += ov[i].z;
        d.w += ov[i].w;
        dr[c] = d;
        if (db16) {
          uint2 w;
          w.x = pack_bf16x2(d.x, d.y);
          w.y = pack_bf16x2(d.z, d.w);
          *reinterpret_cast<uint2*>(db16 + 4 * c) = w;
          if (PUSH) push_store(push, db16 + 4 * c, w);
        }
        float4 a = my[c];
        a.x += d01.x * xh.x;
        a.y += d01.y * xh.y;
        a.z += d23.x * xh.z;
        a.w += d23.y * xh.w;
        my[c] = a;
        float4 b = my[C4 + c];
        b.x += d01.x;
        b.y += d01.y;
        b.z += d23.x;
        b.w += d23.y;
        my[C4 + c] = b;
        if (with_dsum) {
          float4 e = my[2 * C4 + c];
          e.x += d.x;
          e.y += d.y;
          e.z += d.z;
          e.w += d.w;
          my[2 * C4 + c] = e;
        }
      }
    }
  }
  if (PUSH) __threadfence_system();  // pushed rows visible before any later signal
  __syncthreads();
  // CTA: fold the 8 warps' sums into warp 0's slot (fixed order).
  for (int c = threadIdx.x; c < nsum4; c += blockDim.x) {
    float4 t = sacc[c];
#pragma unroll
    for (int w = 1; w < LNB_WARPS; ++w) {
      const float4 u = sacc[w * nsum4 + c];
      t.x += u.x;
      t.y += u.y;
      t.z += u.z;
      t.w += u.w;
    }
    sacc[c] = t;
  }
  cluster_sync_all();
  // Cluster: CTA k adds chunk k of the columns across the cluster's CTAs
  // through DSMEM, in rank order, and writes the cluster's partial row.
  const uint32_t rank = cluster_ctarank();
  const int per = (nsum4 + LNB_CLUSTER - 1) / LNB_CLUSTER;
  const int c0 = rank * per, c1 = min(nsum4, c0 + per);
  float4* out = reinterpret_cast<float4*>(partials) + (int64_t)cluster_id_x() * nsum4;
  for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
    const uint32_t local = smem_u32(sacc + c);
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < LNB_CLUSTER; ++q) {
      const float4 u = ld_shared_cluster_f4(map_shared_rank(local, q));
      t.x += u.x;
      t.y += u.y;
      t.z += u.z;
      t.w += u.w;
    }
    out[c] = t;
  }
  cluster_sync_all();  // peers' shared memory must outlive the reads above
}

// dgamma/dbeta/dsum (+)= sum over the P per-cluster rows of partials[P][3][C]
// (fixed row order). Block = 32 columns x 8 row lanes.
__global__ void __launch_bounds__(256) ln_param_reduce_kernel(
    const float* __restrict__ partials, int P, int C, float* __restrict__ dgamma,
    float* __restrict__ dbeta, float* __restrict__ dsum, int acc_params, int acc_sum) {
  __shared__ float red[8][33];
  const int n = (dsum ? 3 : 2) * C;
  const int c = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (c < n) {
#pragma unroll 4
    for (int r = threadIdx.y; r < P; r += 8) s += partials[(int64_t)r * 3 * C + c];
  }
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < n) {
    float t = 0.f;
#pragma unroll
    for (int y = 0; y < 8; ++y) t += red[y][threadIdx.x];
    if (c < C) {
      dgamma[c] = acc_params ? dgamma[c] + t : t;
    } else if (c < 2 * C) {
      dbeta[c - C] = acc_params ? dbeta[c - C] + t : t;
    } else {
      dsum[c - 2 * C] = acc_sum ? dsum[c - 2 * C] + t : t;
    }
  }
}

// out[c] (+)= sum_r in[r*C + c]. Block = 32 columns x 8 row lanes; each
// lane sums rows y, y+8, ... (several loads in flight), then the 8 lane sums
// are added in fixed order through shared memory: deterministic.
__global__ void __launch_bounds__(256) colsum_f32_kernel(const float* __restrict__ in, int R, int C,
                                                         float* __restrict__ out, int accumulate) {
  __shared__ float red[8][33];
  const int c = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (c < C) {
#pragma unroll 4
    for (int r = threadIdx.y; r < R; r += 8) s += __ldg(in + (int64_t)r * C + c);
  }
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < C) {
    float t = 0.f;
#pragma unroll
    for (int y = 0; y < 8; ++y) t += red[y][threadIdx.x];
    out[c] = accumulate ? out[c] + t : t;
  }
}

constexpr int COLSUM_ROWS = 128;  // rows per partial in the bf16 column sum

// Partial column sums of bf16 in[M, C] over COLSUM_ROWS-row chunks into
// ws[chunk, C]. Block = 32 column groups of 8 (one 16-byte load each) x 8 row
// lanes; fixed-order reduction across the lanes.
__global__ void __launch_bounds__(256) colsum_bf16_partial_kernel(
    const __nv_bfloat16* __restrict__ in, int64_t ld, int M, int C, float* __restrict__ ws) {
  __shared__ float red[8][32 * 8 + 4];
  const int cg = blockIdx.x * 32 + threadIdx.x;  // 8-column group
  const bool active = cg * 8 < C;
  const int r0 = blockIdx.y * COLSUM_ROWS;
  const int r1 = min(M, r0 + COLSUM_ROWS);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  if (active) {
#pragma unroll 4
    for (int r = r0 + threadIdx.y; r < r1; r += 8) {
      const uint4 w = __ldcs(reinterpret_cast<const uint4*>(in + (int64_t)r * ld + cg * 8));
      const uint32_t ws4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(ws4[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[threadIdx.y][threadIdx.x * 8 + j] = acc[j];
  __syncthreads();
  // 256 threads finish 256 columns of this block (32 groups x 8)
  const int t = threadIdx.y * 32 + threadIdx.x;
  const int col = blockIdx.x * 256 + t;
  if (col < C) {
    float sum = 0.f;
#pragma unroll
    for (int y = 0; y < 8; ++y) sum += red[y][t];
    ws[(int64_t)blockIdx.y * C + col] = sum;
  }
}

// --------------------------------------------------------------- embedding ---
// Position of column t of a sequence: pos0 + t below `split`, pos1 + (t -
// split) from it on (a sequence assembled from two separate chunks of the
// full context, as in load-balanced context parallelism).
__device__ __forceinline__ int emb_pos(int t, int pos0, int split, int pos1) {
  return t < split ? pos0 + t : pos1 + (t - split);
}

__global__ void emb_fwd_kernel(const int64_t* __restrict__ idx, const __nv_bfloat16* __restrict__ wte,
                               const __nv_bfloat16* __restrict__ wpe, float* __restrict__ x, int B,
                               int T, int C, int pos0, int split, int pos1) {
  const int64_t total = (int64_t)B * T * (C / 4);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / (C / 4);
    const int c = (int)(i % (C / 4)) * 4;
    const int t = (int)(m % T);
    const int64_t tok = idx[m];
    const uint2 a = *reinterpret_cast<const uint2*>(wte + tok * C + c);
    const uint2 p =
        *reinterpret_cast<const uint2*>(wpe + (int64_t)emb_pos(t, pos0, split, pos1) * C + c);
    const float2 a01 = unpack_bf16x2(a.x), a23 = unpack_bf16x2(a.y);
    const float2 p01 = unpack_bf16x2(p.x), p23 = unpack_bf16x2(p.y);
    reinterpret_cast<float4*>(x)[i] =
        make_float4(a01.x + p01.x, a01.y + p01.y, a23.x + p23.x, a23.y + p23.y);
  }
}

__global__ void emb_bwd_wte_kernel(const int64_t* __restrict__ idx, const float* __restrict__ dx,
                                   float* __restrict__ wte_grad, int64_t M, int C, int V) {
  const int64_t total = M * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / C;
    const int c = (int)(i % C);
    const int64_t tok = idx[m];
    if (tok >= 0 && tok < V) atomicAdd(wte_grad + tok * C + c, dx[i]);
  }
}

__global__ void emb_bwd_wpe_kernel(const float* __restrict__ dx, float* __restrict__ wpe_grad,
                                   int B, int T, int C, int pos0, int split, int pos1) {
  const int64_t total = (int64_t)T * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / C), c = (int)(i % C);
    float s = 0.f;
    for (int b = 0; b < B; ++b) s += dx[((int64_t)b * T + t) * C + c];
    wpe_grad[(int64_t)emb_pos(t, pos0, split, pos1) * C + c] += s;
  }
}

// Deterministic token-embedding gradient: wte_grad[v] += sum of dx[m] over
// the positions m with idx[m] == v, always summed in the same order, so the
// result is bit-reproducible (the atomic scatter above is not).
//   pass A  one CTA per chunk of EMB_CHUNK consecutive positions: the first
//           occurrence of each token in the chunk sums that token's rows of
//           the chunk in position order into part[m_first] and records
//           slots[chunk][token] = m_first;
//   pass B  one warp per vocabulary row: adds its chunks' partials in chunk
//           order into wte_grad and resets the slots it used to -1.
// The slot table [chunks, V] must hold -1 everywhere before pass A; pass B
// leaves it so.
constexpr int EMB_CHUNK = 128;
constexpr int EMB_MAXV4 = 13;  // float4 per lane: C <= 32 * 4 * 13 = 1664

__global__ void __launch_bounds__(256) emb_det_partial_kernel(const int64_t* __restrict__ idx,
                                                              const float* __restrict__ dx,
                                                              int64_t M, int C, int V,
                                                              float* __restrict__ part,
                                                              int* __restrict__ slots) {
  __shared__ int tok[EMB_CHUNK];
  __shared__ int nxt[EMB_CHUNK];  // next position of the same token in the chunk, or -1
  __shared__ int lead[EMB_CHUNK];
  const int64_t m0 = (int64_t)blockIdx.x * EMB_CHUNK;
  const int n = (int)min((int64_t)EMB_CHUNK, M - m0);
  for (int i = threadIdx.x; i < EMB_CHUNK; i += blockDim.x) {
    int t = -1;
    if (i < n) {
      const int64_t v = idx[m0 + i];
      t = (v >= 0 && v < V) ? (int)v : -1;
    }
    tok[i] = t;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int t = tok[i];
    int first = t >= 0, after = -1;
    for (int j = 0; j < i && first; ++j) first = tok[j] != t;
    for (int j = i + 1; j < n && t >= 0; ++j)
      if (tok[j] == t) {
        after = j;
        break;
      }
    lead[i] = first;
    nxt[i] = after;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int i = warp; i < n; i += nw) {
    if (!lead[i]) continue;
    float4 acc[EMB_MAXV4];
#pragma unroll
    for (int u = 0; u < EMB_MAXV4; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = i; j >= 0; j = nxt[j]) {  // this token's positions, ascending
      const float4* row = reinterpret_cast<const float4*>(dx + (m0 + j) * C);
#pragma unroll
      for (int u = 0; u < EMB_MAXV4; ++u) {
        const int c4 = lane + 32 * u;
        if (c4 * 4 < C) {
          const float4 w = __ldg(row + c4);
          acc[u].x += w.x;
          acc[u].y += w.y;
          acc[u].z += w.z;
          acc[u].w += w.w;
        }
      }
    }
    float4* out = reinterpret_cast<float4*>(part + (m0 + i) * C);
#pragma unroll
    for (int u = 0; u < EMB_MAXV4; ++u) {
      const int c4 = lane + 32 * u;
      if (c4 * 4 < C) out[c4] = acc[u];
    }
    if (lane == 0) slots[(int64_t)blockIdx.x * V + tok[i]] = (int)(m0 + i);
  }
}

__global__ void __launch_bounds__(256) emb_det_reduce_kernel(const float* __restrict__ part,
                                                             int* __restrict__ slots,
                                                             int nchunks, int C, int V,
                                                             float* __restrict__ wte_grad) {
  const int v = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (v >= V) return;
  float4 acc[EMB_MAXV4];
#pragma unroll
  for (int u = 0; u < EMB_MAXV4; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
  bool any = false;
  for (int k0 = 0; k0 < nchunks; k0 += 32) {
    const int k = k0 + lane;
    const int sl = k < nchunks ? slots[(int64_t)k * V + v] : -1;
    unsigned hit = __ballot_sync(0xffffffffu, sl >= 0);
    if (sl >= 0) slots[(int64_t)k * V + v] = -1;  // ready for the next call
    while (hit) {  // chunks in ascending order
      const int b = __ffs(hit) - 1;
      hit &= hit - 1;
      const int s = __shfl_sync(0xffffffffu, sl, b);
      const float4* row = reinterpret_cast<const float4*>(part + (int64_t)s * C);
#pragma unroll
      for (int u = 0; u < EMB_MAXV4; ++u) {
        const int c4 = lane + 32 * u;
        if (c4 * 4 < C) {
          const float4 w = row[c4];
          acc[u].x += w.x;
          acc[u].y += w.y;
          acc[u].z += w.z;
          acc[u].w += w.w;
        }
      }
      any = true;
    }
  }
  if (!any) return;
  float4* g = reinterpret_cast<float4*>(wte_grad + (int64_t)v * C);
#pragma unroll
  for (int u = 0; u < EMB_MAXV4; ++u) {
    const int c4 = lane + 32 * u;
    if (c4 * 4 < C) {
      float4 o = g[c4];
      o.x += acc[u].x;
      o.y += acc[u].y;
      o.z += acc[u].z;
      o.w += acc[u].w;
      g[c4] = o;
    }
  }
}

// ----------------------------------------------------------- cross-entropy ---
constexpr int CE_THREADS = 512;

__global__ void __launch_bounds__(CE_THREADS) ce_kernel(__nv_bfloat16* __restrict__ logits,
                                                        int64_t ld,
                                                        const int64_t* __restrict__ targets,
                                                        float* __restrict__ loss_rows, int V,
                                                        int vocab_offset) {
  __shared__ float red_m[CE_THREADS / 32], red_s[CE_THREADS / 32];
  const int64_t row = blockIdx.x;
  __nv_bfloat16* lr = logits + row * ld;
  const int64_t tgt_raw = targets[row];
  const bool ignore = tgt_raw == -100;
  const int64_t tgt = tgt_raw - vocab_offset;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Pass 1: online max / sum-exp over 8-element vectors.
  const int V8 = V / 8;
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < V8; i += CE_THREADS) {
    const uint4 w = reinterpret_cast<const uint4*>(lr)[i];
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 p = unpack_bf16x2(ws[j]);
      f[2 * j] = p.x;
      f[2 * j + 1] = p.y;
    }
    float lm = f[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, f[j]);
    const float nm = fmaxf(m, lm);
    float acc = s * __expf(m - nm);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += __expf(f[j] - nm);
    m = nm;
    s = acc;
  }
  for (int i = V8 * 8 + threadIdx.x; i < V; i += CE_THREADS) {
    const float f = __bfloat162float(lr[i]);
    const float nm = fmaxf(m, f);
    s = s * __expf(m - nm) + __expf(f - nm);
    m = nm;
  }
  // Block reduce (m, s).
  float wm = warp_max(m);
  float ws_ = (m == -INFINITY) ? 0.f : s * __expf(m - wm);
  ws_ = warp_sum(ws_);
  if (lane == 0) {
    red_m[warp] = wm;
    red_s[warp] = ws_;
  }
  __syncthreads();
  float gm = -INFINITY;
  for (int w = 0; w < CE_THREADS / 32; ++w) gm = fmaxf(gm, red_m[w]);
  float gs = 0.f;
  for (int w = 0; w < CE_THREADS / 32; ++w)
    gs += red_m[w] == -INFINITY ? 0.f : red_s[w] * __expf(red_m[w] - gm);
  const float lse = gm + __logf(gs);
  const float inv = 1.f / gs;
  if (threadIdx.x == 0) {
    float l = 0.f;
    if (!ignore && tgt >= 0 && tgt < V) l = lse - __bfloat162float(lr[tgt]);
    loss_rows[row] = ignore ? 0.f : l;
  }
  __syncthreads();  // the target logit is read above before being overwritten below
  // Pass 2: dlogits = softmax - onehot (0 for ignored rows), padded tail zeroed.
  for (int i = threadIdx.x; i < V8; i += CE_THREADS) {
    uint4 w = reinterpret_cast<const uint4*>(lr)[i];
    uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 p = unpack_bf16x2(ws[j]);
      float a = ignore ? 0.f : __expf(p.x - gm) * inv;
      float b = ignore ? 0.f : __expf(p.y - gm) * inv;
      const int64_t c = (int64_t)i * 8 + 2 * j;
      if (!ignore && c == tgt) a -= 1.f;
      if (!ignore && c + 1 == tgt) b -= 1.f;
      ws[j] = pack_bf16x2(a, b);
    }
    reinterpret_cast<uint4*>(lr)[i] = make_uint4(ws[0], ws[1], ws[2], ws[3]);
  }
  for (int i = V8 * 8 + threadIdx.x; i < ld; i += CE_THREADS) {
    float a = 0.f;
    if (i < V && !ignore) {
      a = __expf(__bfloat162float(lr[i]) - gm) * inv;
      if (i == tgt) a -= 1.f;
    }
    lr[i] = __float2bfloat16(a);
  }
}

// Fused lm_head + cross-entropy, step 2 (step 1 is the lm_head GEMM with the
// EPI_CE_STATS epilogue): one warp per row folds the row's (max, sum exp)
// partials into its log-sum-exp and loss. Lane j folds partials j, j+32, ...
// in order, then the 32 lane results are combined in a fixed butterfly order.
__global__ void __launch_bounds__(256) ce_combine_kernel(const float2* __restrict__ stats,
                                                         int nparts, int M,
                                                         const int64_t* __restrict__ targets,
                                                         const float* __restrict__ tgt_logit,
                                                         float* __restrict__ lse_out,
                                                         float* __restrict__ loss_rows) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float m = -INFINITY, s = 0.f;
  for (int j = lane; j < nparts; j += 32) {
    const float2 p = __ldcs(stats + (int64_t)j * M + row);
    if (p.x == -INFINITY) continue;
    const float nm = fmaxf(m, p.x);
    s = s * __expf(m - nm) + p.y * __expf(p.x - nm);
    m = nm;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  if (lane == 0) {
    const float lse = m + __logf(s);
    lse_out[row] = lse;
    loss_rows[row] = targets[row] == -100 ? 0.f : lse - tgt_logit[row];
  }
}

// Step 3: logits -> (softmax - onehot) in place: one read and one write of
// the logits. One warp per row (its log-sum-exp and target loaded once), each
// lane with kCeGradLoads 16-byte vectors (8 bf16 each) in flight. Ignored rows
// and the padded columns [V, ld) become 0.
constexpr int kCeGradLoads = 4;

__device__ __forceinline__ uint4 ce_grad_vec(uint4 w, int col0, int V, float L, int64_t tl,
                                             bool ignore) {
  uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = unpack_bf16x2(ws[j]);
    const int c = col0 + 2 * j;
    const float a = (ignore || c >= V) ? 0.f : __expf(f.x - L) - (c == tl ? 1.f : 0.f);
    const float b = (ignore || c + 1 >= V) ? 0.f : __expf(f.y - L) - (c + 1 == tl ? 1.f : 0.f);
    ws[j] = pack_bf16x2(a, b);
  }
  return make_uint4(ws[0], ws[1], ws[2], ws[3]);
}

__global__ void __launch_bounds__(256) ce_grad_kernel(__nv_bfloat16* __restrict__ logits,
                                                      int64_t ld, int M, int V,
                                                      const float* __restrict__ lse,
                                                      const int64_t* __restrict__ targets,
                                                      int vocab_offset) {
  const int lane = threadIdx.x & 31;
  const int nvec = (int)(ld / 8);
  for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M;
       row += gridDim.x * (blockDim.x >> 5)) {
    const int64_t t = __ldg(targets + row);
    const bool ignore = t == -100;
    const int64_t tl = t - vocab_offset;
    const float L = __ldg(lse + row);
    uint4* rp = reinterpret_cast<uint4*>(logits + (int64_t)row * ld);
    for (int v0 = lane; v0 < nvec; v0 += 32 * kCeGradLoads) {
      uint4 w[kCeGradLoads];
#pragma unroll
      for (int u = 0; u < kCeGradLoads; ++u)
        if (v0 + 32 * u < nvec) w[u] = __ldcs(rp + v0 + 32 * u);
#pragma unroll
      for (int u = 0; u < kCeGradLoads; ++u) {
        const int v = v0 + 32 * u;
        if (v < nvec) __stcs(rp + v, ce_grad_vec(w[u], v * 8, V, L, tl, ignore));
      }
    }
  }
}

__global__ void loss_reduce_kernel(const float* __restrict__ loss_rows,
                                   const int64_t* __restrict__ targets, int M,
                                   float* __restrict__ out) {
  __shared__ float rs[32], rc[32];
  float s = 0.f, c = 0.f;
  for (int i = threadIdx.x; i < M; i += blockDim.x) {
    s += loss_rows[i];
    c += targets[i] != -100 ? 1.f : 0.f;
  }
  s = warp_sum(s);
  c = warp_sum(c);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    rs[warp] = s;
    rc[warp] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float ts = 0.f, tc = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      ts += rs[w];
      tc += rc[w];
    }
    tc = fmaxf(tc, 1.f);
    out[0] = ts / tc;
    out[1] = 1.f / tc;
  }
}

// ------------------------------------------------------------------ AdamW ---
// True when element e lies in one of the sorted, disjoint [lo, hi) decay
// ranges (ranges = [lo0, hi0, lo1, hi1, ...]); a null table means e < n_decay.
__device__ __forceinline__ bool in_decay(int64_t e, int64_t n_decay,
                                         const int64_t* __restrict__ ranges, int nr) {
  if (ranges == nullptr) return e < n_decay;
  int lo = 0, hi = nr;  // find the last range with start <= e
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(ranges + 2 * mid) <= e) lo = mid; else hi = mid;
  }
  return nr > 0 && e >= __ldg(ranges + 2 * lo) && e < __ldg(ranges + 2 * lo + 1);
}

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v,
                             __nv_bfloat16* __restrict__ pb, int64_t n, int64_t n_decay,
                             const int64_t* __restrict__ ranges, int nr,
                             const float* __restrict__ hp, const float* __restrict__ clip) {
  const float lr = hp[0], b1 = hp[1], b2 = hp[2], eps = hp[3], wd = hp[4];
  const float bc1 = hp[5], bc2s = hp[6];
  const float gs = hp[7] * (clip ? clip[0] : 1.f);
  const float step_size = lr / bc1;
  const int64_t n4 = n / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 pv = reinterpret_cast<float4*>(p)[i];
    const float4 gv = reinterpret_cast<const float4*>(g)[i];
    float4 mv = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pp = &pv.x;
    const float* gg = &gv.x;
    float* mm = &mv.x;
    float* vq = &vv.x;
    // Ranges start on 4-element boundaries, so one lookup covers the vector.
    const bool decay = in_decay(i * 4, n_decay, ranges, nr);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gj = gg[j] * gs;
      if (decay) pp[j] *= (1.f - lr * wd);
      mm[j] += (gj - mm[j]) * (1.f - b1);
      vq[j] = vq[j] * b2 + (1.f - b2) * gj * gj;
      const float denom = sqrtf(vq[j]) / bc2s + eps;
      pp[j] += -step_size * (mm[j] / denom);
    }
    reinterpret_cast<float4*>(p)[i] = pv;
    reinterpret_cast<float4*>(m)[i] = mv;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (pb) {
      uint2 w;
      w.x = pack_bf16x2(pv.x, pv.y);
      w.y = pack_bf16x2(pv.z, pv.w);
      reinterpret_cast<uint2*>(pb)[i] = w;
    }
  }
  // tail (n not a multiple of 4)
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const int64_t e = n4 * 4 + threadIdx.x;
    const float gj = g[e] * gs;
    float pj = p[e];
    if (in_decay(e, n_decay, ranges, nr)) pj *= (1.f - lr * wd);
    m[e] += (gj - m[e]) * (1.f - b1);
    v[e] = v[e] * b2 + (1.f - b2) * gj * gj;
    const float denom = sqrtf(v[e]) / bc2s + eps;
    pj += -step_size * (m[e] / denom);
    p[e] = pj;
    if (pb) pb[e] = __float2bfloat16(pj);
  }
}

constexpr int SUMSQ_BLOCKS = 1024;

__global__ void sumsq_partial_kernel(const float* __restrict__ g, int64_t n,
                                     float* __restrict__ ws) {
  __shared__ float red[32];
  float s = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float x = g[i];
    s += x * x;
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    ws[blockIdx.x] = t;
  }
}

__global__ void sum_final_kernel(const float* __restrict__ ws, int n, float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += ws[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    out[0] = t;
  }
}

__global__ void clip_coef_kernel(const float* __restrict__ sumsq, float scale2, float max_norm,
                                 float* __restrict__ clip, float* __restrict__ norm_out) {
  const float norm = sqrtf(sumsq[0] * scale2);
  float c = max_norm / (norm + 1e-6f);
  c = fminf(c, 1.f);
  if (clip) clip[0] = c;
  if (norm_out) norm_out[0] = norm;
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out,
                                     int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16(in[i]);
}
__global__ void cast_bf16_f32_kernel(const __nv_bfloat16* __restrict__ in, float* __restrict__ out,
                                     int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __bfloat162float(in[i]);
}
__global__ void scale_f32_kernel(float* __restrict__ x, int64_t n, float a) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    x[i] *= a;
}

inline int ok() { return launch_succeeded() ? 0 : -11; }

}  // namespace

int layernorm_fwd_launch(const float* x, int64_t ldx, const void* gamma, const void* beta, void* y,
                         int64_t ldy, float* mean, float* rstd, int M, int C, float eps,
                         cudaStream_t s, RowPush push) {
  if (C % 4 || C > 4 * 32 * LN_MAXV_CAP) return -1;
  return ln_dispatch(C, [&](auto nv) {
    auto kern = push.n ? ln_fwd_kernel<decltype(nv)::value, true>
                       : ln_fwd_kernel<decltype(nv)::value, false>;
    kern<<<(M + 7) / 8, 256, 0, s>>>(
        x, ldx, (const __nv_bfloat16*)gamma, (const __nv_bfloat16*)beta, (__nv_bfloat16*)y, ldy,
        mean, rstd, M, C, eps, push);
        count_launches(1);
    return ok();
  });
}

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int layernorm_bwd_ctas(int M) {
  // Two resident CTAs per SM, a whole number of clusters, at least 8 rows each.
  int n = 2 * sm_count();
  const int by_rows = (M + 7) / 8;
  if (n > by_rows) n = by_rows;
  n = (n + LNB_CLUSTER - 1) / LNB_CLUSTER * LNB_CLUSTER;
  return n < LNB_CLUSTER ? LNB_CLUSTER : n;
}

int layernorm_bwd_partial_rows(int M) { return layernorm_bwd_ctas(M) / LNB_CLUSTER; }

int layernorm_bwd_launch(const void* dy, const float* x, const float* mean, const float* rstd,
                         const void* gamma, float* dres, void* dres_bf16, float* partials,
                         float* dgamma, float* dbeta, float* dsum, int M, int C, int accumulate,
                         int acc_params, int acc_sum, cudaStream_t s, RowPush push) {
  if (C % 4 || C > 4 * 32 * LN_MAXV_CAP || M <= 0) return -1;
  const int nblk = layernorm_bwd_ctas(M);
  const int smem = LNB_WARPS * LNB_NSUM * C * (int)sizeof(float);
  const int rc = ln_dispatch(C, [&](auto nv) {
    auto kern = push.n ? ln_bwd_kernel<decltype(nv)::value, true>
                       : ln_bwd_kernel<decltype(nv)::value, false>;
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    kern<<<nblk, 256, smem, s>>>((const __nv_bfloat16*)dy, x, mean, rstd,
                                 (const __nv_bfloat16*)gamma, dres, (__nv_bfloat16*)dres_bf16,
                                 partials, M, C, accumulate, dsum != nullptr, push);
    count_launches(1);
    return ok();
  });
  if (rc) return rc;
  const int n = (dsum ? 3 : 2) * C;
  ln_param_reduce_kernel<<<(n + 31) / 32, dim3(32, 8), 0, s>>>(
      partials, nblk / LNB_CLUSTER, C, dgamma, dbeta, dsum, acc_params, acc_sum);
  count_launches(1);
  return ok();
}

int colsum_f32_launch(const float* in, int R, int C, float* out, int accumulate, cudaStream_t s) {
  colsum_f32_kernel<<<(C + 31) / 32, dim3(32, 8), 0, s>>>(in, R, C, out, accumulate);
  count_launches(1);
  return ok();
}

int colsum_bf16_launch(const void* in, int64_t ld, int M, int C, float* ws, float* out,
                       int accumulate, cudaStream_t s) {
  if (C % 8 || ld % 8 || (reinterpret_cast<uintptr_t>(in) & 15)) return -1;
  const int chunks = (M + COLSUM_ROWS - 1) / COLSUM_ROWS;
  dim3 grid((C + 255) / 256, chunks);
  colsum_bf16_partial_kernel<<<grid, dim3(32, 8), 0, s>>>((const __nv_bfloat16*)in, ld, M, C, ws);
  count_launches(1);
  colsum_f32_kernel<<<(C + 31) / 32, dim3(32, 8), 0, s>>>(ws, chunks, C, out, accumulate);
  count_launches(1);
  return ok();
}

int embedding_fwd_launch(const int64_t* idx, const void* wte, const void* wpe, float* x, int B,
                         int T, int C, int pos0, int split, int pos1, cudaStream_t s) {
  if (C % 4 || split < 0 || split > T || pos0 < 0 || pos1 < 0) return -1;
  emb_fwd_kernel<<<grid_for((int64_t)B * T * C / 4, 256), 256, 0, s>>>(
      idx, (const __nv_bfloat16*)wte, (const __nv_bfloat16*)wpe, x, B, T, C, pos0, split, pos1);
  count_launches(1);
  return ok();
}

int embedding_wte_det_chunks(int64_t M) { return (int)((M + EMB_CHUNK - 1) / EMB_CHUNK); }

int embedding_bwd_launch(const int64_t* idx, const float* dx, float* wte_grad, float* wpe_grad,
                         int B, int T, int C, int V, int pos0, int split, int pos1, cudaStream_t s,
                         float* det_part, int* det_slots) {
  if (split < 0 || split > T || pos0 < 0 || pos1 < 0) return -1;
  const int64_t M = (int64_t)B * T;
  if (wte_grad && det_part && det_slots) {
    if (C % 4 || C > 4 * 32 * EMB_MAXV4) return -1;
    const int nchunks = embedding_wte_det_chunks(M);
    emb_det_partial_kernel<<<nchunks, 256, 0, s>>>(idx, dx, M, C, V, det_part, det_slots);
    emb_det_reduce_kernel<<<(V + 7) / 8, 256, 0, s>>>(det_part, det_slots, nchunks, C, V, wte_grad);
    count_launches(2);
  } else if (wte_grad) {
    emb_bwd_wte_kernel<<<grid_for(M * C, 256), 256, 0, s>>>(idx, dx, wte_grad, M, C, V);
    count_launches(1);
  }
  if (wpe_grad) {
    emb_bwd_wpe_kernel<<<grid_for((int64_t)T * C, 256), 256, 0, s>>>(dx, wpe_grad, B, T, C, pos0,
                                                                     split, pos1);
    count_launches(1);
  }
  return ok();
}

int cross_entropy_fwd_bwd_launch(void* logits, int64_t ld, const int64_t* targets,
                                 float* loss_rows, int M, int V, int vocab_offset,
                                 cudaStream_t s) {
  if (ld % 8 || (reinterpret_cast<uintptr_t>(logits) & 15)) return -1;
  ce_kernel<<<M, CE_THREADS, 0, s>>>((__nv_bfloat16*)logits, ld, targets, loss_rows, V,
                                     vocab_offset);
                                     count_launches(1);
  return ok();
}

__global__ void exp2_fma_test_kernel(const float* __restrict__ x, float* __restrict__ y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = exp2_fma(x[i]);
}

// exp2_fma (common.cuh) elementwise, for the numerics test only.
int exp2_fma_test_launch(const float* x, float* y, int n, cudaStream_t s) {
  exp2_fma_test_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, y, n);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int ce_combine_launch(const void* stats, int nparts, int M, const int64_t* targets,
                      const float* tgt_logit, float* lse, float* loss_rows, cudaStream_t s) {
  if (M <= 0 || nparts <= 0) return -1;
  ce_combine_kernel<<<(M + 7) / 8, 256, 0, s>>>(reinterpret_cast<const float2*>(stats),
                                                     nparts, M, targets, tgt_logit, lse,
                                                     loss_rows);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int ce_grad_launch(void* logits, int64_t ld, int M, int V, const float* lse,
                   const int64_t* targets, int vocab_offset, cudaStream_t s) {
  if (M <= 0 || ld % 8 || V > ld || (reinterpret_cast<uintptr_t>(logits) & 15)) return -1;
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int blocks = std::min((M + 7) / 8, sms * 8);  // 8 rows (warps) per block
  ce_grad_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(logits), ld, M, V, lse,
                                        targets, vocab_offset);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int loss_reduce_launch(const float* loss_rows, const int64_t* targets, int M, float* loss_out,
                       cudaStream_t s) {
  loss_reduce_kernel<<<1, 1024, 0, s>>>(loss_rows, targets, M, loss_out);
  count_launches(1);
  return ok();
}

int adamw_launch(float* p, const float* g, float* m, float* v, void* p_bf16, int64_t n,
                 int64_t n_decay, const int64_t* ranges, int nr, const float* hp,
                 const float* clip, cudaStream_t s) {
  if ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) |
       reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15)
    return -1;
  if (p_bf16 && (reinterpret_cast<uintptr_t>(p_bf16) & 7)) return -1;
  adamw_kernel<<<grid_for(n / 4, 256, 148 * 8), 256, 0, s>>>(p, g, m, v, (__nv_bfloat16*)p_bf16, n,
                                                           n_decay, ranges, nr, hp, clip);
                                                           count_launches(1);
  return ok();
}

int sumsq_launch(const float* g, int64_t n, float* ws, float* out, cudaStream_t s) {
  sumsq_partial_kernel<<<SUMSQ_BLOCKS, 256, 0, s>>>(g, n, ws);
  count_launches(1);
  sum_final_kernel<<<1, 1024, 0, s>>>(ws, SUMSQ_BLOCKS, out);
  count_launches(1);
  return ok();
}

int clip_coef_launch(const float* sumsq, float scale2, float max_norm, float* clip,
                     float* norm_out, cudaStream_t s) {
  clip_coef_kernel<<<1, 1, 0, s>>>(sumsq, scale2, max_norm, clip, norm_out);
  count_launches(1);
  return ok();
}

int cast_f32_bf16_launch(const float* in, void* out, int64_t n, cudaStream_t s) {
  cast_f32_bf16_kernel<<<grid_for(n, 256), 256, 0, s>>>(in, (__nv_bfloat16*)out, n);
  count_launches(1);
  return ok();
}
int cast_bf16_f32_launch(const void* in, float* out, int64_t n, cudaStream_t s) {
  cast_bf16_f32_kernel<<<grid_for(n, 256), 256, 0, s>>>((const __nv_bfloat16*)in, out, n);
  count_launches(1);
  return ok();
}
int scale_f32_launch(float* x, int64_t n, float a, cudaStream_t s) {
  scale_f32_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, n, a);
  count_launches(1);
  return ok();
}

}  // namespace g2b
