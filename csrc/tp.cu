// Tensor parallelism with sequence parallelism over NVLink 5 peer memory
// (sm_100a): the collectives of the Megatron-SP block and the vocab-parallel
// embedding / cross-entropy, each one kernel over symmetric buffers.
//
// Reference semantics: src/transformer_internals/parallel/tensor_parallel.py
// (column-parallel c_attn / c_fc, row-parallel c_proj / mlp c_proj with the
// bias added once after the reduction, per-section q/k/v head split,
// replicated LayerNorms) and the sequence-parallel AG/RS conjugates; the
// vocab-parallel embedding and cross-entropy follow the same algebra with the
// padded vocabulary split in equal row blocks.
//
// Row-block layout: the residual stream is split along tokens, rank r owning
// rows [r*Ms, (r+1)*Ms) of every [M, C] activation. Every symmetric [M, C]
// buffer keeps each rank's rows at that same offset, so a gather is "copy
// peer q's block q into my block q" and a reduce-scatter is "sum block r of
// every peer's buffer".
//
//   tp_ag_rows      all-gather: pull every peer's own row block (P2P loads).
//   tp_rs_rows      reduce-scatter: sum this rank's block of every peer's
//                   partial (bf16, fixed rank order, fp32 math) + bias +
//                   fp32 residual -> fp32 and/or bf16 rows.
//   tp_embed_fwd    x[i] = wte[tok] + wpe[pos]: the wte row is loaded from the
//                   shard of the rank that owns the token (P2P).
//   tp_embed_bwd    wte_grad[tok] += dx[i] into the owner's shard (P2P fp32
//                   atomics), wpe_grad[pos] += dx[i] locally.
//   tp_ce_stats     per row of this rank's logit slice: max, sum exp, target
//                   logit if the target is in the slice.
//   tp_ce_finish    combine every rank's row statistics (P2P loads) into the
//                   row log-sum-exp and loss, and overwrite the local logits
//                   with softmax - onehot.
//   cp_kv_gather    context parallelism: this rank's k/v rows into its block
//                   of the symmetric key/value buffer, then the blocks of the
//                   earlier ranks (P2P loads): all a causal query here sees.
//   cp_kv_reduce    the key/value gradient of this rank's block summed over
//                   the ranks whose queries saw it (P2P loads, rank order).
//
// Every kernel starts with an arrive/wait handshake of CTA j against CTA j of
// every peer (the data it reads were written by kernels that precede the
// peer's launch) and, where a peer reads this rank's buffer, ends with a
// second one so the buffer can be rewritten on return. All waits are bounded
// (ERR_TIMEOUT_PEER, then return).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>

#include "common.cuh"
#include "tp.cuh"

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

__device__ __forceinline__ uint32_t* tflag(uint32_t* base, int phase, int src, int blk) {
  return base + ((phase * kTpMaxRanks + src) * kTpMaxBlocks + blk);
}

// CTA j raises its flag on every peer and waits (bounded) for every peer's
// CTA j; CTA-uniform result.
__device__ bool tp_handshake(const TpArgs& a, int phase, int* fail) {
  const int j = blockIdx.x;
  if (threadIdx.x < a.world)
    st_release_sys(tflag(a.peer_flags[threadIdx.x], phase, a.rank, j), a.epoch);
  if (threadIdx.x < a.world) {
    const uint32_t* f = tflag(a.peer_flags[a.rank], phase, threadIdx.x, j);
    if ((int32_t)(ld_acquire_sys(f) - a.epoch) < 0) {
      const uint64_t t0 = globaltimer_ns();
      while ((int32_t)(ld_acquire_sys(f) - a.epoch) < 0) {
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

__device__ __forceinline__ void finish(const TpArgs& a, int* fail) {
  __threadfence_system();
  __syncthreads();
  tp_handshake(a, 1, fail);
}

// ------------------------------------------------------------- all-gather --
constexpr int kAgUnroll = 8;

// Copy `total` 16-byte vectors from peers into this rank's buffer: element
// `locate(i, q, off)` of the copy is peer q's vector at bf16 offset `off`,
// stored at the same offset here. kAgUnroll independent peer loads are in
// flight per thread before any store.
template <typename F>
__device__ __forceinline__ void peer_copy_unrolled(const TpArgs& a, __nv_bfloat16* mine,
                                                   int64_t total, F locate) {
  const int64_t span = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < total;
       i0 += span * kAgUnroll) {
    uint4 w[kAgUnroll];
    int64_t off[kAgUnroll];
#pragma unroll
    for (int u = 0; u < kAgUnroll; ++u) {
      const int64_t i = i0 + u * span;
      off[u] = -1;
      if (i < total) {
        int q;
        locate(i, q, off[u]);
        w[u] = __ldcg(reinterpret_cast<const uint4*>(
            reinterpret_cast<const __nv_bfloat16*>(a.peer_bufs[q]) + off[u]));
      }
    }
#pragma unroll
    for (int u = 0; u < kAgUnroll; ++u)
      if (off[u] >= 0) *reinterpret_cast<uint4*>(mine + off[u]) = w[u];
  }
}

__global__ void __launch_bounds__(512) tp_ag_rows_kernel(const TpArgs a) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!tp_handshake(a, 0, &fail)) return;
  const int64_t blk_vec = a.rows * a.cols / 8;  // 16-byte vectors per row block
  const int64_t total = a.pushed ? 0 : blk_vec * (a.world - 1);
  uint4* mine = reinterpret_cast<uint4*>(a.peer_bufs[a.rank]);
  // kAgUnroll independent peer loads in flight per thread before any store:
  // NVLink latency is covered by the loads of one wave of the grid
  const int64_t span = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < total;
       i0 += span * kAgUnroll) {
    uint4 w[kAgUnroll];
    int64_t off[kAgUnroll];
#pragma unroll
    for (int u = 0; u < kAgUnroll; ++u) {
      const int64_t i = i0 + u * span;
      off[u] = -1;
      if (i < total) {
        int q = (int)(i / blk_vec);
        q += q >= a.rank;  // skip this rank's own block
        off[u] = (int64_t)q * blk_vec + i % blk_vec;
        w[u] = __ldcg(reinterpret_cast<const uint4*>(a.peer_bufs[q]) + off[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kAgUnroll; ++u)
      if (off[u] >= 0) mine[off[u]] = w[u];
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, (unsigned long long)(a.rows * a.cols * 2 * a.world));
  finish(a, &fail);
}

// --------------------------------------------------------- reduce-scatter --
// One 8-element vector of the reduce-scatter: the fixed-rank-order fp32 sum
// of the W peers' bf16 partials, + bias + fp32 residual, stored as fp32
// and/or bf16.
template <int W>
__device__ __forceinline__ void rs_finish_vec(const TpArgs& a, int64_t v, const uint4 (&w)[W]) {
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
  for (int q = 0; q < W; ++q) {
    const uint32_t ws[4] = {w[q].x, w[q].y, w[q].z, w[q].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(ws[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  }
  const int64_t e0 = v * 8;
  const int col = (int)(e0 % a.cols);
  if (a.bias) {
    const uint4 bw = *reinterpret_cast<const uint4*>(a.bias + col);
    const uint32_t bs[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(bs[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  }
  if (a.resid) {
    const float4 r0 = reinterpret_cast<const float4*>(a.resid + e0)[0];
    const float4 r1 = reinterpret_cast<const float4*>(a.resid + e0)[1];
    acc[0] += r0.x; acc[1] += r0.y; acc[2] += r0.z; acc[3] += r0.w;
    acc[4] += r1.x; acc[5] += r1.y; acc[6] += r1.z; acc[7] += r1.w;
  }
  if (a.out_f32) {
    reinterpret_cast<float4*>(a.out_f32 + e0)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    reinterpret_cast<float4*>(a.out_f32 + e0)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  if (a.out_bf16)
    *reinterpret_cast<uint4*>(a.out_bf16 + e0) =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                   pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
}

template <int W>
__global__ void __launch_bounds__(512) tp_rs_rows_kernel(const TpArgs a) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!tp_handshake(a, 0, &fail)) return;
  const int64_t nvec = a.rows * a.cols / 8;  // 8 bf16 per vector
  // source q: peer q's partial of this rank's rows, or slot q of the local
  // inbox that peer q's GEMM filled
  const int64_t base = a.inbox ? 0 : (int64_t)a.rank * a.rows * a.cols;
  const __nv_bfloat16* src[W];
#pragma unroll
  for (int q = 0; q < W; ++q)
    src[q] = a.inbox ? a.inbox + (int64_t)q * a.rows * a.cols
                     : reinterpret_cast<const __nv_bfloat16*>(a.peer_bufs[q]) + base;
  // U vectors x W peers = 8 (or W) independent peer loads in flight per
  // thread before any arithmetic
  constexpr int U = W >= 8 ? 1 : 8 / W;
  const int64_t span = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v0 < nvec; v0 += span * U) {
    uint4 w[U][W];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + u * span;
      if (v < nvec) {
#pragma unroll
        for (int q = 0; q < W; ++q) w[u][q] = __ldcg(reinterpret_cast<const uint4*>(src[q]) + v);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + u * span;
      if (v < nvec) rs_finish_vec<W>(a, v, w[u]);
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, (unsigned long long)(a.rows * a.cols * 2 * W));
  finish(a, &fail);
}

// -------------------------------------------------------------- embedding --
// One warp per local row; C multiple of 8.
__global__ void __launch_bounds__(256) tp_embed_fwd_kernel(const TpArgs a) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!tp_handshake(a, 0, &fail)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  for (int64_t i = blockIdx.x * (int64_t)nw + warp; i < a.rows; i += (int64_t)gridDim.x * nw) {
    const int64_t m = (int64_t)a.rank * a.rows + i;  // global token index
    const int64_t tok = a.idx[m];
    const int pos = (int)(m % a.T);
    const int q = (int)(tok / a.vocab_per_rank);
    const int64_t vr = tok % a.vocab_per_rank;
    const __nv_bfloat16* wrow =
        reinterpret_cast<const __nv_bfloat16*>(a.peer_bufs[q]) + vr * a.cols;
    const __nv_bfloat16* prow = a.wpe + (int64_t)pos * a.cols;
    float* out = a.out_f32 + i * a.cols;
    for (int c = lane * 8; c < a.cols; c += 256) {
      const uint4 w = __ldcg(reinterpret_cast<const uint4*>(wrow + c));
      const uint4 pw = *reinterpret_cast<const uint4*>(prow + c);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w}, ps[4] = {pw.x, pw.y, pw.z, pw.w};
      float o[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(ws[k]), g = unpack_bf16x2(ps[k]);
        o[2 * k] = f.x + g.x;
        o[2 * k + 1] = f.y + g.y;
      }
      reinterpret_cast<float4*>(out + c)[0] = make_float4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<float4*>(out + c)[1] = make_float4(o[4], o[5], o[6], o[7]);
    }
  }
  // an all-to-all of this rank's bf16 rows in the reference convention
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, (unsigned long long)(a.rows * a.cols * 2));
  finish(a, &fail);
}

__global__ void __launch_bounds__(256) tp_embed_bwd_kernel(const TpArgs a) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!tp_handshake(a, 0, &fail)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  for (int64_t i = blockIdx.x * (int64_t)nw + warp; i < a.rows; i += (int64_t)gridDim.x * nw) {
    const int64_t m = (int64_t)a.rank * a.rows + i;
    const int64_t tok = a.idx[m];
    const int pos = (int)(m % a.T);
    const int q = (int)(tok / a.vocab_per_rank);
    const int64_t vr = tok % a.vocab_per_rank;
    float* grow = reinterpret_cast<float*>(a.peer_bufs[q]) + vr * a.cols;
    float* prow = a.out_f32 + (int64_t)pos * a.cols;  // wpe grad (local)
    const float* dx = a.resid + i * a.cols;
    for (int c = lane; c < a.cols; c += 32) {
      const float g = dx[c];
      atomicAdd(grow + c, g);
      atomicAdd(prow + c, g);
    }
  }
  // an all-to-all of this rank's fp32 gradient rows
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, (unsigned long long)(a.rows * a.cols * 4));
  finish(a, &fail);
}

// ---------------------------------------------------------- cross-entropy --
constexpr int CE_T = 256;

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffff, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = is_max ? fmaxf(t, red[w]) : t + red[w];
  __syncthreads();
  return t;
}

// stats[row] = {max, sum exp(l - max), target logit, 1 if the target is local}
__global__ void __launch_bounds__(CE_T) tp_ce_stats_kernel(const TpArgs a) {
  __shared__ float red[CE_T / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* lr = a.logits + row * a.ld;
  float m = -INFINITY;
  for (int c = threadIdx.x; c < a.vocab_valid; c += blockDim.x)
    m = fmaxf(m, __bfloat162float(lr[c]));
  m = block_reduce(m, red, true);
  float s = 0.f;
  for (int c = threadIdx.x; c < a.vocab_valid; c += blockDim.x)
    s += __expf(__bfloat162float(lr[c]) - m);
  s = block_reduce(s, red, false);
  if (threadIdx.x == 0) {
    const int64_t t = a.idx[row] - a.vocab_start;
    const bool local = a.idx[row] != -100 && t >= 0 && t < a.vocab_valid;
    float* st = a.stats + row * 4;
    st[0] = m;
    st[1] = s;
    st[2] = local ? __bfloat162float(lr[t]) : 0.f;
    st[3] = local ? 1.f : 0.f;
  }
}

// One CTA per group of rows (grid-stride): combine every rank's statistics,
// write the row loss, then dlogits = softmax - onehot over the local slice
// (padded columns get 0).
__global__ void __launch_bounds__(CE_T) tp_ce_finish_kernel(const TpArgs a) {
  __shared__ int fail;
  __shared__ float s_gm, s_inv;
  __shared__ int64_t s_t;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!tp_handshake(a, 0, &fail)) return;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    if (threadIdx.x == 0) {
      float gm = -INFINITY, tl = 0.f;
      float ms[kTpMaxRanks], ss[kTpMaxRanks];
      for (int q = 0; q < a.world; ++q) {
        const float* st = reinterpret_cast<const float*>(a.peer_bufs[q]) + row * 4;
        const float4 v = __ldcg(reinterpret_cast<const float4*>(st));
        ms[q] = v.x;
        ss[q] = v.y;
        if (v.w > 0.f) tl = v.z;
        gm = fmaxf(gm, v.x);
      }
      float tot = 0.f;
      for (int q = 0; q < a.world; ++q) tot += ss[q] * __expf(ms[q] - gm);
      const float lse = gm + __logf(tot);
      const int64_t tgt = a.idx[row];
      a.loss_rows[row] = tgt == -100 ? 0.f : lse - tl;
      s_gm = gm;
      s_inv = 1.f / tot;
      s_t = tgt == -100 ? -1 : tgt - a.vocab_start;
    }
    __syncthreads();
    // softmax as the single-GPU cross-entropy kernel forms it:
    // exp(l - global max) x (1 / global sum)
    const float gm = s_gm, inv = s_inv;
    const int64_t t = s_t;
    const bool ignore = a.idx[row] == -100;
    __nv_bfloat16* lr = a.logits + row * a.ld;
    for (int c = threadIdx.x; c < a.ld; c += blockDim.x) {
      float g = 0.f;
      if (!ignore && c < a.vocab_valid) {
        g = __expf(__bfloat162float(lr[c]) - gm) * inv;
        if (c == t) g -= 1.f;
      }
      lr[c] = __float2bfloat16(g);
    }
    __syncthreads();
  }
  // an all-gather of every rank's [rows, 4] fp32 statistics (output bytes)
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, (unsigned long long)(a.world * a.rows * 16));
  finish(a, &fail);
}

// ---------------------------------------------------- context parallelism --
// Row (b, t) of block q in a [B, world*Tl, cols] buffer.
// Bytes charged per K/V gather or dK/dV reduce-scatter: the reference
// convention (all-gather = output, reduce-scatter = input), i.e. the whole
// [B, world * Tl, 2C] bf16 key/value tensor, whatever the causal split lets
// the kernel skip.
__device__ __forceinline__ unsigned long long cp_convention_bytes(const TpArgs& a) {
  return (unsigned long long)a.B * a.world * a.Tl * a.cols * 2;
}

__device__ __forceinline__ int64_t cp_row(const TpArgs& a, int q, int64_t i) {
  const int64_t b = i / a.Tl, t = i % a.Tl;
  return b * (int64_t)a.world * a.Tl + (int64_t)q * a.Tl + t;
}

// Zig-zag split: chunk k (of 2*world, Tl/2 tokens each) belongs to rank
// k (k < world) or 2*world-1-k; a rank stores its two chunks as the halves of
// each local sequence. zz_row: natural buffer row of row (b, t) of chunk k.
__device__ __forceinline__ int64_t zz_row(const TpArgs& a, int k, int64_t b, int64_t t) {
  const int h = a.Tl / 2;
  return b * (int64_t)a.world * a.Tl + (int64_t)k * h + t;
}
// Chunk of local row i (sequence b = i / Tl; first half -> chunk rank,
// second half -> chunk 2*world-1-rank).
__device__ __forceinline__ int zz_local_chunk(const TpArgs& a, int64_t i, int64_t* b, int64_t* t) {
  const int h = a.Tl / 2;
  const int64_t j = i % a.Tl;
  *b = i / a.Tl;
  *t = j % h;
  return j < h ? a.rank : 2 * a.world - 1 - a.rank;
}

__global__ void __launch_bounds__(512) cp_kv_gather_zz_kernel(const TpArgs a) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  const int C = a.cols / 2;
  const int vpr = a.cols / 8;
  const int h = a.Tl / 2;
  const int64_t nvec = (int64_t)a.B * a.Tl * vpr;   // own vectors (both chunks)
  __nv_bfloat16* mine = reinterpret_cast<__nv_bfloat16*>(a.peer_bufs[a.rank]);
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = v / vpr;
    const int c = (int)(v % vpr) * 8;
    int64_t b, t;
    const int k = zz_local_chunk(a, i, &b, &t);
    const uint4 w = *reinterpret_cast<const uint4*>(a.src + i * a.src_ld + C + c);
    *reinterpret_cast<uint4*>(mine + zz_row(a, k, b, t) * a.cols + c) = w;
  }
  __threadfence_system();
  __syncthreads();
  if (!tp_handshake(a, 0, &fail)) return;
  // chunks 0..2w-1-r except the own ones (r and 2w-1-r): e -> e (e < r) or e + 1
  const int nk = 2 * a.world - 2 - a.rank;
  const int64_t cvec = (int64_t)a.B * h * vpr;      // vectors per chunk
  peer_copy_unrolled(a, mine, cvec * nk, [&](int64_t v, int& q, int64_t& off) {
    const int e = (int)(v / cvec);
    const int k = e < a.rank ? e : e + 1;
    q = k < a.world ? k : 2 * a.world - 1 - k;
    const int64_t vv = v % cvec;
    const int64_t row = vv / vpr;                   // b * h + t
    off = zz_row(a, k, row / h, row % h) * a.cols + (int)(vv % vpr) * 8;
  });
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, cp_convention_bytes(a));
  finish(a, &fail);
}

__global__ void __launch_bounds__(512) cp_kv_reduce_zz_kernel(const TpArgs a) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!tp_handshake(a, 0, &fail)) return;
  const int C = a.cols / 2;
  const int vpr = a.cols / 8;
  const int64_t nvec = (int64_t)a.B * a.Tl * vpr;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = v / vpr;
    const int c = (int)(v % vpr) * 8;
    int64_t b, t;
    const int k = zz_local_chunk(a, i, &b, &t);
    const int64_t off = zz_row(a, k, b, t) * a.cols + c;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int q = 0; q < a.world; ++q) {
      for (int part = 0; part < 2; ++part) {
        // first-half queries of rank q see chunks 0..q, second-half 0..2w-1-q
        const int last = part == 0 ? q : 2 * a.world - 1 - q;
        if (k > last) continue;
        const void* src = part == 0 ? a.peer_bufs[q] : a.peer_bufs2[q];
        const uint4 w = __ldcg(reinterpret_cast<const uint4*>(
            reinterpret_cast<const __nv_bfloat16*>(src) + off));
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(ws[j]);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        }
      }
    }
    *reinterpret_cast<uint4*>(a.out_bf16 + i * a.src_ld + C + c) =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                   pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
  }
  // chunk r is read from 2w-r partials, chunk 2w-1-r from r+1
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, cp_convention_bytes(a));
  finish(a, &fail);
}

__global__ void __launch_bounds__(512) cp_kv_gather_kernel(const TpArgs a) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  const int C = a.cols / 2;
  const int vpr = a.cols / 8;                       // 16-byte vectors per k/v row
  const int64_t nvec = (int64_t)a.B * a.Tl * vpr;   // vectors per block
  __nv_bfloat16* mine = reinterpret_cast<__nv_bfloat16*>(a.peer_bufs[a.rank]);
  // 1. own block from the local qkv rows
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = v / vpr;
    const int c = (int)(v % vpr) * 8;
    const uint4 w = *reinterpret_cast<const uint4*>(a.src + i * a.src_ld + C + c);
    *reinterpret_cast<uint4*>(mine + cp_row(a, a.rank, i) * a.cols + c) = w;
  }
  __threadfence_system();
  __syncthreads();
  if (!tp_handshake(a, 0, &fail)) return;
  // 2. blocks of the earlier ranks from their buffers
  peer_copy_unrolled(a, mine, nvec * a.rank, [&](int64_t v, int& q, int64_t& off) {
    q = (int)(v / nvec);
    const int64_t vv = v % nvec;
    off = cp_row(a, q, vv / vpr) * a.cols + (int)(vv % vpr) * 8;
  });
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, cp_convention_bytes(a));
  finish(a, &fail);
}

// Streaming form of the gather: this rank's k/v rows (both halves of each
// local sequence under the zig-zag split; the order is the local one) into
// its own compact [B, Tl, 2C] symmetric buffer peer_bufs[rank], then, once
// every CTA's stores are fenced at system scope, the launch's last CTA stores
// `epoch` with release semantics into word `rank` of every peer's flag buffer
// (peer_flags[q][rank]). The attention kernels of every rank read these rows
// in place through TMA after seeing that word reach the epoch; no peer data
// moves here. Word kKvPublishCount of this rank's flag buffer counts the
// launch's finished CTAs. The buffer is rewritten one step later, after the
// data-parallel gradient reduction every rank of the group takes part in:
// no rank reaches it while a peer's backward may still read the rows.
__global__ void __launch_bounds__(512) cp_kv_publish_kernel(const TpArgs a) {
  const int C = a.cols / 2;
  const int vpr = a.cols / 8;                       // 16-byte vectors per k/v row
  const int64_t nvec = (int64_t)a.B * a.Tl * vpr;
  __nv_bfloat16* mine = reinterpret_cast<__nv_bfloat16*>(a.peer_bufs[a.rank]);
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = v / vpr;
    const int c = (int)(v % vpr) * 8;
    const uint4 w = *reinterpret_cast<const uint4*>(a.src + i * a.src_ld + C + c);
    *reinterpret_cast<uint4*>(mine + i * a.cols + c) = w;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return;
  uint32_t* count = a.peer_flags[a.rank] + kKvPublishCount;
  if (atomicAdd(count, 1u) != gridDim.x - 1) return;
  *count = 0;
  __threadfence_system();
  for (int q = 0; q < a.world; ++q) st_release_sys(a.peer_flags[q] + a.rank, a.epoch);
  if (a.byte_counter) atomicAdd(a.byte_counter, cp_convention_bytes(a));
}

__global__ void __launch_bounds__(512) cp_kv_reduce_kernel(const TpArgs a) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!tp_handshake(a, 0, &fail)) return;
  const int C = a.cols / 2;
  const int vpr = a.cols / 8;
  const int64_t nvec = (int64_t)a.B * a.Tl * vpr;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = v / vpr;
    const int c = (int)(v % vpr) * 8;
    const int64_t off = cp_row(a, a.rank, i) * a.cols + c;
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
    // every source's load is issued before the first sum (rank order kept)
    uint4 w[kTpMaxRanks];
#pragma unroll
    for (int j = 0; j < kTpMaxRanks; ++j)
      if (a.rank + j < a.world)
        w[j] = __ldcg(reinterpret_cast<const uint4*>(
            reinterpret_cast<const __nv_bfloat16*>(a.peer_bufs[a.rank + j]) + off));
#pragma unroll
    for (int j = 0; j < kTpMaxRanks; ++j) {
      if (a.rank + j >= a.world) break;
      const uint32_t ws[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(ws[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
    *reinterpret_cast<uint4*>(a.out_bf16 + i * a.src_ld + C + c) =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                   pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.byte_counter)
    atomicAdd(a.byte_counter, cp_convention_bytes(a));
  finish(a, &fail);
}

int grid_for_rows(int64_t rows, int per_cta, int cap) {
  int64_t g = (rows + per_cta - 1) / per_cta;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (int)g;
}

bool common_ok(const TpArgs& a) {
  return a.world >= 1 && a.world <= kTpMaxRanks && a.rank >= 0 && a.rank < a.world &&
         a.nblocks >= 1 && a.nblocks <= kTpMaxBlocks;
}

}  // namespace

int tp_ag_rows_launch(TpArgs a, cudaStream_t s) {
  if (!common_ok(a) || a.cols % 8 || a.rows <= 0) return -1;
  tp_ag_rows_kernel<<<a.nblocks, 512, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int tp_rs_rows_launch(TpArgs a, cudaStream_t s) {
  if (!common_ok(a) || a.cols % 8 || a.rows <= 0) return -1;
  switch (a.world) {
    case 1: tp_rs_rows_kernel<1><<<a.nblocks, 512, 0, s>>>(a); break;
    case 2: tp_rs_rows_kernel<2><<<a.nblocks, 512, 0, s>>>(a); break;
    case 3: tp_rs_rows_kernel<3><<<a.nblocks, 512, 0, s>>>(a); break;
    case 4: tp_rs_rows_kernel<4><<<a.nblocks, 512, 0, s>>>(a); break;
    case 5: tp_rs_rows_kernel<5><<<a.nblocks, 512, 0, s>>>(a); break;
    case 6: tp_rs_rows_kernel<6><<<a.nblocks, 512, 0, s>>>(a); break;
    case 7: tp_rs_rows_kernel<7><<<a.nblocks, 512, 0, s>>>(a); break;
    default: tp_rs_rows_kernel<8><<<a.nblocks, 512, 0, s>>>(a); break;
  }
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int tp_embed_fwd_launch(TpArgs a, cudaStream_t s) {
  if (!common_ok(a) || a.cols % 8 || a.vocab_per_rank <= 0) return -1;
  tp_embed_fwd_kernel<<<a.nblocks, 256, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int tp_embed_bwd_launch(TpArgs a, cudaStream_t s) {
  if (!common_ok(a) || a.vocab_per_rank <= 0) return -1;
  tp_embed_bwd_kernel<<<a.nblocks, 256, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int tp_ce_stats_launch(TpArgs a, cudaStream_t s) {
  if (a.rows <= 0 || a.vocab_valid < 0) return -1;  // 0: a slice of padding only
  tp_ce_stats_kernel<<<(unsigned)a.rows, CE_T, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int cp_kv_gather_launch(TpArgs a, cudaStream_t s) {
  if (!common_ok(a) || a.cols % 16 || a.src_ld % 8 || a.B <= 0 || a.Tl <= 0 || !a.src) return -1;
  if (a.zigzag) {
    if (a.Tl % 2) return -1;
    cp_kv_gather_zz_kernel<<<a.nblocks, 512, 0, s>>>(a);
    count_launches(1);
    return launch_succeeded() ? 0 : -11;
  }
  cp_kv_gather_kernel<<<a.nblocks, 512, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int cp_kv_publish_launch(TpArgs a, cudaStream_t s) {
  if (!common_ok(a) || a.cols % 16 || a.src_ld % 8 || a.B <= 0 || a.Tl <= 0 || !a.src ||
      a.world > kKvPublishCount)
    return -1;
  if (a.zigzag && a.Tl % 2) return -1;
  cp_kv_publish_kernel<<<a.nblocks, 512, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int cp_kv_reduce_launch(TpArgs a, cudaStream_t s) {
  if (!common_ok(a) || a.cols % 16 || a.src_ld % 8 || a.B <= 0 || a.Tl <= 0 || !a.out_bf16)
    return -1;
  if (a.zigzag) {
    if (a.Tl % 2 || !a.peer_bufs2) return -1;
    cp_kv_reduce_zz_kernel<<<a.nblocks, 512, 0, s>>>(a);
    count_launches(1);
    return launch_succeeded() ? 0 : -11;
  }
  cp_kv_reduce_kernel<<<a.nblocks, 512, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int tp_ce_finish_launch(TpArgs a, cudaStream_t s) {
  if (!common_ok(a) || a.rows <= 0) return -1;
  tp_ce_finish_kernel<<<a.nblocks, CE_T, 0, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

}  // namespace g2b
