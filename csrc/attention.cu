// Causal flash attention, forward and backward, head_dim 64, bf16 in / fp32
// softmax statistics. Reference semantics: src/transformer_internals/model.py:
// 299-309 (QK^T/sqrt(d), masked_fill(-inf) at absolute positions, softmax, @V).
//
// Design:
//  * Q/K/V are read in place from the fused c_attn output ([B*T, 3C], head h at
//    columns h*64 of each section) and O is written straight into the [B*T, C]
//    layout c_proj consumes: no head split / merge copies (model.py:255-263,
//    :318 are folded away).
//  * Online softmax in the exp2 domain (scores pre-multiplied by
//    scale*log2(e)); only the per-row log2-sum-exp is saved for backward, never
//    the T x T probabilities.
//  * Causal masking is implicit from absolute positions: query i sits at
//    q_offset + i, key j at j. q_offset lets a context-parallel rank attend its
//    local query shard against the gathered full-length K/V (reference
//    sequence_parallel.py:101-132 slices its mask the same way).
//  * Backward is deterministic: one kernel owns a K/V block and accumulates
//    dK/dV over query blocks, a second owns a Q block and accumulates dQ over
//    key blocks. No atomics, so two runs are bitwise identical.
//  * Fragments are mma.sync m16n8k16 (bf16, fp32 accumulate); tiles live in
//    XOR-swizzled shared memory, filled by cp.async double buffering.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>

#include "attention.cuh"
#include "common.cuh"

namespace g2b {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int sz = pred ? 16 : 0;  // src-size 0 => zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a 64-column bf16 tile
// whose rows are 128 bytes, with the chunk index XOR-swizzled by row % 8 so
// that ldmatrix row groups hit 8 different bank quads.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

// Load rows [t0, t0+R) of one head (64 bf16 each) into a swizzled tile;
// rows >= T are zero-filled.
template <int R, int NT>
__device__ __forceinline__ void load_tile(uint32_t tile, const __nv_bfloat16* base, int64_t st,
                                          int t0, int T) {
  for (int i = threadIdx.x; i < R * 8; i += NT) {
    const int r = i >> 3, c = i & 7;
    const int t = t0 + r;
    const bool ok = t < T;
    const __nv_bfloat16* src = base + (int64_t)(ok ? t : 0) * st + c * 8;
    cp_async16(tile + swz(r, c), src, ok);
  }
}

__device__ __forceinline__ const __nv_bfloat16* head_ptr(const HeadView& v, int b, int h) {
  return reinterpret_cast<const __nv_bfloat16*>(v.base) + b * v.sb + h * v.sh;
}
__device__ __forceinline__ __nv_bfloat16* head_ptr_w(const HeadView& v, int b, int h) {
  return reinterpret_cast<__nv_bfloat16*>(v.base) + b * v.sb + h * v.sh;
}

// A-operand fragments of a 16x64 row block of a swizzled tile (rows r0..r0+15).
__device__ __forceinline__ void load_a_frags(uint32_t tile, int r0, uint32_t (*a)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int r = r0 + (lane & 15);
    const int c = kk * 2 + (lane >> 4);
    ldsm_x4(tile + swz(r, c), a[kk][0], a[kk][1], a[kk][2], a[kk][3]);
  }
}

// acc[16 x 64] += A[16 x 64] . T^T where T is a 64x64 tile stored [n][k] (k
// contiguous): the "K-major B" case, e.g. S = Q K^T with T = K.
__device__ __forceinline__ void mma_abt(float (*acc)[4], const uint32_t (*a)[4], uint32_t tile) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
      const int c = kk * 2 + ((lane >> 3) & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(tile + swz(r, c), b0, b1, b2, b3);
      mma16816(acc[2 * np], a[kk], b0, b1);
      mma16816(acc[2 * np + 1], a[kk], b2, b3);
    }
  }
}

// acc[16 x 64] += P[16 x 64] . T where T is a 64x64 tile stored [k][n] (n
// contiguous) and P comes as C-layout fp32 fragments p[8][4] (converted to bf16
// A fragments on the fly): e.g. O += P V.
__device__ __forceinline__ void mma_pt(float (*acc)[4], const float (*p)[4], uint32_t tile) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t a[4];
    a[0] = pack_bf16x2(p[2 * kk][0], p[2 * kk][1]);
    a[1] = pack_bf16x2(p[2 * kk][2], p[2 * kk][3]);
    a[2] = pack_bf16x2(p[2 * kk + 1][0], p[2 * kk + 1][1]);
    a[3] = pack_bf16x2(p[2 * kk + 1][2], p[2 * kk + 1][3]);
#pragma unroll
    for (int dp = 0; dp < 4; ++dp) {
      const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
      const int c = dp * 2 + (lane >> 4);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(tile + swz(r, c), b0, b1, b2, b3);
      mma16816(acc[2 * dp], a, b0, b1);
      mma16816(acc[2 * dp + 1], a, b2, b3);
    }
  }
}

// Store a warp's 16x64 fp32 accumulator (C layout) as bf16 rows t0+.. of a head.
__device__ __forceinline__ void store_rows(__nv_bfloat16* base, int64_t st, int t0, int T,
                                           const float (*acc)[4], float s0, float s1) {
  const int lane = threadIdx.x & 31;
  const int ra = t0 + (lane >> 2), rb = ra + 8;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int c = nt * 8 + 2 * (lane & 3);
    if (ra < T)
      *reinterpret_cast<uint32_t*>(base + (int64_t)ra * st + c) =
          pack_bf16x2(acc[nt][0] * s0, acc[nt][1] * s0);
    if (rb < T)
      *reinterpret_cast<uint32_t*>(base + (int64_t)rb * st + c) =
          pack_bf16x2(acc[nt][2] * s1, acc[nt][3] * s1);
  }
}

// ---------------------------------------------------------------- forward ---
constexpr int FWD_BQ = 128, FWD_BK = 64, FWD_THREADS = 256;

__global__ void __launch_bounds__(FWD_THREADS) attn_fwd_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + FWD_BQ * 128;
  const uint32_t sV0 = sK0 + 2 * FWD_BK * 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int q0 = qb * FWD_BQ;

  const __nv_bfloat16* qp = head_ptr(a.q, b, h);
  const __nv_bfloat16* kp = head_ptr(a.k, b, h);
  const __nv_bfloat16* vp = head_ptr(a.v, b, h);

  int kv_end = a.Tk;
  if (a.causal) kv_end = min(a.Tk, a.q_offset + q0 + FWD_BQ);
  const int nblk = kv_end > 0 ? (kv_end + FWD_BK - 1) / FWD_BK : 0;

  load_tile<FWD_BQ, FWD_THREADS>(sQ, qp, a.q.st, q0, a.Tq);
  cp_async_commit();
  if (nblk > 0) {
    load_tile<FWD_BK, FWD_THREADS>(sK0, kp, a.k.st, 0, a.Tk);
    load_tile<FWD_BK, FWD_THREADS>(sV0, vp, a.v.st, 0, a.Tk);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  uint32_t qa[4][4];
  load_a_frags(sQ, warp * 16, qa);

  const float sl2 = a.scale * kLog2e;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  const int row_a = q0 + warp * 16 + (lane >> 2);
  const int absq[2] = {a.q_offset + row_a, a.q_offset + row_a + 8};

  for (int j = 0; j < nblk; ++j) {
    const int buf = j & 1;
    if (j + 1 < nblk) {
      const int nb = buf ^ 1;
      load_tile<FWD_BK, FWD_THREADS>(sK0 + nb * FWD_BK * 128, kp, a.k.st, (j + 1) * FWD_BK, a.Tk);
      load_tile<FWD_BK, FWD_THREADS>(sV0 + nb * FWD_BK * 128, vp, a.v.st, (j + 1) * FWD_BK, a.Tk);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sK = sK0 + buf * FWD_BK * 128, sV = sV0 + buf * FWD_BK * 128;

    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    mma_abt(s, qa, sK);

    const int kv0 = j * FWD_BK;
    const bool need_mask = (kv0 + FWD_BK > a.Tk) || (a.causal && kv0 + FWD_BK - 1 > a.q_offset + q0);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float v = s[nt][i] * sl2;
        if (need_mask) {
          const int col = kv0 + nt * 8 + 2 * (lane & 3) + (i & 1);
          if (col >= a.Tk || (a.causal && col > absq[i >> 1])) v = -INFINITY;
        }
        s[nt][i] = v;
        mx[i >> 1] = fmaxf(mx[i >> 1], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffff, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffff, mx[r], 2));
      const float mn = fmaxf(m[r], mx[r]);
      const float base = mn == -INFINITY ? 0.f : mn;
      corr[r] = ex2(m[r] - base);
      m[r] = mn;
      mx[r] = base;  // reuse as the subtraction base
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float p = ex2(s[nt][i] - mx[i >> 1]);
        s[nt][i] = p;
        rs[i >> 1] += p;
      }
      o[nt][0] *= corr[0];
      o[nt][1] *= corr[0];
      o[nt][2] *= corr[1];
      o[nt][3] *= corr[1];
    }
    l[0] = l[0] * corr[0] + rs[0];
    l[1] = l[1] * corr[1] + rs[1];
    mma_pt(o, s, sV);
    __syncthreads();
  }

  float inv[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] += __shfl_xor_sync(0xffffffff, l[r], 1);
    l[r] += __shfl_xor_sync(0xffffffff, l[r], 2);
    inv[r] = l[r] > 0.f ? 1.f / l[r] : 0.f;
  }
  __nv_bfloat16* op = head_ptr_w(a.o, b, h);
  store_rows(op, a.o.st, q0 + warp * 16, a.Tq, o, inv[0], inv[1]);
  if ((lane & 3) == 0) {
    float* lse = a.lse + (int64_t)bh * a.Tq;
    if (row_a < a.Tq) lse[row_a] = m[0] + log2f(l[0]);
    if (row_a + 8 < a.Tq) lse[row_a + 8] = m[1] + log2f(l[1]);
  }
}

// ------------------------------------------------------ backward: delta ---
// delta[b,h,t] = sum_d dO[b,t,h,d] * O[b,t,h,d]; one warp per (b,h,t).
// Scalar variant for views whose rows are not 16-byte aligned: one warp per
// row, 4 bytes per lane.
__global__ void attn_bwd_delta_scalar_kernel(const AttnArgs a) {
  const int64_t gw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)a.B * a.H * a.Tq;
  if (gw >= total) return;
  const int t = gw % a.Tq;
  const int bh = gw / a.Tq, b = bh / a.H, h = bh % a.H;
  const __nv_bfloat16* o = head_ptr(a.o, b, h) + (int64_t)t * a.o.st;
  const __nv_bfloat16* g = head_ptr(a.dout, b, h) + (int64_t)t * a.dout.st;
  const float2 ov = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(o)[lane]);
  const float2 gv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(g)[lane]);
  float s = ov.x * gv.x + ov.y * gv.y;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffff, s, off);
  if (lane == 0) a.delta[gw] = s;
}

__global__ void attn_bwd_delta_kernel(const AttnArgs a) {
  // 8 lanes per row, 16 bytes each: a row's 64 bf16 of O and dO are two
  // 128-byte coalesced reads, and a warp covers 4 rows.
  const int64_t gt = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t row = gt >> 3;
  const int sub = threadIdx.x & 7;
  const int64_t total = (int64_t)a.B * a.H * a.Tq;
  float s = 0.f;
  if (row < total) {
    const int t = row % a.Tq;
    const int64_t bh = row / a.Tq;
    const int b = bh / a.H, h = bh % a.H;
    const uint4 ov = reinterpret_cast<const uint4*>(head_ptr(a.o, b, h) + (int64_t)t * a.o.st)[sub];
    const uint4 gv = reinterpret_cast<const uint4*>(head_ptr(a.dout, b, h) + (int64_t)t * a.dout.st)[sub];
    const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 o2 = unpack_bf16x2(ow[i]), g2 = unpack_bf16x2(gw[i]);
      s = fmaf(o2.x, g2.x, s);
      s = fmaf(o2.y, g2.y, s);
    }
  }
#pragma unroll
  for (int off = 4; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffff, s, off);
  if (row < total && sub == 0) a.delta[row] = s;
}

// ---------------------------------------------------- backward: dK / dV ---
constexpr int BWD_B = 64, BWD_THREADS = 128;

__global__ void __launch_bounds__(BWD_THREADS) attn_bwd_dkdv_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sKV = smem_u32(smem);         // K then V (64 rows each)
  const uint32_t sQ0 = sKV + 2 * BWD_B * 128;  // 2 buffers
  const uint32_t sG0 = sQ0 + 2 * BWD_B * 128;  // dO, 2 buffers
  float* sL = reinterpret_cast<float*>(smem + 6 * BWD_B * 128);  // [2][64]
  float* sDl = sL + 2 * BWD_B;                                   // [2][64]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int kv0 = blockIdx.x * BWD_B;

  const __nv_bfloat16* qp = head_ptr(a.q, b, h);
  const __nv_bfloat16* kp = head_ptr(a.k, b, h);
  const __nv_bfloat16* vp = head_ptr(a.v, b, h);
  const __nv_bfloat16* gp = head_ptr(a.dout, b, h);
  const float* lse = a.lse + (int64_t)bh * a.Tq;
  const float* dl = a.delta + (int64_t)bh * a.Tq;

  // Query blocks that can see any key of this block.
  int qstart = 0;
  if (a.causal) qstart = max(0, (kv0 - a.q_offset) / BWD_B);
  const int nq = (a.Tq + BWD_B - 1) / BWD_B;

  auto load_q = [&](int qi, int buf) {
    load_tile<BWD_B, BWD_THREADS>(sQ0 + buf * BWD_B * 128, qp, a.q.st, qi * BWD_B, a.Tq);
    load_tile<BWD_B, BWD_THREADS>(sG0 + buf * BWD_B * 128, gp, a.dout.st, qi * BWD_B, a.Tq);
    for (int i = threadIdx.x; i < BWD_B; i += BWD_THREADS) {
      const int t = qi * BWD_B + i;
      sL[buf * BWD_B + i] = t < a.Tq ? lse[t] : INFINITY;
      sDl[buf * BWD_B + i] = t < a.Tq ? dl[t] : 0.f;
    }
  };

  load_tile<BWD_B, BWD_THREADS>(sKV, kp, a.k.st, kv0, a.Tk);
  load_tile<BWD_B, BWD_THREADS>(sKV + BWD_B * 128, vp, a.v.st, kv0, a.Tk);
  cp_async_commit();
  if (qstart < nq) load_q(qstart, 0);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  uint32_t ka[4][4], va[4][4];
  load_a_frags(sKV, warp * 16, ka);
  load_a_frags(sKV + BWD_B * 128, warp * 16, va);

  float dk[8][4], dv[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) dk[i][j] = dv[i][j] = 0.f;

  const float sl2 = a.scale * kLog2e;
  const int kvr[2] = {kv0 + warp * 16 + (lane >> 2), kv0 + warp * 16 + (lane >> 2) + 8};

  for (int qi = qstart; qi < nq; ++qi) {
    const int buf = (qi - qstart) & 1;
    __syncthreads();
    if (qi + 1 < nq) {
      load_q(qi + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sQ = sQ0 + buf * BWD_B * 128, sG = sG0 + buf * BWD_B * 128;
    const float* L = sL + buf * BWD_B;
    const float* Dl = sDl + buf * BWD_B;
    const int q0 = qi * BWD_B;

    // S^T = K Q^T  (rows: keys of this warp, cols: 64 queries)
    float st[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
    mma_abt(st, ka, sQ);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int qc = nt * 8 + 2 * (lane & 3) + (i & 1);
        float p = ex2(st[nt][i] * sl2 - L[qc]);
        const int kv = kvr[i >> 1];
        if (kv >= a.Tk || (a.causal && a.q_offset + q0 + qc < kv)) p = 0.f;
        st[nt][i] = p;
      }
    }
    // dV += P^T dO
    mma_pt(dv, st, sG);
    // dP^T = V dO^T
    float dpt[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
    mma_abt(dpt, va, sG);
    // dS^T = P^T * (dP^T - delta)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int qc = nt * 8 + 2 * (lane & 3) + (i & 1);
        dpt[nt][i] = st[nt][i] * (dpt[nt][i] - Dl[qc]);
      }
    }
    // dK += dS^T Q
    mma_pt(dk, dpt, sQ);
  }

  __nv_bfloat16* dkp = head_ptr_w(a.dk, b, h);
  __nv_bfloat16* dvp = head_ptr_w(a.dv, b, h);
  store_rows(dkp, a.dk.st, kv0 + warp * 16, a.Tk, dk, a.scale, a.scale);
  store_rows(dvp, a.dv.st, kv0 + warp * 16, a.Tk, dv, 1.f, 1.f);
}

// -------------------------------------------------------- backward: dQ ---
__global__ void __launch_bounds__(BWD_THREADS) attn_bwd_dq_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQG = smem_u32(smem);         // Q then dO
  const uint32_t sK0 = sQG + 2 * BWD_B * 128;  // 2 buffers
  const uint32_t sV0 = sK0 + 2 * BWD_B * 128;  // 2 buffers
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int qb = gridDim.x - 1 - blockIdx.x;
  const int q0 = qb * BWD_B;

  const __nv_bfloat16* qp = head_ptr(a.q, b, h);
  const __nv_bfloat16* kp = head_ptr(a.k, b, h);
  const __nv_bfloat16* vp = head_ptr(a.v, b, h);
  const __nv_bfloat16* gp = head_ptr(a.dout, b, h);

  int kv_end = a.Tk;
  if (a.causal) kv_end = min(a.Tk, a.q_offset + q0 + BWD_B);
  const int nblk = kv_end > 0 ? (kv_end + BWD_B - 1) / BWD_B : 0;

  load_tile<BWD_B, BWD_THREADS>(sQG, qp, a.q.st, q0, a.Tq);
  load_tile<BWD_B, BWD_THREADS>(sQG + BWD_B * 128, gp, a.dout.st, q0, a.Tq);
  cp_async_commit();
  if (nblk > 0) {
    load_tile<BWD_B, BWD_THREADS>(sK0, kp, a.k.st, 0, a.Tk);
    load_tile<BWD_B, BWD_THREADS>(sV0, vp, a.v.st, 0, a.Tk);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  uint32_t qa[4][4], ga[4][4];
  load_a_frags(sQG, warp * 16, qa);
  load_a_frags(sQG + BWD_B * 128, warp * 16, ga);

  const int ra = q0 + warp * 16 + (lane >> 2);
  const float* lse = a.lse + (int64_t)bh * a.Tq;
  const float* dl = a.delta + (int64_t)bh * a.Tq;
  const float Lr[2] = {ra < a.Tq ? lse[ra] : INFINITY, ra + 8 < a.Tq ? lse[ra + 8] : INFINITY};
  const float Dr[2] = {ra < a.Tq ? dl[ra] : 0.f, ra + 8 < a.Tq ? dl[ra + 8] : 0.f};
  const int absq[2] = {a.q_offset + ra, a.q_offset + ra + 8};
  const float sl2 = a.scale * kLog2e;

  float dq[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;

  for (int j = 0; j < nblk; ++j) {
    const int buf = j & 1;
    if (j + 1 < nblk) {
      const int nb = buf ^ 1;
      load_tile<BWD_B, BWD_THREADS>(sK0 + nb * BWD_B * 128, kp, a.k.st, (j + 1) * BWD_B, a.Tk);
      load_tile<BWD_B, BWD_THREADS>(sV0 + nb * BWD_B * 128, vp, a.v.st, (j + 1) * BWD_B, a.Tk);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sK = sK0 + buf * BWD_B * 128, sV = sV0 + buf * BWD_B * 128;
    const int kv0 = j * BWD_B;

    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    mma_abt(s, qa, sK);
    float dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.f;
    mma_abt(dp, ga, sV);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int col = kv0 + nt * 8 + 2 * (lane & 3) + (i & 1);
        float p = ex2(s[nt][i] * sl2 - Lr[i >> 1]);
        if (col >= a.Tk || (a.causal && col > absq[i >> 1])) p = 0.f;
        s[nt][i] = p * (dp[nt][i] - Dr[i >> 1]);
      }
    }
    // dQ += dS K
    mma_pt(dq, s, sK);
    __syncthreads();
  }
  __nv_bfloat16* dqp = head_ptr_w(a.dq, b, h);
  store_rows(dqp, a.dq.st, q0 + warp * 16, a.Tq, dq, a.scale, a.scale);
}

}  // namespace

static int g_attn_impl = 0;
void attn_set_impl(int impl) { g_attn_impl = impl; }
int attn_get_impl() { return g_attn_impl; }

// Grouped key/value heads: 0 = plain multi-head, 1 = grouped (tensor-core
// kernels only), -1 = invalid grouping.
static int kv_grouping(const AttnArgs& a) {
  const int hkv = a.Hkv > 0 ? a.Hkv : a.H;
  if (hkv > a.H || a.H % hkv) return -1;
  return hkv != a.H;
}

int attn_fwd_launch(const AttnArgs& a, cudaStream_t s) {
  if (a.B <= 0 || a.H <= 0 || a.Tq <= 0 || a.Tk <= 0) return -1;
  const int grouped = kv_grouping(a);
  if (grouped < 0) return -1;
  // grouped heads and keys/values streamed from their owners: tensor cores only
  const bool streamed = a.peers && a.peers->world > 0;
  if ((grouped || streamed) && g_attn_impl != 0) return -12;
  if (g_attn_impl == 0) {
    const int rc = attn_fwd_tc_launch(a, s);
    if (rc == 1) return 0;
    if (rc < 0) return rc;
    if (grouped || streamed) return -12;  // these need TMA-compatible layouts
  }
  const int smem = (FWD_BQ + 4 * FWD_BK) * 128;
  dim3 grid((a.Tq + FWD_BQ - 1) / FWD_BQ, a.B * a.H);
  attn_fwd_kernel<<<grid, FWD_THREADS, smem, s>>>(a);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

int attn_bwd_launch(const AttnArgs& a, cudaStream_t s) {
  if (a.B <= 0 || a.H <= 0 || a.Tq <= 0 || a.Tk <= 0) return -1;
  const int grouped = kv_grouping(a);
  if (grouped < 0) return -1;
  // grouped heads and keys/values streamed from their owners: tensor cores only
  const bool streamed = a.peers && a.peers->world > 0;
  if ((grouped || streamed) && g_attn_impl != 0) return -12;
  const int64_t rows = (int64_t)a.B * a.H * a.Tq;
  auto rows16 = [](const HeadView& v) {
    return (reinterpret_cast<uintptr_t>(v.base) & 15) == 0 && (v.st * 2) % 16 == 0 &&
           (v.sh * 2) % 16 == 0 && (v.sb * 2) % 16 == 0;
  };
  if (rows16(a.o) && rows16(a.dout))
    attn_bwd_delta_kernel<<<(unsigned)((rows * 8 + 255) / 256), 256, 0, s>>>(a);
  else
    attn_bwd_delta_scalar_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(a);
  if (g_attn_impl == 0) {
    const int rc = attn_bwd_tc_launch(a, s);
    if (rc == 1) {
      count_launches(1);  // the delta kernel
      return launch_succeeded() ? 0 : -11;
    }
    if (rc < 0) return rc;
    if (grouped || streamed) return -12;  // these need TMA-compatible layouts
  }
  const int smem_kv = 6 * BWD_B * 128 + 4 * BWD_B * 4;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem_kv) != cudaSuccess)
      return -10;
    attr = true;
  }
  dim3 gkv((a.Tk + BWD_B - 1) / BWD_B, a.B * a.H);
  attn_bwd_dkdv_kernel<<<gkv, BWD_THREADS, smem_kv, s>>>(a);
  const int smem_q = 6 * BWD_B * 128;
  dim3 gq((a.Tq + BWD_B - 1) / BWD_B, a.B * a.H);
  attn_bwd_dq_kernel<<<gq, BWD_THREADS, smem_q, s>>>(a);
  count_launches(3);
  return launch_succeeded() ? 0 : -11;
}

}  // namespace g2b
