// Causal flash-attention forward on the 5th-generation tensor cores (sm_100a).
//
// Same contract as attn_fwd_kernel in attention.cu (head_dim 64, bf16 Q/K/V/O,
// log2-domain row LSE saved for backward, implicit causal mask at absolute
// positions q_offset + i vs j), re-designed around tcgen05:
//
//  * A CTA owns TWO 128-query tiles of one (batch, head) and streams 128-key
//    K/V blocks through a 3-stage TMA ring shared by both tiles.
//  * warp 0: TMA producer (4-D tensor maps over the strided head views, so Q,
//    K, V are read straight out of the fused qkv buffer).
//    warp 1: MMA issuer. Per key block and tile: S = Q K^T (128x128x64, both
//    operands K-major, fp32 accumulator in TMEM), then O_tile = P V
//    (128x64x128; P from shared memory, V as an MN-major operand).
//    warps 2-5 / 6-9: one softmax warpgroup per query tile (FA4-style
//    ping-pong: while one group does exponentials the tensor core works on
//    the other tile). A thread owns one query row = one TMEM lane.
//  * Online softmax: pass 1 reads the S row from TMEM for the row max, pass 2
//    re-reads it, exponentiates (exp2 domain), accumulates the row sum and
//    writes P as bf16 into a 128B-swizzled K-major shared tile the next MMA
//    consumes. The per-block P.V product lands in a fresh TMEM accumulator and
//    is folded into a register accumulator with the running max correction
//    one block behind, so the P.V MMA overlaps the next block's softmax.
//  * Every mbarrier wait is bounded (ERR_TIMEOUT_ATTN on expiry).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>

#include "attention.cuh"
#include "common.cuh"

namespace g2b {

PFN_cuTensorMapEncodeTiled_v12000 attn_get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) !=
            cudaSuccess ||
        qres != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

namespace {

constexpr int TQ = 128;  // query rows per tile
constexpr int NG = 2;    // query tiles (softmax warpgroups) per CTA
constexpr int TKV = 128; // keys per block
constexpr int KS = 3;    // K/V ring stages
constexpr int kThreads = 64 + NG * 128;
constexpr int TILE_BYTES = 128 * 128;         // 128 rows x 64 bf16
constexpr int Q_OFF = 0;
constexpr int K_OFF = Q_OFF + NG * TILE_BYTES;
constexpr int V_OFF = K_OFF + KS * TILE_BYTES;
constexpr int P_OFF = V_OFF + KS * TILE_BYTES;  // per group: 2 chunks of 64 keys
constexpr int BAR_OFF = P_OFF + NG * 2 * TILE_BYTES;
constexpr int SMEM_BYTES = BAR_OFF + 512 + 1024;
constexpr float kLog2e = 1.4426950408889634f;

struct TcParams {
  int B, H, Tq, Tk, q_offset, causal;
  float sl2;  // softmax scale * log2(e)
  __nv_bfloat16* o;
  int64_t osb, ost, osh;
  float* lse;
  uint32_t* err;
};

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* q_full = bars;             // 1
  uint64_t* kv_full = bars + 1;        // KS
  uint64_t* kv_empty = kv_full + KS;   // KS
  uint64_t* s_full = kv_empty + KS;    // NG
  uint64_t* p_full = s_full + NG;      // NG
  uint64_t* o_full = p_full + NG;      // NG
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + NG);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int qblk = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int q0 = qblk * (NG * TQ);

  // number of key blocks each tile needs
  int nblk[NG];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    int kv_end = p.Tk;
    if (p.causal) kv_end = min(p.Tk, p.q_offset + q0 + (g + 1) * TQ);
    const bool tile_live = q0 + g * TQ < p.Tq;
    nblk[g] = (tile_live && kv_end > 0) ? (kv_end + TKV - 1) / TKV : 0;
  }
  const int nmax = max(nblk[0], nblk[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int g = 0; g < NG; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], 128);
      mbar_init(&o_full[g], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane_id() == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one() && nmax > 0) {
      mbar_arrive_expect_tx(q_full, NG * TILE_BYTES);
      for (int g = 0; g < NG; ++g)
        tma_load_4d(smem + Q_OFF + g * TILE_BYTES, &tmQ, q_full, 0, h, q0 + g * TQ, b);
      for (int j = 0; j < nmax; ++j) {
        const int st = j % KS;
        if (!mbar_wait_bounded(&kv_empty[st], ((j / KS) & 1) ^ 1, p.err, ERR_TIMEOUT_ATTN,
                               abort_flag))
          break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * TILE_BYTES);
        tma_load_4d(smem + K_OFF + st * TILE_BYTES, &tmK, &kv_full[st], 0, h, j * TKV, b);
        tma_load_4d(smem + V_OFF + st * TILE_BYTES, &tmV, &kv_full[st], 0, h, j * TKV, b);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (elect_one() && nmax > 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(128, 64, 0, 1);
      auto issue_s = [&](int g, int st) {
        const uint32_t qa = smem_u32(smem + Q_OFF + g * TILE_BYTES);
        const uint32_t kb = smem_u32(smem + K_OFF + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tmem + g * 128, umma_desc_sw128(qa + kk * 32, 16, 1024),
                    umma_desc_sw128(kb + kk * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[g]);
      };
      bool ok = mbar_wait_bounded(q_full, 0, p.err, ERR_TIMEOUT_ATTN, abort_flag) &&
                mbar_wait_bounded(&kv_full[0], 0, p.err, ERR_TIMEOUT_ATTN, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int g = 0; g < NG; ++g)
          if (nblk[g] > 0) issue_s(g, 0);
      }
      for (int j = 0; j < nmax && ok; ++j) {
        const int st = j % KS;
        for (int g = 0; g < NG && ok; ++g) {
          if (j >= nblk[g]) continue;
          // P_g(j) written (which also means S_g(j) and O_g(j-1) were consumed)
          if (!mbar_wait_bounded(&p_full[g], j & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t pa = smem_u32(smem + P_OFF + g * 2 * TILE_BYTES);
          const uint32_t vb = smem_u32(smem + V_OFF + st * TILE_BYTES);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma_bf16(tmem + 256 + g * 64,
                      umma_desc_sw128(pa + (ks >> 2) * TILE_BYTES + (ks & 3) * 32, 16, 1024),
                      umma_desc_sw128(vb + ks * 2048, 8192, 1024), idesc_pv, ks > 0 ? 1u : 0u);
          umma_commit(&o_full[g]);
          if (j + 1 < nblk[g]) {
            const int st2 = (j + 1) % KS;
            if (!mbar_wait_bounded(&kv_full[st2], ((j + 1) / KS) & 1, p.err, ERR_TIMEOUT_ATTN,
                                   abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(g, st2);
          }
        }
        umma_commit(&kv_empty[st]);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- softmax
    const int g = (warp - 2) >> 2;
    const int lg = warp & 3;
    const int lane = (int)lane_id();
    const int r = lg * 32 + lane;
    const int row_q = q0 + g * TQ + r;
    const int abs_q = p.q_offset + row_q;
    const int n = nblk[g];
    const uint32_t t_s = tmem + ((uint32_t)(lg * 32) << 16) + g * 128;
    const uint32_t t_o = tmem + ((uint32_t)(lg * 32) << 16) + 256 + g * 64;
    uint8_t* pbuf = smem + P_OFF + g * 2 * TILE_BYTES;
    float m = -INFINITY, l = 0.f, corr_prev = 0.f;
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] = 0.f;
    const int tile_q_min = p.q_offset + q0 + g * TQ;
    bool ok = true;

    auto fold_o = [&](int j) -> bool {  // O = O * corr_prev + O_tmp(j)
      if (!mbar_wait_bounded(&o_full[g], j & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) return false;
      tc_fence_after();
      uint32_t t0[32], t1[32];
      tmem_ld32_async(t_o, t0);
      tmem_ld32_async(t_o + 32, t1);
      tmem_wait_ld_into(t0);
      tmem_wait_ld_into(t1);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        o[i] = fmaf(o[i], corr_prev, __uint_as_float(t0[i]));
        o[32 + i] = fmaf(o[32 + i], corr_prev, __uint_as_float(t1[i]));
      }
      return true;
    };

    for (int j = 0; j < n && ok; ++j) {
      if (!mbar_wait_bounded(&s_full[g], j & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = j * TKV;
      const bool need_mask = (k0 + TKV > p.Tk) || (p.causal && k0 + TKV - 1 > tile_q_min);
      // Keys of this block visible to this row: [k0, k0 + valid).
      int valid = TKV;
      if (need_mask) {
        int lim = p.Tk;
        if (p.causal) lim = min(lim, abs_q + 1);
        valid = max(0, min(TKV, lim - k0));
      }
      // pass 1: row max of the raw scores (8 independent chains; loads one
      // chunk ahead of the arithmetic)
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
      {
        uint32_t a[32], b[32];
        tmem_ld32_async(t_s, a);
        tmem_wait_ld_into(a);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t(&cur)[32] = (c & 1) ? b : a;
          uint32_t(&nxt)[32] = (c & 1) ? a : b;
          if (c < 3) tmem_ld32_async(t_s + (c + 1) * 32, nxt);
          if (need_mask) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float v = (c * 32 + i < valid) ? __uint_as_float(cur[i]) : -INFINITY;
              mx8[i & 7] = fmaxf(mx8[i & 7], v);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(cur[i]));
          }
          if (c < 3) tmem_wait_ld_into(nxt);
        }
      }
      float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      mx = mx == -INFINITY ? -INFINITY : mx * p.sl2;
      const float m_new = fmaxf(m, mx);
      const float base = m_new == -INFINITY ? 0.f : m_new;
      const float corr = ex2f(m - base);
      // the previous block's P.V is done: fold it in (frees O_tmp and P)
      if (j >= 1 && !fold_o(j - 1)) {
        ok = false;
        break;
      }
      // pass 2: p = 2^(s*sl2 - base), row sum (8 chains), bf16 P into the
      // swizzled K-major tile
      float rs8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) rs8[i] = 0.f;
      {
        uint32_t a[32], b[32];
        tmem_ld32_async(t_s, a);
        tmem_wait_ld_into(a);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t(&cur)[32] = (c & 1) ? b : a;
          uint32_t(&nxt)[32] = (c & 1) ? a : b;
          if (c < 3) tmem_ld32_async(t_s + (c + 1) * 32, nxt);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float e[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const int i = q * 8 + t;
              float v = ex2f(fmaf(__uint_as_float(cur[i]), p.sl2, -base));
              if (need_mask) v = (c * 32 + i < valid) ? v : 0.f;
              e[t] = v;
              rs8[t] += v;
            }
            const int jj = c * 4 + q;  // 16-byte chunk (8 keys) index 0..15
            uint4 w;
            w.x = pack_bf16x2(e[0], e[1]);
            w.y = pack_bf16x2(e[2], e[3]);
            w.z = pack_bf16x2(e[4], e[5]);
            w.w = pack_bf16x2(e[6], e[7]);
            *reinterpret_cast<uint4*>(pbuf + (jj >> 3) * TILE_BYTES + r * 128 +
                                      (((jj & 7) ^ (r & 7)) << 4)) = w;
          }
          if (c < 3) tmem_wait_ld_into(nxt);
        }
      }
      fence_proxy_async_shared();
      tc_fence_before();
      mbar_arrive(&p_full[g]);
      const float rs = ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
      l = l * corr + rs;
      corr_prev = corr;
      m = m_new;
    }
    if (ok && n > 0 && fold_o(n - 1) && row_q < p.Tq) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + (int64_t)b * p.osb + (int64_t)row_q * p.ost + (int64_t)h * p.osh;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint4 w;
        w.x = pack_bf16x2(o[q * 8 + 0] * inv, o[q * 8 + 1] * inv);
        w.y = pack_bf16x2(o[q * 8 + 2] * inv, o[q * 8 + 3] * inv);
        w.z = pack_bf16x2(o[q * 8 + 4] * inv, o[q * 8 + 5] * inv);
        w.w = pack_bf16x2(o[q * 8 + 6] * inv, o[q * 8 + 7] * inv);
        reinterpret_cast<uint4*>(orow)[q] = w;
      }
      p.lse[(int64_t)bh * p.Tq + row_q] = m + log2f(l);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// 4-D bf16 map over a strided head view: dims {64 (d), H, T, B}, 64 x 1 x 128 x 1
// boxes (128 rows of one head = one K-major 128B-swizzled tile).
bool make_head_map(CUtensorMap* tm, const HeadView& v, int H, int T, int B) {
  auto enc = attn_get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[4] = {64, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)v.sh * 2, (cuuint64_t)v.st * 2, (cuuint64_t)v.sb * 2};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, v.base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool head_view_tma_ok(const HeadView& v) {
  return (reinterpret_cast<uintptr_t>(v.base) & 15) == 0 && (v.sh * 2) % 16 == 0 &&
         (v.st * 2) % 16 == 0 && (v.sb * 2) % 16 == 0;
}

}  // namespace

// Returns 1 if the tensor-core path ran, 0 if the caller must use the
// mma.sync kernel (layout not TMA-compatible), negative on launch failure.
int attn_fwd_tc_launch(const AttnArgs& a, cudaStream_t s) {
  if (!head_view_tma_ok(a.q) || !head_view_tma_ok(a.k) || !head_view_tma_ok(a.v)) return 0;
  if ((a.o.sh * 2) % 16 || (a.o.st * 2) % 16 || (reinterpret_cast<uintptr_t>(a.o.base) & 15))
    return 0;
  CUtensorMap tq, tk, tv;
  if (!make_head_map(&tq, a.q, a.H, a.Tq, a.B) || !make_head_map(&tk, a.k, a.H, a.Tk, a.B) ||
      !make_head_map(&tv, a.v, a.H, a.Tk, a.B))
    return 0;
  TcParams p;
  p.B = a.B;
  p.H = a.H;
  p.Tq = a.Tq;
  p.Tk = a.Tk;
  p.q_offset = a.q_offset;
  p.causal = a.causal;
  p.sl2 = a.scale * kLog2e;
  p.o = reinterpret_cast<__nv_bfloat16*>(a.o.base);
  p.osb = a.o.sb;
  p.ost = a.o.st;
  p.osh = a.o.sh;
  p.lse = a.lse;
  p.err = a.err;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES) != cudaSuccess)
      return -10;
    attr = true;
  }
  dim3 grid((a.Tq + NG * TQ - 1) / (NG * TQ), a.B * a.H);
  attn_fwd_tc_kernel<<<grid, kThreads, SMEM_BYTES, s>>>(tq, tk, tv, p);
  count_launches(1);
  return cudaGetLastError() == cudaSuccess ? 1 : -11;
}

}  // namespace g2b
