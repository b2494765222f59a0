// Causal flash-attention backward on the 5th-generation tensor cores (sm_100a).
//
// Same contract as the mma.sync backward in attention.cu (head_dim 64, bf16
// Q/K/V/O/dO/dQ/dK/dV, log2-domain LSE from the forward, delta = rowsum(dO*O)
// computed first), deterministic (no atomics), re-designed around tcgen05:
//
//  MODE_KV  one CTA owns 128 keys (K_j, V_j stay in shared memory) and walks
//           the 128-query blocks that can see them. Per block:
//             S^T  = K Q^T    and   dP^T = V dO^T        (two MMAs -> TMEM)
//             P^T  = 2^(S^T*scale*log2e - LSE[q])   (masked),
//             dS^T = P^T * (dP^T - delta[q])              (8 warps, -> smem)
//             dV  += P^T dO   and   dK  += dS^T Q        (TMEM accumulators)
//  MODE_Q   one CTA owns 128 queries (Q_i, dO_i stay) and walks the key blocks
//           they can see:  S = Q K^T, dP = dO V^T, P and dS as above,
//             dQ  += dS K.
//
// A query/key tile is loaded once (TMA, 128B swizzle, rows = sequence
// positions, 64 contiguous head dims): it is the K-major operand of the first
// MMAs and, unchanged, the MN-major operand of the accumulating ones.
// Elementwise work needs no row reductions in backward, so the 128x128 tile is
// split by columns across two warps per TMEM lane quarter (8 warps).
// All mbarrier waits are bounded (ERR_TIMEOUT_ATTN).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "attention.cuh"
#include "common.cuh"

namespace g2b {

PFN_cuTensorMapEncodeTiled_v12000 attn_get_encode_fn();

namespace {

constexpr int MODE_KV = 0, MODE_Q = 1;
constexpr int TB = 128;                       // rows per tile
constexpr int TILE = TB * 128;                // 128 rows x 64 bf16
constexpr int STAGES = 2;                     // streaming-operand ring
constexpr int kThreads = 64 + 256;
// smem: stationary A (16K), stationary A2 (16K), ring of 2 x (X 16K + Y 16K),
// P tile (2 x 16K chunks), dS tile (2 x 16K chunks)
constexpr int SA_OFF = 0;
constexpr int SA2_OFF = SA_OFF + TILE;
constexpr int RING_OFF = SA2_OFF + TILE;
constexpr int P_OFF = RING_OFF + STAGES * 2 * TILE;
constexpr int DS_OFF = P_OFF + 2 * TILE;
constexpr int BAR_OFF = DS_OFF + 2 * TILE;
constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
constexpr float kLog2e = 1.4426950408889634f;

struct BwdParams {
  int H, Tq, Tk, q_offset, causal;
  float sl2, scale;
  const float* lse;
  const float* delta;
  __nv_bfloat16* out1;  // dK (MODE_KV) or dQ (MODE_Q)
  __nv_bfloat16* out2;  // dV (MODE_KV)
  int64_t o1_sb, o1_st, o1_sh, o2_sb, o2_st, o2_sh;
  uint32_t* err;
};

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Write 32 values (quarter `c` of row half `half`) as bf16 into a K-major
// 128B-swizzled tile made of two 16 KB chunks of 64 columns.
__device__ __forceinline__ void put_row_quarter(uint8_t* tile, int r, int half, int c,
                                                const float* v) {
  uint8_t* base = tile + half * TILE + r * 128;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = c * 4 + j;
    uint4 w;
    w.x = pack_bf16x2(v[j * 8 + 0], v[j * 8 + 1]);
    w.y = pack_bf16x2(v[j * 8 + 2], v[j * 8 + 3]);
    w.z = pack_bf16x2(v[j * 8 + 4], v[j * 8 + 5]);
    w.w = pack_bf16x2(v[j * 8 + 6], v[j * 8 + 7]);
    *reinterpret_cast<uint4*>(base + ((q ^ (r & 7)) << 4)) = w;
  }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                       const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmY,
                       const BwdParams p) {
  // MODE_KV: A = K, A2 = V (stationary); X = Q_i, Y = dO_i (streaming)
  // MODE_Q : A = Q, A2 = dO (stationary); X = K_j, Y = V_j (streaming)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* a_full = bars;                 // 1
  uint64_t* x_full = bars + 1;             // STAGES
  uint64_t* x_empty = x_full + STAGES;     // STAGES
  uint64_t* s_full = x_empty + STAGES;     // 1: S and dP ready in TMEM
  uint64_t* e_full = s_full + 1;           // 1: P / dS written to smem (256 arrivals)
  uint64_t* e_free = e_full + 1;           // 1: accumulating MMAs done with P / dS
  uint64_t* acc_full = e_free + 1;         // 1: final accumulators ready
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int blk = (MODE == MODE_Q) ? (gridDim.x - 1 - blockIdx.x) : blockIdx.x;
  const int r0 = blk * TB;  // first key (KV) / query (Q) row of this CTA

  // Range of streaming blocks.
  int it0 = 0, it1 = 0;
  if (MODE == MODE_KV) {
    const int nq = (p.Tq + TB - 1) / TB;
    it0 = p.causal ? max(0, (r0 - p.q_offset) / TB) : 0;
    it1 = (r0 < p.Tk) ? nq : 0;
  } else {
    int kv_end = p.Tk;
    if (p.causal) kv_end = min(p.Tk, p.q_offset + r0 + TB);
    it1 = (r0 < p.Tq && kv_end > 0) ? (kv_end + TB - 1) / TB : 0;
  }
  const int n_it = max(0, it1 - it0);

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(e_full, 256);
    mbar_init(e_free, 1);
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S [0,128) dP [128,256) acc1 [256,320) acc2 [320,384)
  const uint32_t T_S = 0, T_DP = 128, T_A1 = 256, T_A2 = 320;

  if (warp == 0) {
    if (elect_one() && n_it > 0) {
      mbar_arrive_expect_tx(a_full, 2 * TILE);
      tma_load_4d(smem + SA_OFF, &tmA, a_full, 0, h, r0, b);
      tma_load_4d(smem + SA2_OFF, &tmA2, a_full, 0, h, r0, b);
      for (int k = 0; k < n_it; ++k) {
        const int st = k % STAGES;
        if (!mbar_wait_bounded(&x_empty[st], ((k / STAGES) & 1) ^ 1, p.err, ERR_TIMEOUT_ATTN,
                               abort_flag))
          break;
        mbar_arrive_expect_tx(&x_full[st], 2 * TILE);
        const int row = (it0 + k) * TB;
        tma_load_4d(smem + RING_OFF + st * 2 * TILE, &tmX, &x_full[st], 0, h, row, b);
        tma_load_4d(smem + RING_OFF + st * 2 * TILE + TILE, &tmY, &x_full[st], 0, h, row, b);
      }
    }
  } else if (warp == 1) {
    if (elect_one() && n_it > 0) {
      constexpr uint32_t id_ss = umma_idesc_bf16(128, 128, 0, 0);  // K-major x K-major
      constexpr uint32_t id_acc = umma_idesc_bf16(128, 64, 0, 1);  // K-major A, MN-major B
      const uint32_t sa = smem_u32(smem + SA_OFF), sa2 = smem_u32(smem + SA2_OFF);
      const uint32_t sp = smem_u32(smem + P_OFF), sds = smem_u32(smem + DS_OFF);
      bool ok = mbar_wait_bounded(a_full, 0, p.err, ERR_TIMEOUT_ATTN, abort_flag);
      for (int k = 0; k < n_it && ok; ++k) {
        const int st = k % STAGES;
        if (!mbar_wait_bounded(&x_full[st], (k / STAGES) & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sx = smem_u32(smem + RING_OFF + st * 2 * TILE), sy = sx + TILE;
        // S(^T) = A X^T and dP(^T) = A2 Y^T  (K = head dim 64)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          umma_bf16(tmem + T_S, umma_desc_sw128(sa + kk * 32, 16, 1024),
                    umma_desc_sw128(sx + kk * 32, 16, 1024), id_ss, kk > 0 ? 1u : 0u);
          umma_bf16(tmem + T_DP, umma_desc_sw128(sa2 + kk * 32, 16, 1024),
                    umma_desc_sw128(sy + kk * 32, 16, 1024), id_ss, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        // P / dS written by the elementwise warps (they have also consumed S, dP)
        if (!mbar_wait_bounded(e_full, k & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // accumulate over the streaming dimension (K = 128 rows of the tile)
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (ks >> 2) * TILE + (ks & 3) * 32;
          const uint32_t acc = (k > 0 || ks > 0) ? 1u : 0u;
          if (MODE == MODE_KV) {
            // dV += P^T dO ; dK += dS^T Q
            umma_bf16(tmem + T_A2, umma_desc_sw128(sp + off, 16, 1024),
                      umma_desc_sw128(sy + ks * 2048, 8192, 1024), id_acc, acc);
            umma_bf16(tmem + T_A1, umma_desc_sw128(sds + off, 16, 1024),
                      umma_desc_sw128(sx + ks * 2048, 8192, 1024), id_acc, acc);
          } else {
            // dQ += dS K
            umma_bf16(tmem + T_A1, umma_desc_sw128(sds + off, 16, 1024),
                      umma_desc_sw128(sx + ks * 2048, 8192, 1024), id_acc, acc);
          }
        }
        umma_commit(e_free);
        umma_commit(&x_empty[st]);
      }
      if (ok) umma_commit(acc_full);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------- elementwise
    const int ew = warp - 2;
    const int lg = warp & 3;
    const int half = ew >> 2;             // which 64 columns of the 128
    const int lane = (int)lane_id();
    const int r = lg * 32 + lane;         // row of the tile (TMEM lane)
    const int row_pos = r0 + r;           // key (KV) or query (Q) position
    const uint32_t lane_base = tmem + ((uint32_t)(lg * 32) << 16);
    uint8_t* ptile = smem + P_OFF;
    uint8_t* dstile = smem + DS_OFF;
    // MODE_Q: per-row LSE / delta
    float row_lse = 0.f, row_delta = 0.f;
    if (MODE == MODE_Q && row_pos < p.Tq) {
      row_lse = p.lse[(int64_t)bh * p.Tq + row_pos];
      row_delta = p.delta[(int64_t)bh * p.Tq + row_pos];
    }
    const int abs_row = (MODE == MODE_Q) ? p.q_offset + row_pos : row_pos;
    bool ok = true;
    for (int k = 0; k < n_it && ok; ++k) {
      const int c0 = (it0 + k) * TB + half * 64;  // first column position of this half
      if (!mbar_wait_bounded(s_full, k & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // P/dS smem is free once the previous accumulation finished; MMAs
      // complete in issue order, so that happened before S/dP(k) landed.
      if (k > 0 && !mbar_wait_bounded(e_free, (k - 1) & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t sv[32], dv[32];
        tmem_ld32_async(lane_base + T_S + half * 64 + c * 32, sv);
        tmem_ld32_async(lane_base + T_DP + half * 64 + c * 32, dv);
        tmem_wait_ld_into(sv);
        tmem_wait_ld_into(dv);
        float pv[32], dsv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int col = c0 + c * 32 + i;
          const float sc = __uint_as_float(sv[i]);
          const float dp = __uint_as_float(dv[i]);
          float lse, dl;
          bool vis;
          if (MODE == MODE_KV) {
            const bool in = col < p.Tq;
            lse = in ? __ldg(p.lse + (int64_t)bh * p.Tq + col) : 0.f;
            dl = in ? __ldg(p.delta + (int64_t)bh * p.Tq + col) : 0.f;
            vis = in && row_pos < p.Tk && (!p.causal || p.q_offset + col >= abs_row);
          } else {
            lse = row_lse;
            dl = row_delta;
            vis = col < p.Tk && row_pos < p.Tq && (!p.causal || col <= abs_row);
          }
          const float pr = vis ? ex2f(fmaf(sc, p.sl2, -lse)) : 0.f;
          pv[i] = pr;
          dsv[i] = pr * (dp - dl);
        }
        if (MODE == MODE_KV) put_row_quarter(ptile, r, half, c, pv);
        put_row_quarter(dstile, r, half, c, dsv);
      }
      fence_proxy_async_shared();
      tc_fence_before();
      mbar_arrive(e_full);
    }
    // final accumulators -> global (each warp writes its 32 rows, its half of d)
    if (ok && n_it > 0 && mbar_wait_bounded(acc_full, 0, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
      tc_fence_after();
      const int nacc = (MODE == MODE_KV) ? 2 : 1;
      for (int a = 0; a < nacc; ++a) {
        uint32_t v[32];
        tmem_ld32_async(lane_base + (a == 0 ? T_A1 : T_A2) + half * 32, v);
        tmem_wait_ld_into(v);
        const bool inb = (MODE == MODE_KV) ? row_pos < p.Tk : row_pos < p.Tq;
        if (inb) {
          const float sc = (a == 0) ? p.scale : 1.f;  // dK / dQ carry the softmax scale
          __nv_bfloat16* dst = (a == 0) ? p.out1 + (int64_t)b * p.o1_sb + (int64_t)row_pos * p.o1_st +
                                              (int64_t)h * p.o1_sh
                                        : p.out2 + (int64_t)b * p.o2_sb + (int64_t)row_pos * p.o2_st +
                                              (int64_t)h * p.o2_sh;
          dst += half * 32;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[q * 8 + 0]) * sc, __uint_as_float(v[q * 8 + 1]) * sc);
            w.y = pack_bf16x2(__uint_as_float(v[q * 8 + 2]) * sc, __uint_as_float(v[q * 8 + 3]) * sc);
            w.z = pack_bf16x2(__uint_as_float(v[q * 8 + 4]) * sc, __uint_as_float(v[q * 8 + 5]) * sc);
            w.w = pack_bf16x2(__uint_as_float(v[q * 8 + 6]) * sc, __uint_as_float(v[q * 8 + 7]) * sc);
            reinterpret_cast<uint4*>(dst)[q] = w;
          }
        }
      }
    } else if (n_it == 0) {
      // no visible partner block: the gradient of this row is zero
      const bool inb = (MODE == MODE_KV) ? row_pos < p.Tk : row_pos < p.Tq;
      if (inb) {
        const int nacc = (MODE == MODE_KV) ? 2 : 1;
        for (int a = 0; a < nacc; ++a) {
          __nv_bfloat16* dst = (a == 0) ? p.out1 + (int64_t)b * p.o1_sb + (int64_t)row_pos * p.o1_st +
                                              (int64_t)h * p.o1_sh
                                        : p.out2 + (int64_t)b * p.o2_sb + (int64_t)row_pos * p.o2_st +
                                              (int64_t)h * p.o2_sh;
          dst += half * 32;
#pragma unroll
          for (int q = 0; q < 4; ++q) reinterpret_cast<uint4*>(dst)[q] = make_uint4(0, 0, 0, 0);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool head_map(CUtensorMap* tm, const HeadView& v, int H, int T, int B) {
  auto enc = attn_get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[4] = {64, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)v.sh * 2, (cuuint64_t)v.st * 2, (cuuint64_t)v.sb * 2};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, v.base, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tma_ok(const HeadView& v) {
  return (reinterpret_cast<uintptr_t>(v.base) & 15) == 0 && (v.sh * 2) % 16 == 0 &&
         (v.st * 2) % 16 == 0 && (v.sb * 2) % 16 == 0;
}

bool out_ok(const HeadView& v) {
  return (reinterpret_cast<uintptr_t>(v.base) & 15) == 0 && (v.sh * 2) % 16 == 0 &&
         (v.st * 2) % 16 == 0;
}

template <int MODE>
int launch_mode(const CUtensorMap& a, const CUtensorMap& a2, const CUtensorMap& x,
                const CUtensorMap& y, const BwdParams& p, dim3 grid, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_bwd_tc_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES) != cudaSuccess)
      return -10;
    attr = true;
  }
  attn_bwd_tc_kernel<MODE><<<grid, kThreads, SMEM_BYTES, s>>>(a, a2, x, y, p);
  count_launches(1);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

}  // namespace

// Tensor-core backward (after delta has been computed into a.delta): returns
// 1 if it ran, 0 when a layout is not TMA-compatible, negative on failure.
int attn_bwd_tc_launch(const AttnArgs& a, cudaStream_t s) {
  if (!tma_ok(a.q) || !tma_ok(a.k) || !tma_ok(a.v) || !tma_ok(a.dout) || !out_ok(a.dq) ||
      !out_ok(a.dk) || !out_ok(a.dv))
    return 0;
  CUtensorMap tq, tk, tv, tdo;
  if (!head_map(&tq, a.q, a.H, a.Tq, a.B) || !head_map(&tk, a.k, a.H, a.Tk, a.B) ||
      !head_map(&tv, a.v, a.H, a.Tk, a.B) || !head_map(&tdo, a.dout, a.H, a.Tq, a.B))
    return 0;
  BwdParams p;
  p.H = a.H;
  p.Tq = a.Tq;
  p.Tk = a.Tk;
  p.q_offset = a.q_offset;
  p.causal = a.causal;
  p.scale = a.scale;
  p.sl2 = a.scale * kLog2e;
  p.lse = a.lse;
  p.delta = a.delta;
  p.err = a.err;
  // dK / dV
  p.out1 = reinterpret_cast<__nv_bfloat16*>(a.dk.base);
  p.o1_sb = a.dk.sb;
  p.o1_st = a.dk.st;
  p.o1_sh = a.dk.sh;
  p.out2 = reinterpret_cast<__nv_bfloat16*>(a.dv.base);
  p.o2_sb = a.dv.sb;
  p.o2_st = a.dv.st;
  p.o2_sh = a.dv.sh;
  int rc = launch_mode<MODE_KV>(tk, tv, tq, tdo, p, dim3((a.Tk + TB - 1) / TB, a.B * a.H), s);
  if (rc) return rc;
  // dQ
  p.out1 = reinterpret_cast<__nv_bfloat16*>(a.dq.base);
  p.o1_sb = a.dq.sb;
  p.o1_st = a.dq.st;
  p.o1_sh = a.dq.sh;
  p.out2 = nullptr;
  rc = launch_mode<MODE_Q>(tq, tdo, tk, tv, p, dim3((a.Tq + TB - 1) / TB, a.B * a.H), s);
  return rc ? rc : 1;
}

}  // namespace g2b
