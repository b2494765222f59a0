// Causal flash-attention backward on the 5th-generation tensor cores (sm_100a).
//
// Same contract as the mma.sync backward in attention.cu (head_dim 64, bf16
// Q/K/V/O/dO/dQ/dK/dV, log2-domain LSE from the forward, delta = rowsum(dO*O)
// computed first), deterministic (no atomics), re-designed around tcgen05:
//
//  MODE_KV  a tile is 128 keys (K_j, V_j stay in shared memory); the CTA walks
//           the 64-query steps that can see them. Per step:
//             S^T  = K Q^T    and   dP^T = V dO^T        (two MMAs -> TMEM)
//             P^T  = 2^(S^T*scale*log2e - LSE[q])   (masked),
//             dS^T = P^T * (dP^T - delta[q])              (8 warps, -> smem)
//             dV  += P^T dO   and   dK  += dS^T Q        (TMEM accumulators)
//  MODE_Q   a tile is 128 queries (Q_i, dO_i stay); the CTA walks the 64-key
//           steps they can see:  S = Q K^T, dP = dO V^T, P and dS as above,
//             dQ  += dS K.
//
// Pipelining. S/dP live in two TMEM buffers (64 columns each per step), and
// P/dS in two shared-memory buffers, so while the elementwise warps turn step
// g into P/dS, the tensor core accumulates step g-1 and computes S/dP of
// step g+1. The kernel is persistent (one CTA per SM, heavy tiles first under
// the causal mask) with two TMEM accumulator sets, so the write-out of one
// tile overlaps the first steps of the next. In MODE_KV the producer warp
// stages each step's 64 LSE / delta values next to the Q/dO tiles.
//
// A query/key tile is loaded once (TMA, 128B swizzle, rows = sequence
// positions, 64 contiguous head dims): it is the K-major operand of the first
// MMAs and, unchanged, the MN-major operand of the accumulating ones.
// All mbarrier waits are bounded (ERR_TIMEOUT_ATTN).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "attention.cuh"
#include "attention_peers.cuh"
#include "common.cuh"

namespace g2b {

PFN_cuTensorMapEncodeTiled_v12000 attn_get_encode_fn();

namespace {

constexpr int MODE_KV = 0, MODE_Q = 1;
constexpr int TB = 128;                       // stationary rows per tile
constexpr int SB = 64;                        // streaming rows per step
constexpr int ATILE = TB * 128;               // 128 rows x 64 bf16 (16 KB)
constexpr int XTILE = SB * 128;               // 64 rows x 64 bf16 (8 KB)
constexpr int STAGES = 4;                     // streaming-operand ring
#ifndef G2B_BWD_EW_WARPS
#define G2B_BWD_EW_WARPS 16
#endif
constexpr int kEw = G2B_BWD_EW_WARPS;         // elementwise warps (kEw/4 per TMEM lane quarter)
constexpr int NC = 64 / (kEw / 4);            // columns of a step per elementwise thread
constexpr int kEwThreads = kEw * 32;
constexpr int kThreads = 64 + kEwThreads;
// smem: stationary A, A2 (16 KB each); ring of STAGES x (X 8K + Y 8K);
// P and dS double buffers (128 rows x 64 cols bf16 = 16 KB each);
// per-stage LSE/delta (2 x 64 floats); barriers.
constexpr int SA_OFF = 0;
constexpr int SA2_OFF = SA_OFF + ATILE;
constexpr int RING_OFF = SA2_OFF + ATILE;
constexpr int P_OFF = RING_OFF + STAGES * 2 * XTILE;
constexpr int DS_OFF = P_OFF + 2 * ATILE;
constexpr int LD_OFF = DS_OFF + 2 * ATILE;
constexpr int BAR_OFF = LD_OFF + STAGES * 2 * SB * 4;
constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
constexpr float kLog2e = 1.4426950408889634f;

struct BwdParams {
  // H / BH: heads of the stationary operand (key/value heads in MODE_KV,
  // query heads in MODE_Q); grp: query heads per key/value head; Hq: query
  // heads (row blocks of lse / delta).
  int H, BH, Tq, Tk, q_offset, causal, n_blk, n_tiles, grp, Hq;
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

// Tile t of the persistent schedule: (batch*head, first stationary row,
// first streaming row, number of 64-row steps, steps per query head). In
// MODE_KV with grouped heads the steps walk the visible queries of every
// query head of the group in turn (step j: head j / nph of the group, rows
// s0 + (j % nph) * 64), all accumulating into the same dK/dV.
struct TileInfo {
  int bh, r0, s0, n, nph;
};

template <int MODE>
__device__ __forceinline__ TileInfo tile_info(const BwdParams& p, int t) {
  TileInfo ti;
  // Heaviest blocks first: under the causal mask the work of a key block
  // falls with its index (MODE_KV) and that of a query block rises (MODE_Q).
  const int rank = t / p.BH;
  ti.bh = t % p.BH;
  const int blk = (MODE == MODE_KV) ? rank : (p.n_blk - 1 - rank);
  ti.r0 = blk * TB;
  if (MODE == MODE_KV) {
    int q0 = p.causal ? max(0, ti.r0 - p.q_offset) : 0;
    q0 = (q0 / SB) * SB;
    ti.s0 = q0;
    ti.nph = (ti.r0 < p.Tk && q0 < p.Tq) ? (p.Tq - q0 + SB - 1) / SB : 0;
    ti.n = ti.nph * p.grp;
  } else {
    int kv_end = p.Tk;
    if (p.causal) kv_end = min(p.Tk, p.q_offset + ti.r0 + TB);
    ti.s0 = 0;
    ti.n = (ti.r0 < p.Tq && kv_end > 0) ? (kv_end + SB - 1) / SB : 0;
    ti.nph = ti.n;
  }
  return ti;
}

// N-column TMEM load of this thread's lane (asynchronous; see tmem_wait_into).
template <int N>
__device__ __forceinline__ void tmem_ld_nc(uint32_t taddr, uint32_t (&r)[N]) {
  static_assert(N == 16 || N == 32, "16 or 32 columns");
  if constexpr (N == 32) tmem_ld32_async(taddr, r);
  else tmem_ld16_async(taddr, r);
}
template <int N>
__device__ __forceinline__ void tmem_wait_into(uint32_t (&a)[N], uint32_t (&b)[N]) {
  if constexpr (N == 32) {
    tmem_wait_ld_into(a);
    tmem_wait_ld_into(b);
  } else {
    tmem_wait_ld_into16x2(a, b);
  }
}

// Write NC values (columns NC*grp .. +NC of row r) as bf16 into a K-major
// 128B-swizzled 128x64 tile (NC/8 16-byte chunks of the row's 128 bytes).
__device__ __forceinline__ void put_row(uint8_t* tile, int r, int grp, const uint32_t (&v)[NC]) {
  uint8_t* base = tile + r * 128;
#pragma unroll
  for (int j = 0; j < NC / 8; ++j) {
    const int q = grp * (NC / 8) + j;
    uint4 w;
    w.x = pack_bf16x2(__uint_as_float(v[j * 8 + 0]), __uint_as_float(v[j * 8 + 1]));
    w.y = pack_bf16x2(__uint_as_float(v[j * 8 + 2]), __uint_as_float(v[j * 8 + 3]));
    w.z = pack_bf16x2(__uint_as_float(v[j * 8 + 4]), __uint_as_float(v[j * 8 + 5]));
    w.w = pack_bf16x2(__uint_as_float(v[j * 8 + 6]), __uint_as_float(v[j * 8 + 7]));
    *reinterpret_cast<uint4*>(base + ((q ^ (r & 7)) << 4)) = w;
  }
}

// Elementwise step of MODE_KV for one thread's NC columns (queries c0..),
// in place: S^T -> P^T = 2^(S^T*sl2 - lse[q]), dP^T -> dS^T = P^T (dP^T - delta[q]).
// With MASK an element is kept iff its query is in range, the row is in range
// and (causal) the query position is >= min_q (= key position - q_offset).
// The mask test sits outside the element loop so each variant is one
// straight-line block the compiler can interleave across elements.
// Every exponential runs on the exponential unit: the FMA and ALU pipes carry
// the rest of the elementwise work here. Measured on a B200 (16x1024, 12
// heads, both kernels): 2 of every 4 on the FMA pipe (exp2_fma) 0.268 ms, 1 of
// 4 0.259 ms, none 0.2525 ms.
template <bool MASK>
__device__ __forceinline__ void ew_kv(uint32_t (&sv)[NC], uint32_t (&dv)[NC], const float* lse_s,
                                      float sl2, int c0, int Tq, bool row_in, int causal, int min_q) {
  const float4* lse4 = reinterpret_cast<const float4*>(lse_s);
  const float4* dl4 = reinterpret_cast<const float4*>(lse_s + SB);
#pragma unroll
  for (int q = 0; q < NC / 4; ++q) {
    const float4 l = lse4[q], d = dl4[q];
    const float la[4] = {l.x, l.y, l.z, l.w}, da[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int ii = q * 4 + u;
      const float e = fmaf(__uint_as_float(sv[ii]), sl2, -la[u]);
      float pr = ex2f(e);
      if (MASK) {
        const int col = c0 + ii;
        const bool vis = col < Tq && row_in && (!causal || col >= min_q);
        pr = vis ? pr : 0.f;
      }
      sv[ii] = __float_as_uint(pr);
      dv[ii] = __float_as_uint(pr * (__uint_as_float(dv[ii]) - da[u]));
    }
  }
}

// Elementwise step of MODE_Q for one thread's NC columns (keys c0..):
// dP -> dS in place.
template <bool MASK>
__device__ __forceinline__ void ew_q(const uint32_t (&sv)[NC], uint32_t (&dv)[NC], float lse,
                                     float delta, float sl2, int c0, int Tk, bool row_in, int causal,
                                     int abs_row) {
#pragma unroll
  for (int ii = 0; ii < NC; ++ii) {
    const float e = fmaf(__uint_as_float(sv[ii]), sl2, -lse);
    float pr = ex2f(e);
    if (MASK) {
      const int col = c0 + ii;
      const bool vis = col < Tk && row_in && (!causal || col <= abs_row);
      pr = vis ? pr : 0.f;
    }
    dv[ii] = __float_as_uint(pr * (__uint_as_float(dv[ii]) - delta));
  }
}

// KV = KvPeerMaps (context parallelism, streaming): the key/value operand --
// stationary in MODE_KV (tmA / tmA2), streamed in MODE_Q (tmX / tmY) -- is
// loaded through its owner's maps instead.
template <int MODE, class KV>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                       const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmY,
                       const BwdParams p, const __grid_constant__ KV kv) {
  // MODE_KV: A = K, A2 = V (stationary); X = Q, Y = dO (streaming)
  // MODE_Q : A = Q, A2 = dO (stationary); X = K, Y = V (streaming)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* a_full = bars;                 // stationary tiles landed
  uint64_t* a_empty = bars + 1;            // last S/dP MMA of the tile done
  uint64_t* x_full = bars + 2;             // [STAGES]
  uint64_t* x_empty = x_full + STAGES;     // [STAGES]
  uint64_t* s_full = x_empty + STAGES;     // [2] S/dP of a step in TMEM
  uint64_t* s_free = s_full + 2;           // [2] S/dP of a step read out of TMEM (kEwThreads arrivals)
  uint64_t* e_full = s_free + 2;           // [2] P/dS in smem, S/dP consumed (kEwThreads arrivals)
  uint64_t* pds_free = e_full + 2;         // [2] accumulating MMAs done with P/dS
  uint64_t* acc_full = pds_free + 2;       // [2] tile accumulators final
  uint64_t* acc_empty = acc_full + 2;      // [2] accumulators drained (kEwThreads arrivals)
  uint64_t* drain = acc_empty + 2;         // abort path: issued MMAs retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* ld_smem = reinterpret_cast<float*>(smem + LD_OFF);  // [STAGES][2][SB]

  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kEwThreads);
      mbar_init(&e_full[i], kEwThreads);
      mbar_init(&pds_free[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEwThreads);
    }
    mbar_init(drain, 1);
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
  // TMEM columns: S/dP buffer i at [128 i, 128 i + 128) (S then dP, 64 each);
  // accumulator set j at 256 + 128 j: acc1 (+0, 64 cols), acc2 (+64, 64 cols).
  constexpr uint32_t T_ACC = 256;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const int lane = (int)lane_id();
    uint32_t g = 0, i = 0, a_issued = 0;
    uint32_t owners_seen = 0;  // streaming: owners whose publish flag lane 0 saw
    bool ok = true;
    for (int t = blockIdx.x; t < p.n_tiles && ok; t += gridDim.x) {
      const TileInfo ti = tile_info<MODE>(p, t);
      if (ti.n == 0) continue;
      const int b = ti.bh / p.H, h = ti.bh % p.H;
      if (!mbar_wait_bounded(a_empty, (i & 1) ^ 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
        ok = false;
        break;
      }
      if constexpr (KvStreaming<KV>::on && MODE == MODE_KV) {
        int ready = 1, q = 0, row = 0;
        if (lane == 0) {
          q = kv_owner_row(kv, ti.r0, &row);
          ready = kv_owner_ready(kv, q, &owners_seen, p.err, abort_flag);
        }
        if (!__shfl_sync(0xffffffffu, ready, 0)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(a_full, 2 * ATILE);
          tma_load_4d(smem + SA_OFF, &kv.k[q], a_full, 0, h, row, b);
          tma_load_4d(smem + SA2_OFF, &kv.v[q], a_full, 0, h, row, b);
        }
      } else {
        if (lane == 0) {
          mbar_arrive_expect_tx(a_full, 2 * ATILE);
          tma_load_4d(smem + SA_OFF, &tmA, a_full, 0, h, ti.r0, b);
          tma_load_4d(smem + SA2_OFF, &tmA2, a_full, 0, h, ti.r0, b);
        }
      }
      ++a_issued;
      for (int j = 0; j < ti.n; ++j, ++g) {
        const uint32_t st = g % STAGES;
        if (!mbar_wait_bounded(&x_empty[st], ((g / STAGES) & 1) ^ 1, p.err, ERR_TIMEOUT_ATTN,
                               abort_flag)) {
          ok = false;
          break;
        }
        const int row = ti.s0 + (j % ti.nph) * SB;
        // streaming operand's head: the step's query head (MODE_KV) or the
        // tile's key/value head (MODE_Q)
        const int hx = (MODE == MODE_KV) ? h * p.grp + j / ti.nph : h / p.grp;
        if (MODE == MODE_KV) {
          // stage the step's LSE and delta (queries row .. row+63)
          float* dst = ld_smem + st * 2 * SB;
          const int64_t base = ((int64_t)b * p.Hq + hx) * p.Tq;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int q = row + u * 32 + lane;
            const bool in = q < p.Tq;
            dst[u * 32 + lane] = in ? __ldg(p.lse + base + q) : 0.f;
            dst[SB + u * 32 + lane] = in ? __ldg(p.delta + base + q) : 0.f;
          }
          __syncwarp();
        }
        if constexpr (KvStreaming<KV>::on && MODE == MODE_Q) {
          int ready = 1, q = 0, krow = 0;
          if (lane == 0) {
            q = kv_owner_row(kv, row, &krow);
            ready = kv_owner_ready(kv, q, &owners_seen, p.err, abort_flag);
          }
          if (!__shfl_sync(0xffffffffu, ready, 0)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            mbar_arrive_expect_tx(&x_full[st], 2 * XTILE);
            uint8_t* xs = smem + RING_OFF + st * 2 * XTILE;
            tma_load_4d(xs, &kv.k[q], &x_full[st], 0, hx, krow, b);
            tma_load_4d(xs + XTILE, &kv.v[q], &x_full[st], 0, hx, krow, b);
          }
        } else {
          if (lane == 0) {
            mbar_arrive_expect_tx(&x_full[st], 2 * XTILE);
            uint8_t* xs = smem + RING_OFF + st * 2 * XTILE;
            tma_load_4d(xs, &tmX, &x_full[st], 0, hx, row, b);
            tma_load_4d(xs + XTILE, &tmY, &x_full[st], 0, hx, row, b);
          }
        }
        __syncwarp();
      }
      ++i;
    }
    if (*abort_flag && lane == 0) {
      // Another role gave up: wait (bounded) for this warp's copies still in
      // flight before the CTA's shared memory is released.
      if (a_issued) mbar_wait_bounded(a_full, (a_issued - 1) & 1, p.err, ERR_TIMEOUT_ATTN, nullptr);
      for (uint32_t gg = g > STAGES ? g - STAGES : 0; gg < g; ++gg)
        mbar_wait_bounded(&x_full[gg % STAGES], (gg / STAGES) & 1, p.err, ERR_TIMEOUT_ATTN, nullptr);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t id_ss = umma_idesc_bf16(128, SB, 0, 0);  // K-major x K-major
      constexpr uint32_t id_acc = umma_idesc_bf16(128, 64, 0, 1); // K-major A, MN-major B
      const uint32_t sa = smem_u32(smem + SA_OFF), sa2 = smem_u32(smem + SA2_OFF);
      const uint32_t sp0 = smem_u32(smem + P_OFF), sds0 = smem_u32(smem + DS_OFF);
      const uint32_t ring = smem_u32(smem + RING_OFF);
      uint32_t g = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.n_tiles && ok; t += gridDim.x) {
        const TileInfo ti = tile_info<MODE>(p, t);
        if (ti.n == 0) continue;
        const uint32_t acc_base = tmem + T_ACC + (i & 1) * 128;
        if (!mbar_wait_bounded(a_full, i & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag) ||
            !mbar_wait_bounded(&acc_empty[i & 1], ((i >> 1) & 1) ^ 1, p.err, ERR_TIMEOUT_ATTN,
                               abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // S(^T) = A X^T and dP(^T) = A2 Y^T for global step gg (K = head dim)
        // The TMEM buffer of step gg was last used by step gg-2: wait until the
        // elementwise warps have read it out (not until they finish step gg-2).
        auto issue_sd = [&](uint32_t gg, bool last) -> bool {
          const uint32_t st = gg % STAGES;
          if (!mbar_wait_bounded(&s_free[gg & 1], ((gg >> 1) & 1) ^ 1, p.err, ERR_TIMEOUT_ATTN,
                                 abort_flag) ||
              !mbar_wait_bounded(&x_full[st], (gg / STAGES) & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag))
            return false;
          tc_fence_after();
          const uint32_t sx = ring + st * 2 * XTILE, sy = sx + XTILE;
          const uint32_t tb = tmem + (gg & 1) * 128;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            umma_bf16(tb, umma_desc_sw128(sa + kk * 32, 16, 1024),
                      umma_desc_sw128(sx + kk * 32, 16, 1024), id_ss, kk > 0 ? 1u : 0u);
            umma_bf16(tb + SB, umma_desc_sw128(sa2 + kk * 32, 16, 1024),
                      umma_desc_sw128(sy + kk * 32, 16, 1024), id_ss, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[gg & 1]);
          if (last) umma_commit(a_empty);
          return true;
        };
        ok = issue_sd(g, ti.n == 1);
        if (ok && ti.n > 1) ok = issue_sd(g + 1, ti.n == 2);
        for (int j = 0; j < ti.n && ok; ++j, ++g) {
          const uint32_t pb = g & 1, st = g % STAGES;
          // S/dP of step g+2 go to the tensor core before the accumulation of
          // step g, so they are computed while the elementwise warps work on g.
          if (j + 2 < ti.n && !issue_sd(g + 2, j + 3 == ti.n)) {
            ok = false;
            break;
          }
          if (!mbar_wait_bounded(&e_full[pb], (g >> 1) & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sx = ring + st * 2 * XTILE, sy = sx + XTILE;
          const uint32_t sp = sp0 + pb * ATILE, sds = sds0 + pb * ATILE;
          // accumulate over the streaming dimension (K = 64 rows of the step)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t acc = (j > 0 || ks > 0) ? 1u : 0u;
            if (MODE == MODE_KV) {
              // dV += P^T dO ; dK += dS^T Q
              umma_bf16(acc_base + 64, umma_desc_sw128(sp + ks * 32, 16, 1024),
                        umma_desc_sw128(sy + ks * 2048, 8192, 1024), id_acc, acc);
              umma_bf16(acc_base, umma_desc_sw128(sds + ks * 32, 16, 1024),
                        umma_desc_sw128(sx + ks * 2048, 8192, 1024), id_acc, acc);
            } else {
              // dQ += dS K
              umma_bf16(acc_base, umma_desc_sw128(sds + ks * 32, 16, 1024),
                        umma_desc_sw128(sx + ks * 2048, 8192, 1024), id_acc, acc);
            }
          }
          umma_commit(&pds_free[pb]);
          umma_commit(&x_empty[st]);
        }
        if (!ok) break;
        umma_commit(&acc_full[i & 1]);
        ++i;
      }
      if (*abort_flag) {
        // retire every MMA issued so far before TMEM is released
        umma_commit(drain);
        mbar_wait_bounded(drain, 0, p.err, ERR_TIMEOUT_ATTN, nullptr);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------- elementwise
    // Warp w reads TMEM lane quarter w % 4 (a hardware rule) and column group
    // grp (NC of the step's 64 columns).
    const int ew = warp - 2;
    const int lg = warp & 3;
    const int grp = ew >> 2;
    const int lane = (int)lane_id();
    const int r = lg * 32 + lane;         // row of the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
    uint8_t* ptile0 = smem + P_OFF;
    uint8_t* dstile0 = smem + DS_OFF;
    uint32_t g = 0, i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.n_tiles && ok; t += gridDim.x) {
      const TileInfo ti = tile_info<MODE>(p, t);
      const int b = ti.bh / p.H, h = ti.bh % p.H;
      const int row_pos = ti.r0 + r;      // key (KV) or query (Q) position
      const bool row_in = (MODE == MODE_KV) ? row_pos < p.Tk : row_pos < p.Tq;
      if (ti.n == 0) {
        // no visible partner: the gradient of these rows is zero
        if (row_in) {
          const int nacc = (MODE == MODE_KV) ? 2 : 1;
          for (int a = 0; a < nacc; ++a) {
            __nv_bfloat16* dst = (a == 0) ? p.out1 + (int64_t)b * p.o1_sb + (int64_t)row_pos * p.o1_st +
                                                (int64_t)h * p.o1_sh
                                          : p.out2 + (int64_t)b * p.o2_sb + (int64_t)row_pos * p.o2_st +
                                                (int64_t)h * p.o2_sh;
            dst += grp * NC;
#pragma unroll
            for (int q = 0; q < NC / 8; ++q) reinterpret_cast<uint4*>(dst)[q] = make_uint4(0, 0, 0, 0);
          }
        }
        continue;
      }
      // MODE_Q: per-row LSE / delta
      float row_lse = 0.f, row_delta = 0.f;
      if (MODE == MODE_Q && row_in) {
        row_lse = __ldg(p.lse + (int64_t)ti.bh * p.Tq + row_pos);
        row_delta = __ldg(p.delta + (int64_t)ti.bh * p.Tq + row_pos);
      }
      const int abs_row = (MODE == MODE_Q) ? p.q_offset + row_pos : row_pos;
      // tile rows are the stationary block [r0, r0 + 128)
      const int last_row = ti.r0 + TB - 1;
      const bool rows_full = (MODE == MODE_KV) ? last_row < p.Tk : last_row < p.Tq;
      for (int j = 0; j < ti.n; ++j, ++g) {
        const uint32_t pb = g & 1, st = g % STAGES;
        const int cst = ti.s0 + (j % ti.nph) * SB;    // step columns [cst, cst + 64)
        const int c0 = cst + grp * NC;                // this thread's first column
        bool full;
        if (MODE == MODE_KV)
          full = rows_full && cst + SB <= p.Tq && (!p.causal || p.q_offset + cst >= last_row);
        else
          full = rows_full && cst + SB <= p.Tk && (!p.causal || cst + SB - 1 <= p.q_offset + ti.r0);
        if (!mbar_wait_bounded(&s_full[pb], (g >> 1) & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sv[NC], dv[NC];
        const uint32_t tb = tmem + lane_off + pb * 128 + grp * NC;
        tmem_ld_nc(tb, sv);
        tmem_ld_nc(tb + SB, dv);
        tmem_wait_into(sv, dv);
        // S/dP are in registers: the tensor core may overwrite this buffer
        tc_fence_before();
        mbar_arrive(&s_free[pb]);
        if (MODE == MODE_KV) {
          const float* lse_s = ld_smem + st * 2 * SB + grp * NC;
          if (full)
            ew_kv<false>(sv, dv, lse_s, p.sl2, 0, 0, false, 0, 0);
          else
            ew_kv<true>(sv, dv, lse_s, p.sl2, c0, p.Tq, row_in, p.causal, abs_row - p.q_offset);
        } else {
          if (full)
            ew_q<false>(sv, dv, row_lse, row_delta, p.sl2, 0, 0, false, 0, 0);
          else
            ew_q<true>(sv, dv, row_lse, row_delta, p.sl2, c0, p.Tk, row_in, p.causal, abs_row);
        }
        // P/dS buffer pb is free once the accumulation of step g-2 finished
        if (!mbar_wait_bounded(&pds_free[pb], ((g >> 1) & 1) ^ 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
          ok = false;
          break;
        }
        if (MODE == MODE_KV) put_row(ptile0 + pb * ATILE, r, grp, sv);
        put_row(dstile0 + pb * ATILE, r, grp, dv);
        fence_proxy_async_shared();
        tc_fence_before();
        mbar_arrive(&e_full[pb]);
      }
      if (!ok) break;
      // final accumulators -> global (each warp writes its 32 rows, NC dims)
      if (!mbar_wait_bounded(&acc_full[i & 1], (i >> 1) & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t acc_base = tmem + lane_off + T_ACC + (i & 1) * 128 + grp * NC;
      uint32_t v1[NC], v2[NC];
      tmem_ld_nc(acc_base, v1);
      if (MODE == MODE_KV) tmem_ld_nc(acc_base + 64, v2);
      tmem_wait_into(v1, v2);
      tc_fence_before();
      mbar_arrive(&acc_empty[i & 1]);
      ++i;
      if (row_in) {
        const int nacc = (MODE == MODE_KV) ? 2 : 1;
#pragma unroll
        for (int a = 0; a < nacc; ++a) {
          const uint32_t* v = a == 0 ? v1 : v2;
          const float sc = (a == 0) ? p.scale : 1.f;  // dK / dQ carry the softmax scale
          __nv_bfloat16* dst = (a == 0) ? p.out1 + (int64_t)b * p.o1_sb + (int64_t)row_pos * p.o1_st +
                                              (int64_t)h * p.o1_sh
                                        : p.out2 + (int64_t)b * p.o2_sb + (int64_t)row_pos * p.o2_st +
                                              (int64_t)h * p.o2_sh;
          dst += grp * NC;
#pragma unroll
          for (int q = 0; q < NC / 8; ++q) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[q * 8 + 0]) * sc, __uint_as_float(v[q * 8 + 1]) * sc);
            w.y = pack_bf16x2(__uint_as_float(v[q * 8 + 2]) * sc, __uint_as_float(v[q * 8 + 3]) * sc);
            w.z = pack_bf16x2(__uint_as_float(v[q * 8 + 4]) * sc, __uint_as_float(v[q * 8 + 5]) * sc);
            w.w = pack_bf16x2(__uint_as_float(v[q * 8 + 6]) * sc, __uint_as_float(v[q * 8 + 7]) * sc);
            reinterpret_cast<uint4*>(dst)[q] = w;
          }
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

bool head_map(CUtensorMap* tm, const HeadView& v, int H, int T, int B, int rows) {
  auto enc = attn_get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[4] = {64, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)v.sh * 2, (cuuint64_t)v.st * 2, (cuuint64_t)v.sb * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)rows, 1};
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

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int MODE, class KV>
int launch_mode(const CUtensorMap& a, const CUtensorMap& a2, const CUtensorMap& x,
                const CUtensorMap& y, const BwdParams& p, const KV& kv, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_bwd_tc_kernel<MODE, KV>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
      return -10;
    attr = true;
  }
  const int grid = p.n_tiles < num_sms() ? p.n_tiles : num_sms();
  attn_bwd_tc_kernel<MODE, KV><<<grid, kThreads, SMEM_BYTES, s>>>(a, a2, x, y, p, kv);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

}  // namespace


// Tensor-core backward (after delta has been computed into a.delta): returns
// 1 if it ran, 0 when a layout is not TMA-compatible, negative on failure.
// Streaming launches (a.peers) return -12 instead of 0 when a layout does
// not fit: they have no fallback kernel.
int attn_bwd_tc_launch(const AttnArgs& a, cudaStream_t s) {
  const bool stream = a.peers && a.peers->world > 0;
  const int no_fit = stream ? -12 : 0;
  if (!tma_ok(a.q) || !tma_ok(a.dout) || !out_ok(a.dq) || !out_ok(a.dk) || !out_ok(a.dv))
    return no_fit;
  if (!stream && (!tma_ok(a.k) || !tma_ok(a.v))) return 0;
  if (a.B * a.H <= 0 || a.Tq <= 0 || a.Tk <= 0) return no_fit;
  const int Hkv = a.Hkv > 0 ? a.Hkv : a.H;
  if (Hkv > a.H || a.H % Hkv) return -1;
  CUtensorMap tq_a, tk_a, tv_a, tdo_a, tq_x, tk_x, tv_x, tdo_x;
  if (!head_map(&tq_a, a.q, a.H, a.Tq, a.B, TB) || !head_map(&tdo_a, a.dout, a.H, a.Tq, a.B, TB) ||
      !head_map(&tq_x, a.q, a.H, a.Tq, a.B, SB) || !head_map(&tdo_x, a.dout, a.H, a.Tq, a.B, SB))
    return no_fit;
  // streaming: one set of owner maps per box height (128-row stationary
  // tiles for dK/dV, 64-row streamed blocks for dQ); tk_* / tv_* not read
  KvPeerMaps peers_a{}, peers_x{};
  if (stream) {
    auto enc = attn_get_encode_fn();
    if (a.Tk % TB || !make_kv_peer_maps(&peers_a, *a.peers, Hkv, a.B, TB, enc) ||
        !make_kv_peer_maps(&peers_x, *a.peers, Hkv, a.B, SB, enc))
      return -12;
    tk_a = peers_a.k[0];
    tv_a = peers_a.v[0];
    tk_x = peers_x.k[0];
    tv_x = peers_x.v[0];
  } else if (!head_map(&tk_a, a.k, Hkv, a.Tk, a.B, TB) || !head_map(&tv_a, a.v, Hkv, a.Tk, a.B, TB) ||
             !head_map(&tk_x, a.k, Hkv, a.Tk, a.B, SB) || !head_map(&tv_x, a.v, Hkv, a.Tk, a.B, SB)) {
    return 0;
  }
  BwdParams p;
  // dK / dV tiles are per key/value head; each walks its group's query heads
  p.H = Hkv;
  p.BH = a.B * Hkv;
  p.grp = a.H / Hkv;
  p.Hq = a.H;
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
  p.n_blk = (a.Tk + TB - 1) / TB;
  p.n_tiles = p.n_blk * p.BH;
  int rc = stream ? launch_mode<MODE_KV>(tk_a, tv_a, tq_x, tdo_x, p, peers_a, s)
                  : launch_mode<MODE_KV>(tk_a, tv_a, tq_x, tdo_x, p, NoKvPeers{}, s);
  if (rc) return rc;
  // dQ
  p.out1 = reinterpret_cast<__nv_bfloat16*>(a.dq.base);
  p.o1_sb = a.dq.sb;
  p.o1_st = a.dq.st;
  p.o1_sh = a.dq.sh;
  p.out2 = nullptr;
  // dQ tiles are per query head, streaming their key/value head's blocks
  p.H = a.H;
  p.BH = a.B * a.H;
  p.n_blk = (a.Tq + TB - 1) / TB;
  p.n_tiles = p.n_blk * p.BH;
  rc = stream ? launch_mode<MODE_Q>(tq_a, tdo_a, tk_x, tv_x, p, peers_x, s)
              : launch_mode<MODE_Q>(tq_a, tdo_a, tk_x, tv_x, p, NoKvPeers{}, s);
  return rc ? rc : 1;
}

}  // namespace g2b
