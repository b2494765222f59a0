// Persistent, warp-specialised bf16 GEMM for sm_100a on the 5th-generation
// tensor cores (tcgen05.mma, fp32 accumulator in TMEM), fed by TMA.
//
//   C[M,N] = A[M,K] . B[N,K]^T   (A and B each K-major or MN-major)
//
// One CTA per SM (persistent), 320 threads. Tiles are scheduled dynamically:
// CTA b starts with tile b and then takes the next unclaimed tile from a
// global counter, so a CTA that starts late (its SM held by a communication
// kernel running alongside) simply processes fewer tiles. The producer warp
// claims tiles and hands their indices to the MMA and epilogue warps through
// a 4-deep shared-memory queue guarded by mbarriers.
//   warp 0      TMA producer: one elected lane streams A/B k-blocks into a
//               STAGES-deep ring of 128B-swizzled shared-memory stages.
//   warp 1      MMA issuer: allocates TMEM, one elected lane issues
//               tcgen05.mma 128xBNx16 per 16-wide k slice and commits each
//               stage back to the producer; the accumulator is double buffered
//               in TMEM (2 x BN fp32 columns) so tile i+1's MMAs overlap tile
//               i's epilogue.
//   warps 2..9  epilogue: two warps per TMEM lane quarter (tcgen05.ld lets warp
//               w read lanes 32*(w%4)..+31), each owning half the tile's
//               columns. A warp turns 32 accumulator columns of its 32 rows at
//               a time into the fused epilogue result (bias, GELU, GELU
//               backward, fp32 residual add, split-K partial), writes them into
//               a swizzled shared-memory box and issues one TMA bulk tensor
//               store for the box, so global writes are full-line bulk copies.
//               Operands the epilogue reads (residual stream, GELU input) are
//               prefetched into registers one chunk ahead.
//
// The GEMMs of GPT-2 (reference: src/transformer_internals/model.py:201-203
// c_attn, :318-319 c_proj, :333-334 c_fc/c_proj, :474-480 lm_head) all map on
// this kernel: forward (both operands K-major), data gradient (B MN-major) and
// weight gradient (both MN-major, split-K over the token dimension).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "gemm.cuh"

namespace g2b {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kStageBuf = 4096;  // per epilogue warp: one 32x32 fp32 box / two bf16 boxes

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // double-buffered accumulator
  static constexpr int EPI_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFFSET = EPI_OFFSET + kEpiWarps * kStageBuf;
  static constexpr int SMEM_BYTES = BAR_OFFSET + 256 + 1024 /*alignment slack*/;
};

struct GemmDev {
  int M, N, K;
  int m_tiles, n_tiles, splits, kb_per_split, kb_total;
  void* out;
  int64_t ldo;
  void* aux;
  int64_t ldaux;
  const __nv_bfloat16* bias;
  const float* alpha_ptr;
  float alpha;
  int accumulate;
  int64_t split_stride;
  int vec_ok;
  uint32_t* err;
  int* sched;  // {next tile - gridDim.x, finished CTAs}: dynamic scheduling, or null
  float2* ce_stats;
  const int64_t* ce_targets;
  float* ce_tgt_logit;
  int ce_vocab_offset;
  void* const* owner_out;
  int owner_rows;
  int owner_self;
  int m_fast;  // tile order: 1 = consecutive tiles walk M (wide-N GEMMs), 0 = walk N
};

// Row and column tile of linear tile `rem` (within one split). With more N
// tiles than M tiles (the lm_head: 197 x 64), walking M first keeps the few
// B tiles in flight and all of A in L2, so each operand streams from HBM once;
// otherwise walking N first does the same for A.
__device__ __forceinline__ void tile_mn(const GemmDev& p, int rem, int m_tiles, int& mi, int& ni) {
  if (p.m_fast) {
    mi = rem % m_tiles;
    ni = rem / m_tiles;
  } else {
    mi = rem / p.n_tiles;
    ni = rem % p.n_tiles;
  }
}

// Online (max, sum exp) of one epilogue thread's row over its chunks of one
// tile (EPI_CE_STATS): the logits are rounded to bf16 first, as stored.
struct CeRow {
  float m, s;
  int64_t tgt;  // target column relative to this launch's column 0, or -1
};

__device__ __forceinline__ void ce_begin(const GemmDev& p, int row, CeRow& st) {
  st.m = -INFINITY;
  st.s = 0.f;
  st.tgt = -1;
  if (row < p.M) {
    const int64_t t = p.ce_targets[row];
    st.tgt = t < 0 ? -1 : t - p.ce_vocab_offset;
  }
}

__device__ __forceinline__ void ce_chunk(const GemmDev& p, int row, int n0, float* v, CeRow& st) {
  float cm = -INFINITY;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = __bfloat162float(__float2bfloat16_rn(v[i]));
    if (n0 + i < p.N) cm = fmaxf(cm, v[i]);
  }
  if (cm != -INFINITY) {
    const float nm = fmaxf(st.m, cm);
    float acc = st.s * __expf(st.m - nm);
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (n0 + i < p.N) acc += __expf(v[i] - nm);
    st.m = nm;
    st.s = acc;
  }
  if (st.tgt >= n0 && st.tgt < n0 + 32 && st.tgt < p.N && row < p.M) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (n0 + i == st.tgt) t = v[i];
    p.ce_tgt_logit[row] = t;
  }
}

__device__ __forceinline__ void ce_end(const GemmDev& p, int row, int slot, const CeRow& st) {
  if (row < p.M) p.ce_stats[(int64_t)slot * p.M + row] = make_float2(st.m, st.s);
}

// Per-launch tile counters for dynamic scheduling (see gemm_tcgen05_kernel).
// Launches take slots round-robin; the last CTA of a launch resets its slot,
// so a slot is zero again long before it is handed out anew.
constexpr int kSchedSlots = 64;
__device__ int g_gemm_sched[kSchedSlots * 2];

// ---------------------------------------------------------------- TMA store
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* smem_src, int32_t x,
                                             int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tmap)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;"); }
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Per-chunk operand the epilogue reads besides the accumulator (prefetched).
struct EpiIn {
  float f[32];  // fp32 residual source / old fp32 output, or unpacked GELU input
};

template <int EPI>
__device__ __forceinline__ void load_epi_in(const GemmDev& p, int row, int n0, EpiIn& in) {
  const bool rd_f32 = (EPI == EPI_RESID_F32) || (EPI == EPI_F32 && p.accumulate);
  const bool rd_bf16 = (EPI == EPI_GELU_BWD);
  if (!rd_f32 && !rd_bf16) return;
  if (row >= p.M || n0 >= p.N) {
#pragma unroll
    for (int i = 0; i < 32; ++i) in.f[i] = 0.f;
    return;
  }
  const bool full = (n0 + 32 <= p.N) && p.vec_ok;
  if (rd_f32) {
    const float* src = (EPI == EPI_RESID_F32 && p.aux != nullptr)
                           ? reinterpret_cast<const float*>(p.aux) + (int64_t)row * p.ldaux + n0
                           : reinterpret_cast<const float*>(p.out) + (int64_t)row * p.ldo + n0;
    if (full) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 w = __ldcs(reinterpret_cast<const float4*>(src) + q);
        in.f[4 * q] = w.x;
        in.f[4 * q + 1] = w.y;
        in.f[4 * q + 2] = w.z;
        in.f[4 * q + 3] = w.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) in.f[i] = (n0 + i < p.N) ? src[i] : 0.f;
    }
  } else {
    const __nv_bfloat16* a =
        reinterpret_cast<const __nv_bfloat16*>(p.aux) + (int64_t)row * p.ldaux + n0;
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 u = __ldcs(reinterpret_cast<const uint4*>(a) + q);
        const uint32_t us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(us[j]);
          in.f[q * 8 + 2 * j] = f.x;
          in.f[q * 8 + 2 * j + 1] = f.y;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) in.f[i] = (n0 + i < p.N) ? __bfloat162float(a[i]) : 0.f;
    }
  }
}

// Turns the scaled accumulator chunk v[32] into the epilogue result(s):
// v (main output) and z (second output: GELU pre-activation).
template <int EPI>
__device__ __forceinline__ void epi_math(const GemmDev& p, int n0, float* v, const EpiIn& in,
                                         float* z) {
  if (EPI == EPI_BF16 || EPI == EPI_BIAS_GELU || EPI == EPI_RESID_F32) {
    if (p.bias != nullptr) {
      if (n0 + 32 <= p.N && p.vec_ok) {
        const uint4* bp = reinterpret_cast<const uint4*>(p.bias + n0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 w = __ldg(bp + q);
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = unpack_bf16x2(ws[j]);
            v[q * 8 + 2 * j] += f.x;
            v[q * 8 + 2 * j + 1] += f.y;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n0 + i < p.N) v[i] += __bfloat162float(p.bias[n0 + i]);
      }
    }
  }
  if (EPI == EPI_BIAS_GELU) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      z[i] = v[i];
      v[i] = gelu_tanh_f(v[i]);
    }
  } else if (EPI == EPI_GELU_BWD) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= gelu_tanh_grad_f(in.f[i]);
  } else if (EPI == EPI_RESID_F32 || (EPI == EPI_F32 && p.accumulate)) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += in.f[i];
  }
}

// Write one thread's 32 results into its row of a swizzled staging box:
// bf16 rows are 64 B (SWIZZLE_64B: 16-byte chunk ^= (row/2)%4), fp32 rows
// 128 B (SWIZZLE_128B: chunk ^= row%8), matching the output tensor maps.
__device__ __forceinline__ void stage_bf16(uint8_t* box, int r, const float* y) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack_bf16x2(y[q * 8 + 0], y[q * 8 + 1]);
    w.y = pack_bf16x2(y[q * 8 + 2], y[q * 8 + 3]);
    w.z = pack_bf16x2(y[q * 8 + 4], y[q * 8 + 5]);
    w.w = pack_bf16x2(y[q * 8 + 6], y[q * 8 + 7]);
    *reinterpret_cast<uint4*>(box + r * 64 + ((q ^ ((r >> 1) & 3)) << 4)) = w;
  }
}
__device__ __forceinline__ void stage_f32(uint8_t* box, int r, const float* y) {
#pragma unroll
  for (int q = 0; q < 8; ++q)
    *reinterpret_cast<float4*>(box + r * 128 + ((q ^ (r & 7)) << 4)) =
        make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
}

// Direct (non-TMA) store of one thread's row chunk, for unaligned outputs.
template <int EPI>
__device__ __forceinline__ void store_direct(const GemmDev& p, int row, int n0, const float* y,
                                             const float* z, int split) {
  if (row >= p.M || n0 >= p.N) return;
  const bool full = (n0 + 32 <= p.N) && p.vec_ok;
  if (EPI == EPI_RESID_F32 || EPI == EPI_F32) {
    float* o = reinterpret_cast<float*>(p.out) + (int64_t)split * p.split_stride +
               (int64_t)row * p.ldo + n0;
    if (full) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4*>(o)[q] = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
    } else {
      for (int i = 0; i < 32 && n0 + i < p.N; ++i) o[i] = y[i];
    }
  } else {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)row * p.ldo + n0;
    if (p.owner_out) {
      const int q = row / p.owner_rows;
      o = reinterpret_cast<__nv_bfloat16*>(p.owner_out[q]) +
          (int64_t)(row - q * p.owner_rows) * p.ldo + n0;
    }
    __nv_bfloat16* a = EPI == EPI_BIAS_GELU
                           ? reinterpret_cast<__nv_bfloat16*>(p.aux) + (int64_t)row * p.ldaux + n0
                           : nullptr;
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16x2(y[q * 8 + 0], y[q * 8 + 1]);
        w.y = pack_bf16x2(y[q * 8 + 2], y[q * 8 + 3]);
        w.z = pack_bf16x2(y[q * 8 + 4], y[q * 8 + 5]);
        w.w = pack_bf16x2(y[q * 8 + 6], y[q * 8 + 7]);
        reinterpret_cast<uint4*>(o)[q] = w;
        if (EPI == EPI_BIAS_GELU) {
          uint4 u;
          u.x = pack_bf16x2(z[q * 8 + 0], z[q * 8 + 1]);
          u.y = pack_bf16x2(z[q * 8 + 2], z[q * 8 + 3]);
          u.z = pack_bf16x2(z[q * 8 + 4], z[q * 8 + 5]);
          u.w = pack_bf16x2(z[q * 8 + 6], z[q * 8 + 7]);
          reinterpret_cast<uint4*>(a)[q] = u;
        }
      }
    } else {
      for (int i = 0; i < 32 && n0 + i < p.N; ++i) {
        o[i] = __float2bfloat16(y[i]);
        if (EPI == EPI_BIAS_GELU) a[i] = __float2bfloat16(z[i]);
      }
    }
  }
}

template <int BN, int EPI, int A_MN, int B_MN, int TMA_ST>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmO,
                        const __grid_constant__ CUtensorMap tmX, const GemmDev p) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr bool F32_OUT = (EPI == EPI_RESID_F32 || EPI == EPI_F32);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFFSET);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* tq_full = tempty_bar + 2;   // [4] tile index written
  uint64_t* tq_empty = tq_full + 4;      // [4] tile index read by MMA + epilogue
  int* tile_q = reinterpret_cast<int*>(tq_empty + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_q + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int tiles_per_split = p.m_tiles * p.n_tiles;
  const int num_tiles = tiles_per_split * p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 32 * kEpiWarps);
    }
    for (int q = 0; q < 4; ++q) {
      mbar_init(&tq_full[q], 1);
      mbar_init(&tq_empty[q], 1 + 32 * kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane_id() == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (TMA_ST) {
      tma_prefetch_desc(&tmO);
      if (EPI == EPI_BIAS_GELU) tma_prefetch_desc(&tmX);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int tile = blockIdx.x;
      for (int r = 0; ok; ++r) {
        // publish this tile (or the end marker) to the MMA and epilogue warps
        const int slot = r & 3;
        if (!mbar_wait_bounded(&tq_empty[slot], ((r >> 2) & 1) ^ 1, p.err, ERR_TIMEOUT_PRODUCER,
                               abort_flag))
          break;
        tile_q[slot] = tile < num_tiles ? tile : -1;
        mbar_arrive(&tq_full[slot]);
        if (tile >= num_tiles) break;
        const int cur = tile;
        tile = p.sched ? (int)gridDim.x + atomicAdd(p.sched, 1) : tile + (int)gridDim.x;
        const int split = cur / tiles_per_split;
        const int rem = cur % tiles_per_split;
        int mi, ni;
        tile_mn(p, rem, p.m_tiles, mi, ni);
        const int m0 = mi * BM;
        const int n0 = ni * BN;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1, p.err, ERR_TIMEOUT_PRODUCER,
                                 abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          const int k0 = kb * BK;
          if (A_MN) {
            tma_load_2d(sa, &tmA, &full_bar[stage], m0, k0);
            tma_load_2d(sa + 64 * BK * 2, &tmA, &full_bar[stage], m0 + 64, k0);
          } else {
            tma_load_2d(sa, &tmA, &full_bar[stage], k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_2d(sb + c * 64 * BK * 2, &tmB, &full_bar[stage], n0 + c * 64, k0);
          } else {
            tma_load_2d(sb, &tmB, &full_bar[stage], k0, n0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int slot = r & 3;
        if (!mbar_wait_bounded(&tq_full[slot], (r >> 2) & 1, p.err, ERR_TIMEOUT_MMA, abort_flag))
          break;
        const int tile = tile_q[slot];
        mbar_arrive(&tq_empty[slot]);
        if (tile < 0) break;
        const int split = tile / tiles_per_split;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1, p.err, ERR_TIMEOUT_MMA,
                               abort_flag))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, p.err, ERR_TIMEOUT_MMA, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // K-major: advance 16 elements = 32 bytes inside the swizzle row.
            // MN-major: advance 16 k-rows of 128 bytes.
            const uint64_t ad = A_MN ? umma_desc_sw128(sa + kk * 2048, 64 * BK * 2, 1024)
                                     : umma_desc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? umma_desc_sw128(sb + kk * 2048, 64 * BK * 2, 1024)
                                     : umma_desc_sw128(sb + kk * 32, 16, 1024);
            umma_bf16(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------- epilogue
    const int ew = warp - 2;              // 0..7
    const int lg = warp & 3;              // TMEM lane quarter this warp may read
    const int col_half = ew >> 2;         // which half of the tile's columns
    const int lane = (int)lane_id();
    const int r_local = lg * 32 + lane;   // row within the tile
    constexpr int CHUNKS = BN / 64;       // 32-column chunks per warp
    // two bf16 boxes per warp (the cross-entropy statistics epilogue keeps
    // one: measured 1.37 ms with one, 1.57 ms with two, on different machines)
    constexpr bool kDblBox = !F32_OUT && EPI != EPI_BIAS_GELU && EPI != EPI_CE_STATS;
    uint8_t* box = smem + Cfg::EPI_OFFSET + ew * kStageBuf;
    int acc = 0;
    uint32_t acc_phase = 0;
    float alpha = p.alpha;
    if (p.alpha_ptr) alpha *= *p.alpha_ptr;
    EpiIn in_next;
    for (int r = 0;; ++r) {
      const int slot = r & 3;
      if (!mbar_wait_bounded(&tq_full[slot], (r >> 2) & 1, p.err, ERR_TIMEOUT_EPILOGUE, abort_flag))
        break;
      const int tile = tile_q[slot];
      mbar_arrive(&tq_empty[slot]);
      if (tile < 0) break;
      const int split = tile / tiles_per_split;
      const int rem = tile % tiles_per_split;
      int mi, ni;
      tile_mn(p, rem, p.m_tiles, mi, ni);
      const int m0 = mi * BM;
      const int n0 = ni * BN;
      const int row = m0 + r_local;
      const int c0 = n0 + col_half * (BN / 2);
      load_epi_in<EPI>(p, row, c0, in_next);
      CeRow ce;
      if (EPI == EPI_CE_STATS) ce_begin(p, row, ce);
      // row-owner output: a tile owned by another GPU goes out by direct stores
      const bool peer_tile = p.owner_out && (m0 / p.owner_rows) != p.owner_self;
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, p.err, ERR_TIMEOUT_EPILOGUE, abort_flag))
        break;
      tc_fence_after();
      const uint32_t t_row =
          tmem_base + ((uint32_t)(lg * 32) << 16) + acc * BN + col_half * (BN / 2);
#pragma unroll 1
      for (int c = 0; c < CHUNKS; ++c) {
        float v[32], z[32];
        tmem_ld32(t_row + c * 32, v);
        tmem_wait_ld();
        if (c == CHUNKS - 1) {
          tc_fence_before();
          mbar_arrive(&tempty_bar[acc]);
        }
        EpiIn in = in_next;
        if (c + 1 < CHUNKS) load_epi_in<EPI>(p, row, c0 + (c + 1) * 32, in_next);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= alpha;
        epi_math<EPI>(p, c0 + c * 32, v, in, z);
        if (EPI == EPI_CE_STATS) ce_chunk(p, row, c0 + c * 32, v, ce);
        if (TMA_ST && !peer_tile) {
          // A bf16 box (2 KB) is half the warp's staging buffer: alternate
          // halves, so only the store of two chunks ago must have finished
          // reading its box; an fp32 box (or GELU's output + input pair)
          // fills it and waits for the previous chunk's store.
          uint8_t* bx = kDblBox ? box + (c & 1) * 2048 : box;
          if (lane == 0) {
            if (kDblBox) bulk_wait_read1();
            else bulk_wait_read0();
          }
          __syncwarp();
          if (F32_OUT) {
            stage_f32(bx, lane, v);
          } else {
            stage_bf16(bx, lane, v);
            if (EPI == EPI_BIAS_GELU) stage_bf16(box + 2048, lane, z);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmO, bx, c0 + c * 32, m0 + lg * 32, split);
            if (EPI == EPI_BIAS_GELU) tma_store_3d(&tmX, box + 2048, c0 + c * 32, m0 + lg * 32, 0);
            bulk_commit();
          }
        } else {
          store_direct<EPI>(p, row, c0 + c * 32, v, z, split);
        }
      }
      if (EPI == EPI_CE_STATS) ce_end(p, row, 2 * (n0 / BN) + col_half, ce);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (TMA_ST && lane == 0) bulk_wait0();
    // rows stored into other GPUs' memory are visible before a later signal
    if (p.owner_out) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  if (p.sched && threadIdx.x == 0) {
    // every claim of this CTA precedes this point; the last CTA to get here
    // knows no claim on this slot is outstanding and resets it
    __threadfence();
    if (atomicAdd(p.sched + 1, 1) == (int)gridDim.x - 1) {
      p.sched[0] = 0;
      p.sched[1] = 0;
      __threadfence();
    }
  }
}

// ------------------------------------------------------------- CTA pairs ---
// The same GEMM with one 256x256 output tile per PAIR of CTAs (a cluster of
// two on neighbouring SMs) and one tcgen05.mma.cta_group::2 of M = 256,
// N = 256 per 16-wide k slice. Each CTA loads its own 128 rows of A and its
// own 128 rows of B per k-block (32 KB instead of the 48 KB a 128x256 tile of
// one CTA needs), so the operand bytes streamed from L2 per FLOP fall by a
// third; each CTA's TMEM holds its 128 rows of the accumulator and its
// epilogue is the single-CTA one.
//   leader (cluster rank 0): claims tiles and publishes them to both CTAs'
//     queues; its full barriers count both CTAs' TMA bytes; its MMA warp
//     issues the pair MMAs and commits to the barriers of both CTAs.
//   peer (rank 1): its producer streams its halves into its own stages,
//     signalling the leader's full barrier; its epilogue drains its TMEM and
//     releases the accumulator on the leader's barrier.
// No load is a multicast: every TMA copy writes the issuing CTA's own shared
// memory from this GPU's global memory.
constexpr int kPairStages = 6;
// Launches that pass the shape policy in use_pairs() run on CTA pairs unless
// the caller or G2B_GEMM_PAIR says otherwise.
constexpr bool kPairDefault = true;

struct PairCfg {
  static constexpr int BN = 256;                     // tile N of the pair
  static constexpr int STAGES = kPairStages;
  static constexpr int A_BYTES = BM * BK * 2;        // this CTA's 128 rows of A
  static constexpr int B_BYTES = (BN / 2) * BK * 2;  // this CTA's 128 rows of B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int EPI_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFFSET = EPI_OFFSET + kEpiWarps * kStageBuf;
  static constexpr int SMEM_BYTES = BAR_OFFSET + 256 + 1024;
};
static_assert(PairCfg::SMEM_BYTES <= 232448, "pair GEMM exceeds the shared-memory limit");

// Arrivals a tile-queue slot needs before the leader may reuse it: the
// leader's MMA warp and 8 epilogue warps, the peer's producer and 8 epilogue
// warps.
constexpr int kPairQueueArrivals = 2 + 2 * kEpiWarps;

template <int EPI, int A_MN, int B_MN, int TMA_ST>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmO,
                     const __grid_constant__ CUtensorMap tmX, const GemmDev p) {
  using Cfg = PairCfg;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int BN = Cfg::BN;
  constexpr bool F32_OUT = (EPI == EPI_RESID_F32 || EPI == EPI_F32);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFFSET);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* tq_full = tempty_bar + 2;
  uint64_t* tq_empty = tq_full + 4;
  int* tile_q = reinterpret_cast<int*>(tq_empty + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_q + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = (int)(blockIdx.x >> 1);
  const int npairs = (int)(gridDim.x >> 1);
  const int m_tiles = (p.M + 2 * BM - 1) / (2 * BM);  // 256-row tiles
  const int tiles_per_split = m_tiles * p.n_tiles;
  const int num_tiles = tiles_per_split * p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);   // used on the leader: its arrive.expect_tx
      mbar_init(&empty_bar[s], 1);  // the leader's MMA commit, in both CTAs
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 2 * kEpiWarps);  // leader only: both CTAs' warps
    }
    for (int q = 0; q < 4; ++q) {
      mbar_init(&tq_full[q], 1);
      mbar_init(&tq_empty[q], kPairQueueArrivals);  // leader only
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane_id() == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (TMA_ST) {
      tma_prefetch_desc(&tmO);
      if (EPI == EPI_BIAS_GELU) tma_prefetch_desc(&tmX);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // both CTAs' barriers are initialised before either touches the other's
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int tile = pair;
      const uint32_t lead_full0 = cluster_addr(&full_bar[0], 0);
      for (int r = 0; ok; ++r) {
        const int slot = r & 3;
        int cur;
        if (leader) {
          if (!mbar_wait_bounded(&tq_empty[slot], ((r >> 2) & 1) ^ 1, p.err, ERR_TIMEOUT_PRODUCER,
                                 abort_flag))
            break;
          cur = tile < num_tiles ? tile : -1;
          tile_q[slot] = cur;
          st_cluster_u32(cluster_addr(&tile_q[slot], 1), (uint32_t)cur);
          mbar_arrive(&tq_full[slot]);
          mbar_arrive_cluster(cluster_addr(&tq_full[slot], 1));
          if (cur < 0) break;
          tile = p.sched ? npairs + atomicAdd(p.sched, 1) : tile + npairs;
        } else {
          if (!mbar_wait_bounded_cluster(&tq_full[slot], (r >> 2) & 1, p.err, ERR_TIMEOUT_PRODUCER,
                                         abort_flag))
            break;
          cur = tile_q[slot];
          mbar_arrive_cluster(cluster_addr(&tq_empty[slot], 0));
          if (cur < 0) break;
        }
        const int split = cur / tiles_per_split;
        const int rem = cur % tiles_per_split;
        int mi, ni;
        tile_mn(p, rem, m_tiles, mi, ni);
        const int m0 = mi * 2 * BM + (int)rank * BM;
        const int nb = ni * BN + (int)rank * (BN / 2);
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1, p.err, ERR_TIMEOUT_PRODUCER,
                                 abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          const uint32_t fb = lead_full0 + stage * 8;
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::STAGE_BYTES);
          const int k0 = kb * BK;
          if (A_MN) {
            tma_load_2d_pair(sa, &tmA, fb, m0, k0);
            tma_load_2d_pair(sa + 64 * BK * 2, &tmA, fb, m0 + 64, k0);
          } else {
            tma_load_2d_pair(sa, &tmA, fb, k0, m0);
          }
          if (B_MN) {
            tma_load_2d_pair(sb, &tmB, fb, nb, k0);
            tma_load_2d_pair(sb + 64 * BK * 2, &tmB, fb, nb + 64, k0);
          } else {
            tma_load_2d_pair(sb, &tmB, fb, k0, nb);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (leader)
    if (leader && elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(2 * BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int slot = r & 3;
        if (!mbar_wait_bounded(&tq_full[slot], (r >> 2) & 1, p.err, ERR_TIMEOUT_MMA, abort_flag))
          break;
        const int tile = tile_q[slot];
        mbar_arrive(&tq_empty[slot]);
        if (tile < 0) break;
        const int split = tile / tiles_per_split;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1, p.err, ERR_TIMEOUT_MMA,
                               abort_flag))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, p.err, ERR_TIMEOUT_MMA, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? umma_desc_sw128(sa + kk * 2048, 64 * BK * 2, 1024)
                                     : umma_desc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? umma_desc_sw128(sb + kk * 2048, 64 * BK * 2, 1024)
                                     : umma_desc_sw128(sb + kk * 32, 16, 1024);
            umma_bf16_pair(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          // the stage is free in both CTAs once these MMAs have read it
          umma_commit_pair_mask(&empty_bar[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair_mask(&tfull_bar[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------- epilogue
    const int ew = warp - 2;
    const int lg = warp & 3;
    const int col_half = ew >> 2;
    const int lane = (int)lane_id();
    const int r_local = lg * 32 + lane;
    constexpr int CHUNKS = BN / 64;
    constexpr bool kDblBox = !F32_OUT && EPI != EPI_BIAS_GELU && EPI != EPI_CE_STATS;
    uint8_t* box = smem + Cfg::EPI_OFFSET + ew * kStageBuf;
    const uint32_t lead_tempty0 = cluster_addr(&tempty_bar[0], 0);
    const uint32_t lead_tq_empty0 = cluster_addr(&tq_empty[0], 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    float alpha = p.alpha;
    if (p.alpha_ptr) alpha *= *p.alpha_ptr;
    EpiIn in_next;
    for (int r = 0;; ++r) {
      const int slot = r & 3;
      const bool got = leader ? mbar_wait_bounded(&tq_full[slot], (r >> 2) & 1, p.err,
                                                  ERR_TIMEOUT_EPILOGUE, abort_flag)
                              : mbar_wait_bounded_cluster(&tq_full[slot], (r >> 2) & 1, p.err,
                                                          ERR_TIMEOUT_EPILOGUE, abort_flag);
      if (!got) break;
      const int tile = tile_q[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead_tq_empty0 + slot * 8);
      if (tile < 0) break;
      const int split = tile / tiles_per_split;
      const int rem = tile % tiles_per_split;
      int mi, ni;
      tile_mn(p, rem, m_tiles, mi, ni);
      const int m0 = mi * 2 * BM + (int)rank * BM;
      const int n0 = ni * BN;
      const int row = m0 + r_local;
      const int c0 = n0 + col_half * (BN / 2);
      load_epi_in<EPI>(p, row, c0, in_next);
      CeRow ce;
      if (EPI == EPI_CE_STATS) ce_begin(p, row, ce);
      // row-owner output: a tile owned by another GPU goes out by direct stores
      const bool peer_tile = p.owner_out && (m0 / p.owner_rows) != p.owner_self;
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, p.err, ERR_TIMEOUT_EPILOGUE, abort_flag))
        break;
      tc_fence_after();
      const uint32_t t_row =
          tmem_base + ((uint32_t)(lg * 32) << 16) + acc * BN + col_half * (BN / 2);
#pragma unroll 1
      for (int c = 0; c < CHUNKS; ++c) {
        float v[32], z[32];
        tmem_ld32(t_row + c * 32, v);
        tmem_wait_ld();
        if (c == CHUNKS - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(lead_tempty0 + acc * 8);
        }
        EpiIn in = in_next;
        if (c + 1 < CHUNKS) load_epi_in<EPI>(p, row, c0 + (c + 1) * 32, in_next);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= alpha;
        epi_math<EPI>(p, c0 + c * 32, v, in, z);
        if (EPI == EPI_CE_STATS) ce_chunk(p, row, c0 + c * 32, v, ce);
        if (TMA_ST && !peer_tile) {
          uint8_t* bx = kDblBox ? box + (c & 1) * 2048 : box;  // as in the single-CTA kernel
          if (lane == 0) {
            if (kDblBox) bulk_wait_read1();
            else bulk_wait_read0();
          }
          __syncwarp();
          if (F32_OUT) {
            stage_f32(bx, lane, v);
          } else {
            stage_bf16(bx, lane, v);
            if (EPI == EPI_BIAS_GELU) stage_bf16(box + 2048, lane, z);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmO, bx, c0 + c * 32, m0 + lg * 32, split);
            if (EPI == EPI_BIAS_GELU) tma_store_3d(&tmX, box + 2048, c0 + c * 32, m0 + lg * 32, 0);
            bulk_commit();
          }
        } else {
          store_direct<EPI>(p, row, c0 + c * 32, v, z, split);
        }
      }
      if (EPI == EPI_CE_STATS) ce_end(p, row, 2 * (n0 / BN) + col_half, ce);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (TMA_ST && lane == 0) bulk_wait0();
    // rows stored into other GPUs' memory are visible before a later signal
    if (p.owner_out) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  // neither CTA leaves while the other may still signal its barriers or the
  // leader's MMAs may still read its shared memory
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
  if (leader && p.sched && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.sched + 1, 1) == npairs - 1) {
      p.sched[0] = 0;
      p.sched[1] = 0;
      __threadfence();
    }
  }
}

// ------------------------------------------------------------------ host ---
// Device address of a scheduling slot (the symbol's address on the current
// device, looked up once per device).
int* gemm_sched_slot() {
  static int* base[64] = {nullptr};
  static std::atomic<unsigned> seq{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!base[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_gemm_sched) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;  // static scheduling
    }
    base[dev] = static_cast<int*>(ptr);
  }
  return base[dev] + 2 * (seq.fetch_add(1, std::memory_order_relaxed) % kSchedSlots);
}
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
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

// 2-D bf16 operand map: inner extent `inner` (contiguous), outer extent `outer`
// with row stride `ld` elements; box = 64 (inner, 128 B) x box_outer; 128B swizzle.
bool make_tmap_2d(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t outer, int64_t ld,
                  uint32_t box_outer) {
  auto enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D output map {N, M, S} (row stride ld, S slabs of M rows), 32x32x1 boxes,
// swizzle 64B for bf16 / 128B for fp32 (one box row = the swizzle span).
bool make_tmap_out(CUtensorMap* tm, const void* base, uint64_t N, uint64_t M, uint64_t S,
                   int64_t ld, int esize) {
  auto enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {N, M, S};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * esize,
                           static_cast<cuuint64_t>(ld) * esize * M};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(tm, esize == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   esize == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

struct Maps {
  CUtensorMap a, b, o, x;
};

template <int BN, int EPI, int A_MN, int B_MN, int TMA_ST>
int launch_cfg(const Maps& m, const GemmDev& d, int grid, cudaStream_t s) {
  auto kern = gemm_tcgen05_kernel<BN, EPI, A_MN, B_MN, TMA_ST>;
  constexpr int smem = GemmCfg<BN>::SMEM_BYTES;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return -10;
    attr_set = true;
  }
  kern<<<grid, kThreads, smem, s>>>(m.a, m.b, m.o, m.x, d);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

template <int BN, int EPI, int TMA_ST>
int dispatch_major(int amn, int bmn, const Maps& m, const GemmDev& d, int grid, cudaStream_t s) {
  if (!amn && !bmn) return launch_cfg<BN, EPI, 0, 0, TMA_ST>(m, d, grid, s);
  if (!amn && bmn) return launch_cfg<BN, EPI, 0, 1, TMA_ST>(m, d, grid, s);
  if (amn && bmn) return launch_cfg<BN, EPI, 1, 1, TMA_ST>(m, d, grid, s);
  return launch_cfg<BN, EPI, 1, 0, TMA_ST>(m, d, grid, s);
}

template <int BN, int EPI>
int dispatch_st(int tma_st, int amn, int bmn, const Maps& m, const GemmDev& d, int grid,
                cudaStream_t s) {
  return tma_st ? dispatch_major<BN, EPI, 1>(amn, bmn, m, d, grid, s)
                : dispatch_major<BN, EPI, 0>(amn, bmn, m, d, grid, s);
}

template <int BN>
int dispatch_epi(int epi, int tma_st, int amn, int bmn, const Maps& m, const GemmDev& d, int grid,
                 cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: return dispatch_st<BN, EPI_BF16>(tma_st, amn, bmn, m, d, grid, s);
    case EPI_BIAS_GELU: return dispatch_st<BN, EPI_BIAS_GELU>(tma_st, amn, bmn, m, d, grid, s);
    case EPI_RESID_F32: return dispatch_st<BN, EPI_RESID_F32>(tma_st, amn, bmn, m, d, grid, s);
    case EPI_F32: return dispatch_st<BN, EPI_F32>(tma_st, amn, bmn, m, d, grid, s);
    case EPI_GELU_BWD: return dispatch_st<BN, EPI_GELU_BWD>(tma_st, amn, bmn, m, d, grid, s);
    case EPI_CE_STATS: return dispatch_st<BN, EPI_CE_STATS>(tma_st, amn, bmn, m, d, grid, s);
  }
  return -3;
}

// Largest number of CTA pairs of the pair kernel that can be resident at
// once (a pair needs two free SMs of one GPC), looked up once per
// instantiation; falls back to half the SMs.
template <typename K>
int max_pairs(K kern, int smem) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (num_sms() / 2), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (void*)kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = num_sms() / 2;
  }
  return std::min(n, num_sms() / 2);
}

template <int EPI, int A_MN, int B_MN, int TMA_ST>
int launch_pair_cfg(const Maps& m, GemmDev d, int tiles, int max_ctas, cudaStream_t s) {
  auto kern = gemm_pair_kernel<EPI, A_MN, B_MN, TMA_ST>;
  constexpr int smem = PairCfg::SMEM_BYTES;
  static int pairs_cap = 0;
  if (!pairs_cap) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return -10;
    pairs_cap = max_pairs(kern, smem);
  }
  int pairs = pairs_cap;
  if (max_ctas > 0) pairs = std::max(1, std::min(pairs, max_ctas / 2));
  if (pairs > tiles) pairs = tiles;
  d.sched = tiles > pairs ? gemm_sched_slot() : nullptr;
  kern<<<2 * pairs, kThreads, smem, s>>>(m.a, m.b, m.o, m.x, d);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

template <int EPI, int TMA_ST>
int pair_major(int amn, int bmn, const Maps& m, const GemmDev& d, int tiles, int max_ctas,
               cudaStream_t s) {
  if (!amn && !bmn) return launch_pair_cfg<EPI, 0, 0, TMA_ST>(m, d, tiles, max_ctas, s);
  if (!amn && bmn) return launch_pair_cfg<EPI, 0, 1, TMA_ST>(m, d, tiles, max_ctas, s);
  if (amn && bmn) return launch_pair_cfg<EPI, 1, 1, TMA_ST>(m, d, tiles, max_ctas, s);
  return launch_pair_cfg<EPI, 1, 0, TMA_ST>(m, d, tiles, max_ctas, s);
}

template <int EPI>
int pair_st(int tma_st, int amn, int bmn, const Maps& m, const GemmDev& d, int tiles,
            int max_ctas, cudaStream_t s) {
  return tma_st ? pair_major<EPI, 1>(amn, bmn, m, d, tiles, max_ctas, s)
                : pair_major<EPI, 0>(amn, bmn, m, d, tiles, max_ctas, s);
}

int pair_epi(int epi, int tma_st, int amn, int bmn, const Maps& m, const GemmDev& d, int tiles,
             int max_ctas, cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: return pair_st<EPI_BF16>(tma_st, amn, bmn, m, d, tiles, max_ctas, s);
    case EPI_BIAS_GELU: return pair_st<EPI_BIAS_GELU>(tma_st, amn, bmn, m, d, tiles, max_ctas, s);
    case EPI_RESID_F32: return pair_st<EPI_RESID_F32>(tma_st, amn, bmn, m, d, tiles, max_ctas, s);
    case EPI_F32: return pair_st<EPI_F32>(tma_st, amn, bmn, m, d, tiles, max_ctas, s);
    case EPI_GELU_BWD: return pair_st<EPI_GELU_BWD>(tma_st, amn, bmn, m, d, tiles, max_ctas, s);
    case EPI_CE_STATS: return pair_st<EPI_CE_STATS>(tma_st, amn, bmn, m, d, tiles, max_ctas, s);
  }
  return -3;
}

// Whether a launch runs on CTA pairs: the caller's choice (0 / 1), else the
// G2B_GEMM_PAIR environment variable (0 / 1), else the built-in policy.
bool use_pairs(const GemmArgs& a) {
  static int env = -2;
  if (env == -2) {
    const char* e = getenv("G2B_GEMM_PAIR");
    env = (e && (e[0] == '0' || e[0] == '1')) ? e[0] - '0' : -1;
  }
  int want = a.pair >= 0 ? a.pair : env;
  if (a.bn != 256 || a.M < 2 * BM) return false;  // needs a full 256-row pair tile
  if (want >= 0) return want == 1;
  // Measured on B200 at GPT-2 shapes (CUDA events, same box): pairs win where
  // the epilogue is light and operand streaming dominates -- weight
  // gradients (fp32 out), data gradients (B MN-major), the residual-add
  // forward and the wide lm_head GEMMs -- and lose where the GELU epilogues
  // (forward and backward) set the pace, since a pair's accumulator is
  // released only when both CTAs' epilogues have drained it.
  if (a.epilogue == EPI_BIAS_GELU || a.epilogue == EPI_GELU_BWD) return false;
  if (a.epilogue == EPI_BF16 && !a.b_mn_major && a.N < 8192) return false;
  // Short, narrow GEMMs (attn c_proj forward and data gradient: K = N = 768)
  // lose on pairs: 0.0489 vs 0.0442 ms and 0.0284 vs 0.0251 ms.
  if (a.K <= 1024 && a.N < 8192 && a.splits <= 1) return false;
  return kPairDefault;
}

__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits,
                                     int64_t split_stride, float* __restrict__ out, int64_t ldo,
                                     int M, int N, int accumulate) {
  const int64_t n4 = N / 4;
  const int64_t total = (int64_t)M * n4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n4, c = (i % n4) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < splits; ++s) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(ws + s * split_stride + r * N + c));
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    float4* o = reinterpret_cast<float4*>(out + r * ldo + c);
    if (accumulate) {
      const float4 old = *o;
      acc.x += old.x;
      acc.y += old.y;
      acc.z += old.z;
      acc.w += old.w;
    }
    *o = acc;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

int gemm_bf16_launch(const GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return -1;
  if (a.bn != 256 && a.bn != 128) return -2;
  // TMA operand loads: 16-byte aligned base and row stride.
  if (!aligned16(a.A) || !aligned16(a.B)) return -4;
  if ((a.lda * 2) % 16 || (a.ldb * 2) % 16) return -5;
  if (a.splits > 1 && a.epilogue != EPI_F32) return -6;
  Maps maps;
  const int BN = a.bn;
  bool ok = a.a_mn_major ? make_tmap_2d(&maps.a, a.A, a.M, a.K, a.lda, BK)
                         : make_tmap_2d(&maps.a, a.A, a.K, a.M, a.lda, BM);
  if (!ok) return -7;
  const bool pairs = use_pairs(a);
  ok = a.b_mn_major ? make_tmap_2d(&maps.b, a.B, a.N, a.K, a.ldb, BK)
                    : make_tmap_2d(&maps.b, a.B, a.K, a.N, a.ldb, pairs ? BN / 2 : BN);
  if (!ok) return -8;

  GemmDev d;
  d.M = a.M;
  d.N = a.N;
  d.K = a.K;
  d.m_tiles = (a.M + BM - 1) / BM;
  d.n_tiles = (a.N + BN - 1) / BN;
  d.kb_total = (a.K + BK - 1) / BK;
  d.splits = a.splits < 1 ? 1 : a.splits;
  if (d.splits > d.kb_total) d.splits = d.kb_total;
  d.kb_per_split = (d.kb_total + d.splits - 1) / d.splits;
  d.splits = (d.kb_total + d.kb_per_split - 1) / d.kb_per_split;
  const bool split_mode = d.splits > 1;
  if (split_mode && (a.workspace == nullptr || a.N % 4 || a.ldo % 4)) return -9;
  // Split-K: each split writes an fp32 partial [M, N] (row stride N) into the
  // workspace; a deterministic reduction then adds them into `out` in order.
  d.out = split_mode ? a.workspace : a.out;
  d.ldo = split_mode ? a.N : a.ldo;
  d.aux = a.aux;
  d.ldaux = a.ldaux;
  d.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  d.alpha_ptr = a.alpha_ptr;
  d.alpha = a.alpha;
  d.accumulate = split_mode ? 0 : a.accumulate;
  d.split_stride = split_mode ? (int64_t)a.M * a.N : 0;
  d.err = a.err;
  d.ce_stats = reinterpret_cast<float2*>(a.ce_stats);
  d.ce_targets = a.ce_targets;
  d.ce_tgt_logit = a.ce_tgt_logit;
  d.ce_vocab_offset = a.ce_vocab_offset;
  d.owner_out = a.owner_out;
  d.owner_rows = a.owner_rows;
  d.owner_self = a.owner_self;
  d.m_fast = d.n_tiles > (pairs ? (a.M + 2 * BM - 1) / (2 * BM) : d.m_tiles) ? 1 : 0;
  if (a.owner_out && (a.owner_rows <= 0 || (a.epilogue != EPI_BF16) || split_mode)) return -13;
  if (a.epilogue == EPI_CE_STATS &&
      (!a.ce_stats || !a.ce_targets || !a.ce_tgt_logit || split_mode || a.bias))
    return -12;
  const int esz = (a.epilogue == EPI_F32 || a.epilogue == EPI_RESID_F32) ? 4 : 2;
  bool vec = aligned16(d.out) && ((d.ldo * esz) % 16 == 0);
  if (a.aux)
    vec = vec && aligned16(a.aux) &&
          ((a.ldaux * (a.epilogue == EPI_RESID_F32 ? 4 : 2)) % 16 == 0);
  if (a.bias) vec = vec && aligned16(a.bias);
  d.vec_ok = vec ? 1 : 0;

  // TMA stores need the same alignment as the vector path. Row-owner output:
  // tiles of this GPU's rows (owner_self) are TMA-stored into `out`, which is
  // this GPU's inbox, other tiles use direct stores into the owners' memory.
  int tma_st = (vec && (!a.owner_out || a.owner_self >= 0)) ? 1 : 0;
  if (tma_st) {
    ok = make_tmap_out(&maps.o, d.out, a.N, a.M, d.splits, d.ldo, esz);
    if (ok && a.epilogue == EPI_BIAS_GELU) ok = make_tmap_out(&maps.x, a.aux, a.N, a.M, 1, a.ldaux, 2);
    if (!ok) tma_st = 0;
  }
  if (!tma_st) {
    maps.o = maps.a;  // unused placeholders
    maps.x = maps.a;
  } else if (a.epilogue != EPI_BIAS_GELU) {
    maps.x = maps.o;
  }

  if (pairs) {
    const int ptiles = (a.M + 2 * BM - 1) / (2 * BM) * d.n_tiles * d.splits;
    int rc = pair_epi(a.epilogue, tma_st, a.a_mn_major, a.b_mn_major, maps, d, ptiles, a.max_ctas,
                      stream);
    if (rc != 0 || !split_mode) return rc;
    return splitk_reduce_launch(reinterpret_cast<const float*>(a.workspace), d.splits,
                                d.split_stride, reinterpret_cast<float*>(a.out), a.ldo, a.M, a.N,
                                a.accumulate, stream);
  }
  const int tiles = d.m_tiles * d.n_tiles * d.splits;
  int grid = a.max_ctas > 0 ? a.max_ctas : num_sms();
  if (grid > tiles) grid = tiles;
  // more tiles than CTAs: claim them dynamically (each tile's result is
  // independent, so the order of claims does not change any output bit)
  d.sched = tiles > grid ? gemm_sched_slot() : nullptr;
  int rc = BN == 256 ? dispatch_epi<256>(a.epilogue, tma_st, a.a_mn_major, a.b_mn_major, maps, d, grid, stream)
                     : dispatch_epi<128>(a.epilogue, tma_st, a.a_mn_major, a.b_mn_major, maps, d, grid, stream);
  if (rc != 0 || !split_mode) return rc;
  return splitk_reduce_launch(reinterpret_cast<const float*>(a.workspace), d.splits,
                              d.split_stride, reinterpret_cast<float*>(a.out), a.ldo, a.M, a.N,
                              a.accumulate, stream);
}

int splitk_reduce_launch(const float* ws, int splits, int64_t split_stride, float* out,
                         int64_t ldo, int M, int N, int accumulate, cudaStream_t stream) {
  if (N % 4 || ldo % 4) return -1;
  const int64_t total = (int64_t)M * (N / 4);
  int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 8);
  splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(ws, splits, split_stride, out, ldo, M, N,
                                                   accumulate);
  count_launches(1);
  return launch_succeeded() ? 0 : -11;
}

}  // namespace g2b
