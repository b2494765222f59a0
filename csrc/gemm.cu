// Persistent, warp-specialised bf16 GEMM for sm_100a on the 5th-generation
// tensor cores (tcgen05.mma, fp32 accumulator in TMEM), fed by TMA.
//
//   C[M,N] = A[M,K] . B[N,K]^T   (A and B each K-major or MN-major)
//
// One CTA per SM (persistent; tiles strided by gridDim.x), 192 threads:
//   warp 0      TMA producer: one elected lane streams A/B k-blocks into a
//               STAGES-deep ring of 128B-swizzled shared-memory stages.
//   warp 1      MMA issuer: allocates TMEM, one elected lane issues
//               tcgen05.mma 128xBNx16 per 16-wide k slice and commits each
//               stage back to the producer; the accumulator is double buffered
//               in TMEM (2 x BN fp32 columns) so tile i+1's MMAs overlap tile
//               i's epilogue.
//   warps 2..5  epilogue: tcgen05.ld the accumulator (one TMEM lane = one
//               output row per thread), apply the fused epilogue (bias, GELU,
//               GELU backward, fp32 residual add, split-K partial) and store.
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

#include "common.cuh"
#include "gemm.cuh"

namespace g2b {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // double-buffered accumulator
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
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
};

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmDev& p, int row, int n0, float* v) {
  if (row >= p.M || n0 >= p.N) return;
  const bool full = (n0 + 32 <= p.N) && p.vec_ok;
  float bias[32];
  if (p.bias != nullptr && (EPI == EPI_BF16 || EPI == EPI_BIAS_GELU || EPI == EPI_RESID_F32)) {
    if (full) {
      const uint4* bp = reinterpret_cast<const uint4*>(p.bias + n0);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w = __ldg(bp + q);
        uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = unpack_bf16x2(ws[j]);
          bias[q * 8 + 2 * j] = f.x;
          bias[q * 8 + 2 * j + 1] = f.y;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        bias[i] = (n0 + i < p.N) ? __bfloat162float(p.bias[n0 + i]) : 0.f;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) bias[i] = 0.f;
  }

  if (EPI == EPI_BF16 || EPI == EPI_BIAS_GELU) {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)row * p.ldo + n0;
    __nv_bfloat16* a = EPI == EPI_BIAS_GELU
                           ? reinterpret_cast<__nv_bfloat16*>(p.aux) + (int64_t)row * p.ldaux + n0
                           : nullptr;
    float y[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      v[i] += bias[i];
      y[i] = EPI == EPI_BIAS_GELU ? gelu_tanh_f(v[i]) : v[i];
    }
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
          u.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
          u.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
          u.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
          u.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
          reinterpret_cast<uint4*>(a)[q] = u;
        }
      }
    } else {
      for (int i = 0; i < 32 && n0 + i < p.N; ++i) {
        o[i] = __float2bfloat16(y[i]);
        if (EPI == EPI_BIAS_GELU) a[i] = __float2bfloat16(v[i]);
      }
    }
  } else if (EPI == EPI_GELU_BWD) {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)row * p.ldo + n0;
    const __nv_bfloat16* a =
        reinterpret_cast<const __nv_bfloat16*>(p.aux) + (int64_t)row * p.ldaux + n0;
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u = reinterpret_cast<const uint4*>(a)[q];
        uint32_t us[4] = {u.x, u.y, u.z, u.w};
        float g[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = unpack_bf16x2(us[j]);
          g[2 * j] = v[q * 8 + 2 * j] * gelu_tanh_grad_f(f.x);
          g[2 * j + 1] = v[q * 8 + 2 * j + 1] * gelu_tanh_grad_f(f.y);
        }
        uint4 w;
        w.x = pack_bf16x2(g[0], g[1]);
        w.y = pack_bf16x2(g[2], g[3]);
        w.z = pack_bf16x2(g[4], g[5]);
        w.w = pack_bf16x2(g[6], g[7]);
        reinterpret_cast<uint4*>(o)[q] = w;
      }
    } else {
      for (int i = 0; i < 32 && n0 + i < p.N; ++i)
        o[i] = __float2bfloat16(v[i] * gelu_tanh_grad_f(__bfloat162float(a[i])));
    }
  } else {  // fp32 outputs
    float* o = reinterpret_cast<float*>(p.out) + (int64_t)row * p.ldo + n0;
    const bool add_old = (EPI == EPI_RESID_F32) || (p.accumulate != 0);
    // The residual epilogue may read its old value from a separate fp32 source
    // (aux) so the stream can advance out of place: out = aux + acc + bias.
    const float* src = (EPI == EPI_RESID_F32 && p.aux != nullptr)
                           ? reinterpret_cast<const float*>(p.aux) + (int64_t)row * p.ldaux + n0
                           : o;
    if (full) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 r = make_float4(v[q * 4] + bias[q * 4], v[q * 4 + 1] + bias[q * 4 + 1],
                               v[q * 4 + 2] + bias[q * 4 + 2], v[q * 4 + 3] + bias[q * 4 + 3]);
        if (add_old) {
          float4 old = reinterpret_cast<const float4*>(src)[q];
          r.x += old.x;
          r.y += old.y;
          r.z += old.z;
          r.w += old.w;
        }
        reinterpret_cast<float4*>(o)[q] = r;
      }
    } else {
      for (int i = 0; i < 32 && n0 + i < p.N; ++i) {
        float r = v[i] + bias[i];
        if (add_old) r += src[i];
        o[i] = r;
      }
    }
  }
}

template <int BN, int EPI, int A_MN, int B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmDev p) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
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
      mbar_init(&tempty_bar[b], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane_id() == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
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
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int split = tile / tiles_per_split;
        const int rem = tile % tiles_per_split;
        const int m0 = (rem / p.n_tiles) * BM;
        const int n0 = (rem % p.n_tiles) * BN;
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
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
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
    const int lane_grp = warp & 3;  // TMEM lanes 32*lane_grp .. +31
    const int row_in_tile = lane_grp * 32 + lane_id();
    int acc = 0;
    uint32_t acc_phase = 0;
    float alpha = p.alpha;
    if (p.alpha_ptr) alpha *= *p.alpha_ptr;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int split = tile / tiles_per_split;
      const int rem = tile % tiles_per_split;
      const int m0 = (rem / p.n_tiles) * BM;
      const int n0 = (rem % p.n_tiles) * BN;
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, p.err, ERR_TIMEOUT_EPILOGUE, abort_flag))
        break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(lane_grp * 32) << 16) + acc * BN;
      GemmDev q = p;
      if (EPI == EPI_F32 && p.splits > 1)
        q.out = reinterpret_cast<float*>(p.out) + (int64_t)split * p.split_stride;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(t_row + c * 32, v);
        tmem_wait_ld();
        if (c == BN / 32 - 1) {
          tc_fence_before();
          mbar_arrive(&tempty_bar[acc]);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= alpha;
        epilogue_chunk<EPI>(q, m0 + row_in_tile, n0 + c * 32, v);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host ---
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

// 2-D bf16 tensor map: inner extent `inner` (contiguous), outer extent `outer`
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

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, int EPI, int A_MN, int B_MN>
int launch_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const GemmDev& d, int grid,
               cudaStream_t s) {
  auto kern = gemm_tcgen05_kernel<BN, EPI, A_MN, B_MN>;
  constexpr int smem = GemmCfg<BN>::SMEM_BYTES;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return -10;
    attr_set = true;
  }
  kern<<<grid, kThreads, smem, s>>>(ta, tb, d);
  count_launches(1);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

template <int BN, int EPI>
int dispatch_major(int amn, int bmn, const CUtensorMap& ta, const CUtensorMap& tb,
                   const GemmDev& d, int grid, cudaStream_t s) {
  if (!amn && !bmn) return launch_cfg<BN, EPI, 0, 0>(ta, tb, d, grid, s);
  if (!amn && bmn) return launch_cfg<BN, EPI, 0, 1>(ta, tb, d, grid, s);
  if (amn && bmn) return launch_cfg<BN, EPI, 1, 1>(ta, tb, d, grid, s);
  return launch_cfg<BN, EPI, 1, 0>(ta, tb, d, grid, s);
}

template <int BN>
int dispatch_epi(int epi, int amn, int bmn, const CUtensorMap& ta, const CUtensorMap& tb,
                 const GemmDev& d, int grid, cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: return dispatch_major<BN, EPI_BF16>(amn, bmn, ta, tb, d, grid, s);
    case EPI_BIAS_GELU: return dispatch_major<BN, EPI_BIAS_GELU>(amn, bmn, ta, tb, d, grid, s);
    case EPI_RESID_F32: return dispatch_major<BN, EPI_RESID_F32>(amn, bmn, ta, tb, d, grid, s);
    case EPI_F32: return dispatch_major<BN, EPI_F32>(amn, bmn, ta, tb, d, grid, s);
    case EPI_GELU_BWD: return dispatch_major<BN, EPI_GELU_BWD>(amn, bmn, ta, tb, d, grid, s);
  }
  return -3;
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
      float4 v = *reinterpret_cast<const float4*>(ws + s * split_stride + r * N + c);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    float4* o = reinterpret_cast<float4*>(out + r * ldo + c);
    if (accumulate) {
      float4 old = *o;
      acc.x += old.x;
      acc.y += old.y;
      acc.z += old.z;
      acc.w += old.w;
    }
    *o = acc;
  }
}

}  // namespace

int gemm_bf16_launch(const GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return -1;
  if (a.bn != 256 && a.bn != 128) return -2;
  // TMA: 16-byte aligned base and row stride.
  if ((reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.B) & 15)) return -4;
  if ((a.lda * 2) % 16 || (a.ldb * 2) % 16) return -5;
  if (a.splits > 1 && a.epilogue != EPI_F32) return -6;
  CUtensorMap ta, tb;
  const int BN = a.bn;
  bool ok;
  if (a.a_mn_major)
    ok = make_tmap_2d(&ta, a.A, a.M, a.K, a.lda, BK);
  else
    ok = make_tmap_2d(&ta, a.A, a.K, a.M, a.lda, BM);
  if (!ok) return -7;
  if (a.b_mn_major)
    ok = make_tmap_2d(&tb, a.B, a.N, a.K, a.ldb, BK);
  else
    ok = make_tmap_2d(&tb, a.B, a.K, a.N, a.ldb, BN);
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
  d.split_stride = (int64_t)a.M * a.N;
  d.err = a.err;
  const int esz = (a.epilogue == EPI_F32 || a.epilogue == EPI_RESID_F32) ? 4 : 2;
  bool vec = (reinterpret_cast<uintptr_t>(d.out) % 16 == 0) && ((d.ldo * esz) % 16 == 0);
  if (a.aux)
    vec = vec && (reinterpret_cast<uintptr_t>(a.aux) % 16 == 0) &&
          ((a.ldaux * (a.epilogue == EPI_RESID_F32 ? 4 : 2)) % 16 == 0);
  if (a.bias) vec = vec && (reinterpret_cast<uintptr_t>(a.bias) % 16 == 0);
  if (split_mode) vec = vec && (d.split_stride * 4) % 16 == 0;
  d.vec_ok = vec ? 1 : 0;

  const int tiles = d.m_tiles * d.n_tiles * d.splits;
  int grid = a.max_ctas > 0 ? a.max_ctas : num_sms();
  if (grid > tiles) grid = tiles;
  int rc = BN == 256
               ? dispatch_epi<256>(a.epilogue, a.a_mn_major, a.b_mn_major, ta, tb, d, grid, stream)
               : dispatch_epi<128>(a.epilogue, a.a_mn_major, a.b_mn_major, ta, tb, d, grid, stream);
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
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

}  // namespace g2b
