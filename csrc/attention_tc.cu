// Causal flash-attention forward on the 5th-generation tensor cores (sm_100a).
//
// Same contract as attn_fwd_kernel in attention.cu (head_dim 64, bf16 Q/K/V/O,
// log2-domain row LSE saved for backward, implicit causal mask at absolute
// positions q_offset + i vs j), re-designed around tcgen05:
//
//  * Persistent: one CTA per SM walks work items (TWO 128-query tiles of one
//    (batch, head)) in a snake order over heaviest-first items, and streams
//    128-key K/V blocks through a 3-stage TMA ring shared by both tiles. Q is
//    double-buffered and every barrier phase is a running count, so the next
//    item's Q loads and first S = Q K^T overlap this item's last softmax and
//    its O write-out.
//  * warp 0: TMA producer (4-D tensor maps over the strided head views, so Q,
//    K, V are read straight out of the fused qkv buffer).
//    warp 1: MMA issuer. Per key block and tile: S = Q K^T (128x128x64, both
//    operands K-major, fp32 accumulator in TMEM), then O_tile = P V
//    (128x64x128; P from shared memory, V as an MN-major operand).
//    warps 2-5 / 6-9: one softmax warpgroup per query tile (FA4-style
//    ping-pong: while one group does exponentials the tensor core works on
//    the other tile). A thread owns one query row = one TMEM lane.
//  * Online softmax: a pass over the S row (TMEM) for its max, a second pass
//    that writes P (exp2 domain) as bf16 into a 128B-swizzled K-major shared
//    tile the P.V MMA consumes; each pass keeps two 32-column loads in
//    flight. O accumulates in TMEM across key blocks. The running max
//    is raised lazily -- only when a row's max grows by more than 2^8 -- in
//    which case the softmax warp rescales O in TMEM (ld, scale, st) before
//    the next P.V accumulates. The previous P.V is always complete by then
//    (it precedes this block's S on the in-order tensor pipe).
//  * Every mbarrier wait is bounded (ERR_TIMEOUT_ATTN on expiry).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>

#include "attention.cuh"
#include "attention_peers.cuh"
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
constexpr int NG = 2;    // query tiles (softmax warpgroups) per work item
constexpr int TKV = 64;  // keys per block
constexpr int KS = 5;    // K/V ring stages
constexpr int QB = 2;    // Q buffers (the next item's Q loads during this one)
constexpr int kThreads = 64 + NG * 128;
constexpr int QTILE = 128 * 128;   // 128 rows x 64 bf16
constexpr int KVTILE = 64 * 128;   // 64 rows x 64 bf16
constexpr int PTILE = 128 * 128;   // 128 query rows x 64 keys bf16
constexpr int Q_OFF = 0;
constexpr int K_OFF = Q_OFF + QB * NG * QTILE;
constexpr int V_OFF = K_OFF + KS * KVTILE;
constexpr int P_OFF = V_OFF + KS * KVTILE;  // [NG][2] double-buffered P tiles
constexpr int BAR_OFF = P_OFF + NG * 2 * PTILE;
constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
constexpr float kLog2e = 1.4426950408889634f;
// TMEM columns: S of tile g, buffer b at g*128 + b*64; O of tile g at 256 + g*64.
constexpr uint32_t kTmemCols = 512;

struct TcParams {
  int B, H, Tq, Tk, q_offset, causal;
  int n_qpairs, n_items;
  int grp;    // query heads per key/value head
  float sl2;  // softmax scale * log2(e)
  __nv_bfloat16* o;
  int64_t osb, ost, osh;
  float* lse;
  uint32_t* err;
#ifdef G2B_ATTN_FWD_TRACE
  unsigned long long* trace;  // [3 roles][256 blocks][8 events] of CTA 0 (%globaltimer ns)
#endif
};

#ifdef G2B_ATTN_FWD_TRACE
#define FTR(role, c, ev)                                                                  \
  do {                                                                                    \
    if (p.trace && blockIdx.x == 0 && (c) < 256)                                         \
      p.trace[((role) * 256 + (c)) * 8 + (ev)] = globaltimer_ns();                        \
  } while (0)
#else
#define FTR(role, c, ev) \
  do {                   \
  } while (0)
#endif

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Work item w -> (query-tile pair, batch*head). Items are ordered heaviest
// first under the causal mask (last query pairs see the most keys).
struct Item {
  int q0, bh, nblk[NG], nmax;
};
__device__ __forceinline__ Item item_of(const TcParams& p, int w) {
  Item it;
  const int BH = p.B * p.H;
  const int qpair = p.n_qpairs - 1 - w / BH;
  it.bh = w % BH;
  it.q0 = qpair * (NG * TQ);
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    int kv_end = p.Tk;
    if (p.causal) kv_end = min(p.Tk, p.q_offset + it.q0 + (g + 1) * TQ);
    const bool tile_live = it.q0 + g * TQ < p.Tq;
    it.nblk[g] = (tile_live && kv_end > 0) ? (kv_end + TKV - 1) / TKV : 0;
  }
  it.nmax = max(it.nblk[0], it.nblk[1]);
  return it;
}

// The r-th item of this CTA: snake order over rounds of gridDim.x items, which
// balances the heavy-first cost classes across CTAs without shared state.
__device__ __forceinline__ int item_index(int r) {
  const int G = gridDim.x;
  return r * G + ((r & 1) ? (G - 1 - (int)blockIdx.x) : (int)blockIdx.x);
}

// Of a block's 64 exponentials per row, kMufu run on the exponential unit and
// the rest on the FMA pipe (exp2_fma). Measured on a B200 (16x1024, 12 heads):
// 32 -> 0.0935 ms, 40 and 48 -> 0.0903 ms, 64 -> 0.0935 ms.
constexpr int kMufu = 48;

// KV = NoKvPeers: keys and values through tmK / tmV. KV = KvPeerMaps
// (context parallelism, streaming): each key block through its owner's maps.
template <class KV>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const TcParams p,
                       const __grid_constant__ KV kv) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* q_full = bars;              // QB
  uint64_t* q_empty = q_full + QB;      // QB
  uint64_t* kv_full = q_empty + QB;     // KS
  uint64_t* kv_empty = kv_full + KS;    // KS
  uint64_t* s_full = kv_empty + KS;     // NG x 2 (S double buffer)
  uint64_t* p_full = s_full + 2 * NG;   // NG
  // o_full[2g + b]: P.V of tile g's blocks with count parity b is complete
  // (phase k of barrier b = the P.V of block count 2k + b)
  uint64_t* o_full = p_full + NG;       // NG x 2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 2 * NG);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    for (int i = 0; i < QB; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < KS; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int g = 0; g < NG; ++g) {
      mbar_init(&s_full[2 * g], 1);
      mbar_init(&s_full[2 * g + 1], 1);
      mbar_init(&p_full[g], 128);
      mbar_init(&o_full[2 * g], 1);
      mbar_init(&o_full[2 * g + 1], 1);
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
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int kv_count = 0;  // K/V blocks issued by this CTA so far (ring position)
      int qi = 0;        // items loaded so far (Q buffer position)
      uint32_t owners_seen = 0;  // streaming: owners whose publish flag was seen
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int w = item_index(r);
        if (w >= p.n_items) break;
        const Item it = item_of(p, w);
        if (it.nmax == 0) continue;
        const int b = it.bh / p.H, h = it.bh % p.H;
        const int qb = qi % QB;
        if (!mbar_wait_bounded(&q_empty[qb], ((qi / QB) & 1) ^ 1, p.err, ERR_TIMEOUT_ATTN,
                               abort_flag))
          break;
        ++qi;
        mbar_arrive_expect_tx(&q_full[qb], NG * QTILE);
        for (int g = 0; g < NG; ++g)
          tma_load_4d(smem + Q_OFF + (qb * NG + g) * QTILE, &tmQ, &q_full[qb], 0, h,
                      it.q0 + g * TQ, b);
        for (int j = 0; j < it.nmax; ++j, ++kv_count) {
          const int st = kv_count % KS;
          if (!mbar_wait_bounded(&kv_empty[st], ((kv_count / KS) & 1) ^ 1, p.err,
                                 ERR_TIMEOUT_ATTN, abort_flag)) {
            ok = false;
            break;
          }
          if constexpr (KvStreaming<KV>::on) {
            int row;
            const int q = kv_owner_row(kv, j * TKV, &row);
            if (!kv_owner_ready(kv, q, &owners_seen, p.err, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&kv_full[st], 2 * KVTILE);
            tma_load_4d(smem + K_OFF + st * KVTILE, &kv.k[q], &kv_full[st], 0, h / p.grp, row, b);
            tma_load_4d(smem + V_OFF + st * KVTILE, &kv.v[q], &kv_full[st], 0, h / p.grp, row, b);
          } else {
            mbar_arrive_expect_tx(&kv_full[st], 2 * KVTILE);
            tma_load_4d(smem + K_OFF + st * KVTILE, &tmK, &kv_full[st], 0, h / p.grp, j * TKV, b);
            tma_load_4d(smem + V_OFF + st * KVTILE, &tmV, &kv_full[st], 0, h / p.grp, j * TKV, b);
          }
        }
      }
      if (*abort_flag) {
        // A role gave up (this one on a peer's flag, or another on a
        // barrier): wait (bounded) for this warp's copies still in flight
        // before the CTA's shared memory is released.
        if (qi) mbar_wait_bounded(&q_full[(qi - 1) % QB], ((qi - 1) / QB) & 1, p.err, ERR_TIMEOUT_ATTN,
                                  nullptr);
        for (int kc = kv_count > KS ? kv_count - KS : 0; kc < kv_count; ++kc)
          mbar_wait_bounded(&kv_full[kc % KS], (kc / KS) & 1, p.err, ERR_TIMEOUT_ATTN, nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    // Per tile g and block c (running count): S(c) = Q K_c^T into S buffer
    // c%2, P.V(c) accumulated into O. S(c+2) is issued right after P.V(c),
    // so S is always one block ahead of the softmax warps.
    if (elect_one()) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, TKV, 0, 0);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(128, 64, 0, 1);
      int kv_count = 0;
      int cnt[NG] = {0, 0};  // blocks of each tile processed so far (barrier phases)
      int qi = 0;
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int w = item_index(r);
        if (w >= p.n_items) break;
        const Item it = item_of(p, w);
        if (it.nmax == 0) continue;
        const int qb = qi % QB;
        const uint32_t qphase = (qi / QB) & 1;
        ++qi;
        auto kv_wait = [&](int kc) {
          return mbar_wait_bounded(&kv_full[kc % KS], (kc / KS) & 1, p.err, ERR_TIMEOUT_ATTN,
                                   abort_flag);
        };
        auto issue_s = [&](int g, int c, int st) {  // S of tile g, block count c, stage st
          const uint32_t qa = smem_u32(smem + Q_OFF + (qb * NG + g) * QTILE);
          const uint32_t kb = smem_u32(smem + K_OFF + st * KVTILE);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + g * 128 + (c & 1) * 64, umma_desc_sw128(qa + kk * 32, 16, 1024),
                      umma_desc_sw128(kb + kk * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(&s_full[2 * g + (c & 1)]);
        };
        ok = mbar_wait_bounded(&q_full[qb], qphase, p.err, ERR_TIMEOUT_ATTN, abort_flag);
        // S of blocks 0 and 1 for both tiles. Both S buffers are free: the
        // previous item's last S was consumed before its last P.V was issued.
        for (int jb = 0; jb < 2 && ok; ++jb) {
          if (jb >= it.nmax) break;
          if (!kv_wait(kv_count + jb)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int g = 0; g < NG; ++g)
            if (jb < it.nblk[g]) issue_s(g, cnt[g] + jb, (kv_count + jb) % KS);
        }
        for (int j = 0; j < it.nmax && ok; ++j) {
          const int kc = kv_count + j;
          const int st = kc % KS;
          const bool next_ready = j + 2 < it.nmax;
          if (next_ready && !kv_wait(kc + 2)) {
            ok = false;
            break;
          }
          for (int g = 0; g < NG && ok; ++g) {
            if (j >= it.nblk[g]) continue;
            const int c = cnt[g] + j;
            // P(c) written: S(c) consumed, O rescaled if the row max moved
            if (!mbar_wait_bounded(&p_full[g], c & 1, p.err, ERR_TIMEOUT_ATTN, abort_flag)) {
              ok = false;
              break;
            }
            FTR(g, c, 3);
            tc_fence_after();
            const uint32_t pa = smem_u32(smem + P_OFF + (g * 2 + (c & 1)) * PTILE);
            const uint32_t vb = smem_u32(smem + V_OFF + st * KVTILE);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma_bf16(tmem + 256 + g * 64, umma_desc_sw128(pa + ks * 32, 16, 1024),
                        umma_desc_sw128(vb + ks * 2048, 8192, 1024), idesc_pv,
                        (ks > 0 || j > 0) ? 1u : 0u);
            umma_commit(&o_full[2 * g + (c & 1)]);
            if (j + 2 < it.nblk[g]) issue_s(g, c + 2, (kc + 2) % KS);
          }
          umma_commit(&kv_empty[st]);
        }
        umma_commit(&q_empty[qb]);  // every S of this item has read its Q
        kv_count += it.nmax;
        for (int g = 0; g < NG; ++g) cnt[g] += it.nblk[g];
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- softmax
    // One thread = one query row = one TMEM lane. Per 64-key block: the S row
    // (two 32-column TMEM loads, one wait) is held in registers, its max
    // taken, and P = 2^(s*sl2 - m) written as bf16 into this tile's P buffer
    // c%2 (128B-swizzled, K-major) for the P.V MMA, which accumulates into O
    // in TMEM. The running max m is raised lazily: only when a row's block
    // max exceeds it by more than kRescale (log2 units), in which case O and
    // l are rescaled; otherwise the stale m keeps every p <= 2^kRescale.
    constexpr float kRescale = 8.f;
    const int g = (warp - 2) >> 2;
    const int lg = warp & 3;
    const int lane = (int)lane_id();
    const int r_row = lg * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(lg * 32) << 16);
    const uint32_t t_o = lane_base + 256 + g * 64;
    const bool tr = lg == 0 && lane == 0;
    int cnt = 0;    // blocks of this tile processed so far (barrier phases)
    bool ok = true;
    for (int r = 0; ok; ++r) {
      const int w = item_index(r);
      if (w >= p.n_items) break;
      const Item it = item_of(p, w);
      const int n = it.nblk[g];
      if (n == 0) continue;
      const int b = it.bh / p.H, h = it.bh % p.H;
      const int row_q = it.q0 + g * TQ + r_row;
      const int abs_q = p.q_offset + row_q;
      const int tile_q_min = p.q_offset + it.q0 + g * TQ;
      // The two groups exponentiate independently: making them take turns on
      // the exponential unit (one group's max/P work overlapping the other's
      // exponentials) measured 0.0910 ms against 0.0858 ms without, once
      // neither waits for the previous block's P.V.
      float m = -INFINITY, l = 0.f;

      for (int j = 0; j < n && ok; ++j) {
        const int c = cnt + j;
        if (tr) FTR(g, c, 0);
        if (!mbar_wait_bounded(&s_full[2 * g + (c & 1)], (c >> 1) & 1, p.err, ERR_TIMEOUT_ATTN,
                               abort_flag)) {
          ok = false;
          break;
        }
        if (tr) FTR(g, c, 1);
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
        uint32_t sa[32], sb[32];
        const uint32_t t_s = lane_base + g * 128 + (c & 1) * 64;
        tmem_ld32_async(t_s, sa);
        tmem_ld32_async(t_s + 32, sb);
        tmem_wait_ld_into(sa);
        tmem_wait_ld_into(sb);
        if (tr) FTR(g, c, 4);
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float va = i < valid ? __uint_as_float(sa[i]) : -INFINITY;
            const float vb = i + 32 < valid ? __uint_as_float(sb[i]) : -INFINITY;
            mx8[i & 7] = fmaxf(mx8[i & 7], fmaxf(va, vb));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            mx8[i & 7] = fmaxf(mx8[i & 7], fmaxf(__uint_as_float(sa[i]), __uint_as_float(sb[i])));
        }
        float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                         fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        mx = mx == -INFINITY ? -INFINITY : mx * p.sl2;
        if (tr) FTR(g, c, 2);
        // Raise the running max lazily (warp-uniform decision); O is rescaled
        // after P is written, when the S registers are dead.
        bool rescale = false;
        float corr = 1.f;
        if (j == 0) {
          m = mx;  // O is overwritten by this block's P.V: nothing to rescale
        } else {
          const bool need = mx > m + kRescale;
          if (__any_sync(0xffffffffu, need)) {
            rescale = true;
            const float m_new = need ? mx : m;
            corr = ex2f(m - m_new);
            l *= corr;
            m = m_new;
          }
        }
        const float base = m == -INFINITY ? 0.f : m;
        uint8_t* pbuf = smem + P_OFF + (g * 2 + (c & 1)) * PTILE;
        // All 64 exponentials first (in place, independent: the exponential
        // unit stays busy), then the masked row sum and the bf16 P tile.
        // the exponential unit takes the first kMufu keys, the FMA pipe the
        // rest (exp2_fma): the two pipes run side by side
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          sa[i] = __float_as_uint(ex2f(fmaf(__uint_as_float(sa[i]), p.sl2, -base)));
          const float xb = fmaf(__uint_as_float(sb[i]), p.sl2, -base);
          sb[i] = __float_as_uint(i < kMufu - 32 ? ex2f(xb) : exp2_fma(xb));
        }
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (i >= valid) sa[i] = 0u;
            if (i + 32 >= valid) sb[i] = 0u;
          }
        }
        // P buffer c%2 was last read by P.V(c-2): wait for it (long done in
        // the steady state; an earlier item's P.V was already waited for)
        if (c >= 2 && !mbar_wait_bounded(&o_full[2 * g + (c & 1)], ((c - 2) >> 1) & 1, p.err,
                                         ERR_TIMEOUT_ATTN, abort_flag)) {
          ok = false;
          break;
        }
        float rs8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) rs8[i] = 0.f;
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {  // 16-byte chunk (8 keys) index
          const uint32_t* e = jj < 4 ? sa + jj * 8 : sb + (jj - 4) * 8;
#pragma unroll
          for (int t = 0; t < 8; ++t) rs8[t] += __uint_as_float(e[t]);
          uint4 wv;
          wv.x = pack_bf16x2(__uint_as_float(e[0]), __uint_as_float(e[1]));
          wv.y = pack_bf16x2(__uint_as_float(e[2]), __uint_as_float(e[3]));
          wv.z = pack_bf16x2(__uint_as_float(e[4]), __uint_as_float(e[5]));
          wv.w = pack_bf16x2(__uint_as_float(e[6]), __uint_as_float(e[7]));
          *reinterpret_cast<uint4*>(pbuf + r_row * 128 + (((jj & 7) ^ (r_row & 7)) << 4)) = wv;
        }
        if (tr) FTR(g, c, 5);
        // O is rescaled only once P.V(c-1) is complete; otherwise P.V(c-1)
        // is not waited for here, so the tensor core runs it while this
        // group turns the next S into P. Each parity barrier is still
        // waited for phase by phase (P.V(k) at block k+2), never more than
        // one phase behind, so its parity cannot alias.
        if (rescale &&
            !mbar_wait_bounded(&o_full[2 * g + ((c - 1) & 1)], ((c - 1) >> 1) & 1, p.err,
                               ERR_TIMEOUT_ATTN, abort_flag)) {
          ok = false;
          break;
        }
        if (rescale) {
          tc_fence_after();
          uint32_t t0[32], t1[32];
          tmem_ld32_async(t_o, t0);
          tmem_ld32_async(t_o + 32, t1);
          tmem_wait_ld_into(t0);
          tmem_wait_ld_into(t1);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            t0[i] = __float_as_uint(__uint_as_float(t0[i]) * corr);
            t1[i] = __float_as_uint(__uint_as_float(t1[i]) * corr);
          }
          tmem_st32(t_o, t0);
          tmem_st32(t_o + 32, t1);
          tmem_wait_st();
        }
        if (tr) FTR(g, c, 6);
        fence_proxy_async_shared();
        tc_fence_before();
        if (tr) FTR(g, c, 7);
        mbar_arrive(&p_full[g]);
        l += ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
      }
      if (!ok) break;
      // epilogue: O = (sum over blocks of P.V) / l, read once the last P.V is done
      const int c_end = cnt + n - 1;  // the item's last block: its P.V completes after all others
      if (!mbar_wait_bounded(&o_full[2 * g + (c_end & 1)], (c_end >> 1) & 1, p.err, ERR_TIMEOUT_ATTN,
                             abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t t0[32], t1[32];
      tmem_ld32_async(t_o, t0);
      tmem_ld32_async(t_o + 32, t1);
      tmem_wait_ld_into(t0);
      tmem_wait_ld_into(t1);
      // the next item's first P.V overwrites O only after this warp's next
      // p_full arrive, which follows these loads in program order
      cnt += n;
      if (row_q < p.Tq) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __nv_bfloat16* orow =
            p.o + (int64_t)b * p.osb + (int64_t)row_q * p.ost + (int64_t)h * p.osh;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t* src = q < 4 ? t0 + q * 8 : t1 + (q - 4) * 8;
          uint4 wv;
          wv.x = pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
          wv.y = pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
          wv.z = pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
          wv.w = pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
          reinterpret_cast<uint4*>(orow)[q] = wv;
        }
        p.lse[(int64_t)it.bh * p.Tq + row_q] = m + log2f(l);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// 4-D bf16 map over a strided head view: dims {64 (d), H, T, B}, 64 x 1 x rows x 1
// boxes (`rows` rows of one head = one K-major 128B-swizzled tile).
bool make_head_map(CUtensorMap* tm, const HeadView& v, int H, int T, int B, int rows) {
  auto enc = attn_get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[4] = {64, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)v.sh * 2, (cuuint64_t)v.st * 2, (cuuint64_t)v.sb * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)rows, 1};
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

#ifdef G2B_ATTN_FWD_TRACE
unsigned long long* g_attn_fwd_trace = nullptr;  // set by a tracing harness
#endif

// Returns 1 if the tensor-core path ran, 0 if the caller must use the
// mma.sync kernel (layout not TMA-compatible), negative on launch failure.
// Streaming launches (a.peers) return -12 instead of 0 when a layout does not
// fit: they have no fallback kernel.
int attn_fwd_tc_launch(const AttnArgs& a, cudaStream_t s) {
  const bool stream = a.peers && a.peers->world > 0;
  const int no_fit = stream ? -12 : 0;
  if (!head_view_tma_ok(a.q)) return no_fit;
  if (!stream && (!head_view_tma_ok(a.k) || !head_view_tma_ok(a.v))) return 0;
  if ((a.o.sh * 2) % 16 || (a.o.st * 2) % 16 || (reinterpret_cast<uintptr_t>(a.o.base) & 15))
    return no_fit;
  const int Hkv = a.Hkv > 0 ? a.Hkv : a.H;
  if (Hkv > a.H || a.H % Hkv) return -1;
  CUtensorMap tq, tk, tv;
  if (!make_head_map(&tq, a.q, a.H, a.Tq, a.B, TQ)) return no_fit;
  KvPeerMaps peer_maps{};
  if (stream) {
    // key blocks never straddle two owners; tmK / tmV are not read
    if (a.Tk % TKV || !make_kv_peer_maps(&peer_maps, *a.peers, Hkv, a.B, TKV, attn_get_encode_fn()))
      return -12;
    tk = peer_maps.k[0];
    tv = peer_maps.v[0];
  } else if (!make_head_map(&tk, a.k, Hkv, a.Tk, a.B, TKV) ||
             !make_head_map(&tv, a.v, Hkv, a.Tk, a.B, TKV)) {
    return 0;
  }
  TcParams p;
  p.B = a.B;
  p.H = a.H;
  p.grp = a.H / Hkv;
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
#ifdef G2B_ATTN_FWD_TRACE
  p.trace = g_attn_fwd_trace;
#endif
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_fwd_tc_kernel<NoKvPeers>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(attn_fwd_tc_kernel<KvPeerMaps>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
      return -10;
    attr = true;
  }
  p.n_qpairs = (a.Tq + NG * TQ - 1) / (NG * TQ);
  p.n_items = p.n_qpairs * a.B * a.H;
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int grid = p.n_items < sms ? p.n_items : sms;  // persistent: one CTA per SM
  if (stream)
    attn_fwd_tc_kernel<KvPeerMaps><<<grid, kThreads, SMEM_BYTES, s>>>(tq, tk, tv, p, peer_maps);
  else
    attn_fwd_tc_kernel<NoKvPeers><<<grid, kThreads, SMEM_BYTES, s>>>(tq, tk, tv, p, NoKvPeers{});
  count_launches(1);
  return launch_succeeded() ? 1 : -11;
}

}  // namespace g2b
