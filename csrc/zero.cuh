// Host-side interface of the fused ZeRO-2 kernels (csrc/zero.cu).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "comm.cuh"

namespace g2b {

constexpr int kZeroMaxBlocks = 160;  // flag / norm slots per (phase, rank)

// Arguments shared by both kernels. Every rank owns symmetric gradient (fp32)
// and parameter (bf16) buffers over the same flat layout, a flag array
// ([2][kCommMaxRanks][kZeroMaxBlocks] uint32) and a norm-slot array
// ([2][kZeroMaxBlocks][kCommMaxRanks] uint64); peer_*[q] is rank q's buffer
// mapped into this process. buckets is a device int64 table [nb][4] of
// {lo, hi, slice, shard_offset}.
struct ZeroArgs {
  float** peer_grad = nullptr;
  // zero_rs with a bf16 wire: when set, the ranks' gradients are read from
  // these bf16 copies (same offsets as peer_grad) instead, summed in fp32
  __nv_bfloat16** peer_grad16 = nullptr;
  __nv_bfloat16** peer_shadow = nullptr;
  uint32_t** peer_flags = nullptr;
  unsigned long long** peer_norm = nullptr;
  int rank = 0, world = 1;
  const int64_t* buckets = nullptr;
  int nb = 0;
  int bucket = 0;          // zero_rs: the bucket to reduce
  int rs_blocks = 64;      // grid of every zero_rs launch (partials layout)
  float* gsh = nullptr;    // averaged gradient shard (local)
  float* master = nullptr;
  float* exp_avg = nullptr;
  float* exp_avg_sq = nullptr;
  float* sumsq_parts = nullptr;  // [nb][rs_blocks]
  const int64_t* decay_ranges = nullptr;  // flat [lo, hi) pairs, sorted
  int nr = 0;
  const float* hp = nullptr;  // lr, beta1, beta2, eps, wd, bc1, sqrt(bc2), grad scale
  float max_norm = 0.f;       // <= 0: no clipping
  float scale = 1.f;          // 1/p applied in the reduce-scatter
  uint32_t epoch = 1;         // strictly increasing per launch, same on every rank, >= 1
  unsigned long long* byte_counter = nullptr;
  float* norm_out = nullptr;
  uint32_t* err = nullptr;
  int64_t wait_budget_ns = 2000000000ll;
  // zero_rs: end with a second handshake so that on exit every peer has
  // finished reading this rank's gradient buffer (ZeRO-3 reuses it at once).
  int done_handshake = 0;
  // zero_ag (ZeRO-3 parameter gather): peer_shard[q] is rank q's bf16 shard
  // storage; the unit's slices are gathered into gather_dst[0, span).
  __nv_bfloat16** peer_shard = nullptr;
  __nv_bfloat16* gather_dst = nullptr;
  int64_t ag_span = 0, ag_slice = 0, ag_offset = 0;
};

int zero_rs_launch(const ZeroArgs& a, cudaStream_t s);
int zero_adamw_ag_launch(const ZeroArgs& a, int nblocks, cudaStream_t s);

// ZeRO-3 all-gather of one unit: gather_dst[e] = shard of rank e / ag_slice at
// ag_offset + e % ag_slice, for e in [0, ag_span), by P2P loads (16-byte
// vectors; ag_slice and ag_span multiples of 64). Starts with a handshake so
// that every peer's previous optimiser step has finished writing its shard.
int zero_ag_launch(const ZeroArgs& a, int nblocks, cudaStream_t s);

}  // namespace g2b
