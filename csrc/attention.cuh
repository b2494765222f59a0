// Host-side interface of the causal flash-attention kernels (csrc/attention.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace g2b {

// Strided view of one of q/k/v/o/dq/dk/dv: element (b, h, t, d) lives at
//   base[b*sb + t*st + h*sh + d]   (d contiguous, head_dim == 64).
struct HeadView {
  void* base = nullptr;
  int64_t sb = 0, st = 0, sh = 0;
};

// Context-parallel keys and values read in place from their owners (the
// streaming form of the all-gather-KV attention). Rank q of the group keeps
// its own rows of every sequence in a symmetric buffer mapped into this
// process at base[q]: [B, Tl, 2C] bf16, keys in columns [0, C), values in
// [v_off, v_off + C). Key position k (natural order over the whole sequence)
// belongs to
//   contiguous split:  rank k / Tl, local row k % Tl;
//   zig-zag split:     chunk c = k / (Tl/2), rank c (c < world) or
//                      2*world-1-c, local row (c < world ? 0 : Tl/2) + k % (Tl/2).
// Before its first read from rank q a kernel waits (bounded) until
// flags[q] has reached `epoch`: rank q stores the epoch there with a system-
// scope release once its rows are in place (cp_kv_publish).
constexpr int kKvMaxOwners = 8;
struct KvPeers {
  int world = 0;            // 0: keys and values come from AttnArgs::k / v
  int zigzag = 0;
  int Tl = 0;               // rows per sequence in each owner's buffer
  void* base[kKvMaxOwners] = {};
  int64_t sb = 0, st = 0;   // element strides of an owner buffer (sequence, row)
  int64_t v_off = 0;        // element offset of the value columns
  const uint32_t* flags = nullptr;
  uint32_t epoch = 0;
};

struct AttnArgs {
  HeadView q, k, v, o;      // forward inputs / output (bf16)
  HeadView dout, dq, dk, dv;  // backward (bf16)
  float* lse = nullptr;     // [B, H, Tq] log2-domain row log-sum-exp (fp32)
  float* delta = nullptr;   // [B, H, Tq] rowsum(dO * O) scratch (fp32)
  int B = 0, H = 0, Tq = 0, Tk = 0;
  // Key/value heads (grouped-query / multi-query attention): query head h
  // reads key/value head h / (H / Hkv); 0 means Hkv = H. Grouped heads run on
  // the tensor-core kernels only.
  int Hkv = 0;
  int q_offset = 0;         // absolute position of query 0 (context parallel)
  int causal = 1;
  float scale = 0.125f;     // softmax scale (1/sqrt(head_dim))
  uint32_t* err = nullptr;
  // Set: keys and values are read from their owners (tensor-core kernels
  // only; k / v are ignored). Tk still counts natural key positions.
  const KvPeers* peers = nullptr;
};

int attn_fwd_launch(const AttnArgs& a, cudaStream_t s);

// Tensor-core (tcgen05) forward: 1 = ran, 0 = layout not TMA-compatible.
int attn_fwd_tc_launch(const AttnArgs& a, cudaStream_t s);

// Kernel selection for the forward: 0 = tensor cores when possible (default),
// 1 = always the mma.sync kernel (kept as a cross-check).
void attn_set_impl(int impl);
int attn_get_impl();
int attn_bwd_launch(const AttnArgs& a, cudaStream_t s);

// Tensor-core (tcgen05) backward, run after delta is computed: 1 = ran,
// 0 = layout not TMA-compatible.
int attn_bwd_tc_launch(const AttnArgs& a, cudaStream_t s);

}  // namespace g2b
