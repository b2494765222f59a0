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
