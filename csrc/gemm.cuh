// Host-side interface of the tcgen05 GEMM (csrc/gemm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace g2b {

// Epilogues fused into the GEMM. `acc` is the fp32 tile result, scaled by alpha
// (and by *alpha_ptr when given), `b` a bf16 bias broadcast along rows.
enum GemmEpilogue : int {
  EPI_BF16 = 0,        // out(bf16)  = acc + b
  EPI_BIAS_GELU = 1,   // aux(bf16)  = acc + b ; out(bf16) = gelu_tanh(acc + b)
  EPI_RESID_F32 = 2,   // out(fp32) = (aux or out)(fp32) + acc + b   (residual add)
  EPI_F32 = 3,         // out(fp32)  = acc (+ out if accumulate) ; split-K partials
  EPI_GELU_BWD = 4,    // out(bf16)  = acc * gelu_tanh'(aux)
  // Cross-entropy statistics (the lm_head forward): out(bf16) = acc (the
  // logits); for every row and every 128-column half of a 256-wide tile
  // column n_tile, ce_stats[(2 * n_tile + half) * M + row] = (max, sum exp(x -
  // max)) of that half's bf16-rounded logits below N; ce_tgt_logit[row] = the
  // bf16-rounded logit of column ce_targets[row] - ce_vocab_offset when this
  // launch covers it.
  EPI_CE_STATS = 5,
};

struct GemmArgs {
  // C[M,N] = A[M,K] * B[N,K]^T. A is K-major when a_mn_major == 0 (row m holds
  // K contiguous elements, stride lda), M-major otherwise (row k holds M
  // contiguous elements, stride lda). Same convention for B with N.
  const void* A = nullptr;
  const void* B = nullptr;
  int64_t lda = 0, ldb = 0;
  int a_mn_major = 0, b_mn_major = 0;
  int M = 0, N = 0, K = 0;
  int epilogue = EPI_BF16;
  void* out = nullptr;
  int64_t ldo = 0;
  void* aux = nullptr;
  int64_t ldaux = 0;
  const void* bias = nullptr;       // bf16 [N] or null
  const float* alpha_ptr = nullptr;  // optional device scalar multiplied into acc
  float alpha = 1.0f;
  int accumulate = 0;               // EPI_F32 only
  int splits = 1;                   // split-K count (EPI_F32 only)
  void* workspace = nullptr;        // fp32 [splits, M, N] when splits > 1
  int bn = 256;                     // tile N: 256 or 128
  int max_ctas = 0;                 // 0 = one CTA per SM
  int pair = -1;                    // 1: 256x256 tiles on CTA pairs (cta_group::2), 0: one
                                    // CTA per 128xbn tile, -1: library default
  uint32_t* err = nullptr;          // error word (device)
  // EPI_CE_STATS only
  void* ce_stats = nullptr;             // float2 [2 * ceil(N / 256), M]
  const int64_t* ce_targets = nullptr;  // int64 [M] (ignore_index -100 never matches)
  float* ce_tgt_logit = nullptr;        // fp32 [M]
  int ce_vocab_offset = 0;              // first vocabulary id of column 0
  // Row-owner output (tensor-parallel GEMM -> reduce-scatter): when set, row
  // m of the result is stored at owner_out[m / owner_rows] + (m % owner_rows)
  // * ldo -- device array of base addresses, typically in other GPUs' memory
  // (plain peer stores, one 16-byte vector at a time). bf16 epilogues only.
  void* const* owner_out = nullptr;
  int owner_rows = 0;
  int owner_self = -1;  // this GPU's index in owner_out: its rows keep the TMA-store path
};

// Returns 0 on success, a negative code for unsupported arguments.
int gemm_bf16_launch(const GemmArgs& args, cudaStream_t stream);

// Deterministic reduction of split-K partials: out[M,N] (+)= sum_s ws[s]
// (fp32; summed in split order).
int splitk_reduce_launch(const float* ws, int splits, int64_t split_stride, float* out,
                         int64_t ldo, int M, int N, int accumulate, cudaStream_t stream);

}  // namespace g2b
