// Host-side interface of the memory-bound kernels: LayerNorm, embedding,
// column reductions, cross-entropy, AdamW and gradient-norm clipping.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace g2b {

// Rows a kernel also stores into other GPUs' copies of its output buffer
// (tensor parallelism pushes each rank's LayerNorm rows to every peer): the
// row at address p in the local buffer goes to bases[j] + (p - local) too.
struct RowPush {
  void* const* bases = nullptr;  // device array of n peer base addresses
  int n = 0;
  const void* local = nullptr;   // local base the offsets are taken from
};


// LayerNorm over rows of an fp32 residual stream x[M, C] (row stride ldx) with
// bf16 gamma/beta; writes bf16 y (row stride ldy) and fp32 mean/rstd [M].
int layernorm_fwd_launch(const float* x, int64_t ldx, const void* gamma, const void* beta,
                         void* y, int64_t ldy, float* mean, float* rstd, int M, int C, float eps,
                         cudaStream_t s, RowPush push = RowPush());

// LayerNorm backward. dy bf16 [M,C]; x fp32; writes/accumulates the fp32
// residual gradient dres[M,C] (dres = (accumulate ? dres : 0) + dx) and its bf16
// copy dres_bf16 (may be null); dgamma/dbeta (+)= their column sums
// (acc_params) and, when dsum is non-null, dsum (+)= the column sum of the
// written dres (acc_sum) -- the bias gradient of the projection that produced
// this residual stream. `partials` is scratch of
// layernorm_bwd_partial_rows(M) * 3 * C floats. Two launches, deterministic.
int layernorm_bwd_launch(const void* dy, const float* x, const float* mean, const float* rstd,
                         const void* gamma, float* dres, void* dres_bf16, float* partials,
                         float* dgamma, float* dbeta, float* dsum, int M, int C, int accumulate,
                         int acc_params, int acc_sum, cudaStream_t s, RowPush push = RowPush());
int layernorm_bwd_partial_rows(int M);

// out[c] (+)= sum_r in[r, c] for fp32 in[R, C] (deterministic, row order).
int colsum_f32_launch(const float* in, int R, int C, float* out, int accumulate, cudaStream_t s);

// Bias gradient: out[c] (+)= sum_m in[m, c] for bf16 in[M, C] (row stride ld),
// deterministic two-stage (partials in `ws`, >= ceil(M/128)*C floats).
int colsum_bf16_launch(const void* in, int64_t ld, int M, int C, float* ws, float* out,
                       int accumulate, cudaStream_t s);

// x[b*T+t, :] = wte[idx[b,t]] + wpe[pos(t)]   (bf16 tables, fp32 out), with
// pos(t) = pos0 + t for t < split and pos1 + (t - split) from there on
// (split = T: one contiguous range).
int embedding_fwd_launch(const int64_t* idx, const void* wte, const void* wpe, float* x, int B,
                         int T, int C, int pos0, int split, int pos1, cudaStream_t s);

// Embedding backward: wte_grad[idx[m]] += dx[m] (fp32 atomics), and
// wpe_grad[pos(t)] (+)= sum_b dx[b*T+t] (deterministic; pos as above).
// With det_part (fp32 [B*T, C]) and det_slots (int32 [embedding_wte_det_chunks(B*T), V],
// all -1 before the first call, left so by every call) the token-embedding
// gradient is summed in a fixed order (bit-reproducible); without, by fp32
// atomics.
int embedding_bwd_launch(const int64_t* idx, const float* dx, float* wte_grad, float* wpe_grad,
                         int B, int T, int C, int V, int pos0, int split, int pos1, cudaStream_t s,
                         float* det_part = nullptr, int* det_slots = nullptr);
int embedding_wte_det_chunks(int64_t M);

// Cross-entropy over bf16 logits [M, V] (row stride ld) against int64 targets
// (ignore_index -100). Writes loss_rows[M] (0 for ignored rows) and overwrites
// the logits in place with dlogits = softmax - onehot (0 rows for ignored
// targets), unscaled. Columns in [V, ld) are zeroed.
int cross_entropy_fwd_bwd_launch(void* logits, int64_t ld, const int64_t* targets,
                                 float* loss_rows, int M, int V, int vocab_offset,
                                 cudaStream_t s);

// loss_out[0] = sum(loss_rows)/count ; loss_out[1] = 1/count (count = non-ignored
// targets, clamped to >= 1); deterministic single-block reduction.
// Fused lm_head + cross-entropy (after the EPI_CE_STATS GEMM): per-row
// log-sum-exp and loss from the GEMM's partials, then the in-place gradient
// logits -> softmax - onehot (0 for ignored rows and padded columns).
int ce_combine_launch(const void* stats, int nparts, int M, const int64_t* targets,
                      const float* tgt_logit, float* lse, float* loss_rows, cudaStream_t s);
int ce_grad_launch(void* logits, int64_t ld, int M, int V, const float* lse,
                   const int64_t* targets, int vocab_offset, cudaStream_t s);

// exp2_fma (the FMA-pipe 2^x of the softmax kernels) over n floats; tests only.
int exp2_fma_test_launch(const float* x, float* y, int n, cudaStream_t s);

int loss_reduce_launch(const float* loss_rows, const int64_t* targets, int M, float* loss_out,
                       cudaStream_t s);

// Fused AdamW over flat fp32 buffers, torch _single_tensor_adamw order.
// hp (device): [0]=lr [1]=beta1 [2]=beta2 [3]=eps [4]=weight_decay
//              [5]=bias_correction1 [6]=sqrt(bias_correction2) [7]=grad scale
// clip (device, optional): multiplier on the gradient (global-norm clip).
// Weight decay applies to elements inside the sorted, disjoint, 4-aligned
// ranges table [lo0, hi0, lo1, hi1, ...] (nr ranges, device memory); with a
// null table it applies to elements [0, n_decay).
int adamw_launch(float* p, const float* g, float* m, float* v, void* p_bf16, int64_t n,
                 int64_t n_decay, const int64_t* ranges, int nr, const float* hp,
                 const float* clip, cudaStream_t s);

// Sum of squares of fp32 g[n] into out[0] (deterministic two-stage, ws >= 1024).
int sumsq_launch(const float* g, int64_t n, float* ws, float* out, cudaStream_t s);

// clip[0] = min(1, max_norm / (sqrt(sumsq[0]*scale2) + 1e-6)); norm_out[0] = norm.
int clip_coef_launch(const float* sumsq, float scale2, float max_norm, float* clip,
                     float* norm_out, cudaStream_t s);

// Casts and simple elementwise helpers.
int cast_f32_bf16_launch(const float* in, void* out, int64_t n, cudaStream_t s);
int cast_bf16_f32_launch(const void* in, float* out, int64_t n, cudaStream_t s);
int scale_f32_launch(float* x, int64_t n, float a, cudaStream_t s);

}  // namespace g2b
