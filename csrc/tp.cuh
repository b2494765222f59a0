// Host-side interface of the tensor-/sequence-parallel kernels (csrc/tp.cu).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace g2b {

constexpr int kTpMaxRanks = 8;
constexpr int kTpMaxBlocks = 160;  // flag slots per (phase, rank)

// peer_bufs[q] is rank q's symmetric buffer of the operation (bf16 rows for
// the gather / reduce-scatter / embedding table, fp32 for the embedding
// gradient, fp32 [M, 4] statistics for the cross-entropy); peer_flags[q] is
// rank q's flag array ([2][kTpMaxRanks][kTpMaxBlocks] uint32).
struct TpArgs {
  void** peer_bufs = nullptr;
  uint32_t** peer_flags = nullptr;
  int rank = 0, world = 1;
  int64_t rows = 0;   // rows per rank (gather / reduce-scatter / embedding), all rows (CE)
  int cols = 0;       // row length in elements
  int nblocks = 64;
  uint32_t epoch = 1;
  // reduce-scatter epilogue
  const __nv_bfloat16* bias = nullptr;  // [cols] or null
  const float* resid = nullptr;         // fp32 [rows, cols] or null (embedding bwd: dx)
  float* out_f32 = nullptr;             // fp32 [rows, cols] (embedding: x / wpe grad)
  __nv_bfloat16* out_bf16 = nullptr;
  // embedding
  const int64_t* idx = nullptr;         // all M token ids (CE: targets)
  const __nv_bfloat16* wpe = nullptr;
  int T = 1;
  int64_t vocab_per_rank = 0;
  // cross-entropy
  __nv_bfloat16* logits = nullptr;      // [rows, ld] local vocabulary slice
  int64_t ld = 0;
  int vocab_valid = 0;                  // real (unpadded) columns of the slice
  int64_t vocab_start = 0;
  float* stats = nullptr;               // this rank's [rows, 4]
  float* loss_rows = nullptr;
  unsigned long long* byte_counter = nullptr;
  uint32_t* err = nullptr;
  int64_t wait_budget_ns = 2000000000ll;
  // context parallelism (cp_kv_gather / cp_kv_reduce): B sequences of
  // world * Tl tokens; this rank owns tokens [rank*Tl, (rank+1)*Tl) of each.
  // peer_bufs[q] is rank q's [B, world*Tl, 2C] bf16 key/value buffer; `src`
  // (gather) / `out_bf16` (reduce) is this rank's fused qkv [B*Tl, ld] whose
  // columns [C, 3C) hold k and v.
  const __nv_bfloat16* src = nullptr;
  int64_t src_ld = 0;
  int B = 0, Tl = 0;
  // Load-balanced (zig-zag) split: the sequence is 2*world chunks of Tl/2
  // tokens and rank r owns chunks r and 2*world-1-r, stored as the two
  // halves of each local sequence; the key/value buffers keep the natural
  // order. The reduce then reads two partial buffers per rank: peer_bufs
  // (queries of the first half) and peer_bufs2 (queries of the second half).
  int zigzag = 0;
  void** peer_bufs2 = nullptr;
  // Fused forms. pushed (gather): the rows were already stored into every
  // rank's buffer by the kernel that produced them (RowPush), so the gather
  // only synchronises. inbox (reduce-scatter): every rank's GEMM stored its
  // partial of this rank's rows into this rank's inbox, [world][rows][cols]
  // bf16 (slot = source rank), so the sum reads local memory only.
  int pushed = 0;
  const __nv_bfloat16* inbox = nullptr;
};

int tp_ag_rows_launch(TpArgs a, cudaStream_t s);
int tp_rs_rows_launch(TpArgs a, cudaStream_t s);
int tp_embed_fwd_launch(TpArgs a, cudaStream_t s);
int tp_embed_bwd_launch(TpArgs a, cudaStream_t s);
int tp_ce_stats_launch(TpArgs a, cudaStream_t s);
int tp_ce_finish_launch(TpArgs a, cudaStream_t s);

// Context parallelism, all-gather-KV form: copy this rank's k/v rows into its
// own block of the symmetric key/value buffer, then pull the blocks of every
// earlier rank (the only keys a causal query of this rank can see). `cols` = 2C.
// Zig-zag: own chunks to their natural rows, then every other chunk up to
// 2*world-1-rank from its owner.
int cp_kv_gather_launch(TpArgs a, cudaStream_t s);
// Streaming form: copy this rank's k/v rows (local order) into its compact
// [B, Tl, 2C] buffer peer_bufs[rank] and publish `epoch` into word `rank` of
// every peer's flag buffer (system-scope release, after all rows are fenced).
// The flag buffers here are the small publish buffers of kKvPublishWords
// words, not the handshake arrays above.
constexpr int kKvPublishCount = 8;                    // finished-CTA counter word
constexpr int kKvPublishWords = kKvPublishCount + 8;  // words per rank
int cp_kv_publish_launch(TpArgs a, cudaStream_t s);
// Reduce-scatter of the key/value gradients: this rank's block summed over
// ranks rank..world-1 (the ranks whose queries saw these keys), in rank
// order, into columns [C, 3C) of the local dqkv rows (out_bf16, ld).
// Zig-zag: each own chunk k summed over ranks q (ascending) of the first-half
// partials where k <= q and the second-half partials where k <= 2*world-1-q.
int cp_kv_reduce_launch(TpArgs a, cudaStream_t s);

}  // namespace g2b
