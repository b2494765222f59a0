// Host-side interface of the KV-cached decoding kernels (csrc/decode.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace g2b {

int decode_embed_launch(const int64_t* tok, const int* lens, const void* wte, const void* wpe, float* x,
                        int B, int C, cudaStream_t s);
int decode_attn_launch(const void* qkv, int64_t ld, void* kc, void* vc, const int* lens, float* part_o,
                       float* part_ml, void* out, int64_t ld_out, int B, int H, int Hkv, int Tmax,
                       float scale, cudaStream_t s);
int decode_partials_numel(int B, int H, int Tmax);
// Attention kernel of decode_attn_launch: 1 = one position a warp (default),
// 2 = four positions a warp on 16-byte vectors (query groups of up to 4
// heads; other shapes keep kernel 1).
void decode_set_impl(int impl);
int decode_get_impl();
int decode_argmax_launch(const void* logits, int64_t ld, int V, int64_t* tok, int* lens, int64_t* hist,
                         int Tmax, int B, cudaStream_t s);

}  // namespace g2b
