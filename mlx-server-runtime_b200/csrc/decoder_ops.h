// Launchers of the decoder-layer operators (decoder_ops.cu): RMSNorm, RoPE with the
// paged KV append, paged attention, the quantized embedding lookup and the per-step
// position advance of a decode loop.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "launch.h"

namespace mlxq {

cudaError_t launch_rms_norm(int dtype, const void* x, const void* delta, const void* w, void* y,
                            void* sum_out, int rows, int D, float eps, bool overlap,
                            cudaStream_t st);
cudaError_t launch_rope_append(int dtype, const void* qkv, int ld, void* q_out, void* k_cache,
                               void* v_cache, const int32_t* positions, const int32_t* slots,
                               int tokens, int Hq, int Hkv, int hd, float log2_base, bool overlap,
                               cudaStream_t st);
size_t attn_decode_workspace(int B, int Hkv, int max_kv_len, int head_dim);
cudaError_t launch_attn_decode(int dtype, const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* block_table, int max_blocks, const int32_t* kv_lens,
                               int max_kv_len, void* out, int B, int Hq, int Hkv, int hd, int page,
                               float scale, void* workspace, bool overlap, cudaStream_t st);
size_t attn_prefill_smem(int hd);
cudaError_t launch_attn_prefill(int dtype, const void* q, const int32_t* cu_q, int max_q_len,
                                const void* k_cache, const void* v_cache,
                                const int32_t* block_table, int max_blocks,
                                const int32_t* kv_lens, void* out, int B, int Hq, int Hkv, int hd,
                                int page, float scale, bool overlap, cudaStream_t st);
cudaError_t launch_embed(int dtype, int bits, const int32_t* ids, int n, const uint32_t* wq,
                         const void* scales, const void* biases, void* out, int vocab, int K,
                         int gs, bool overlap, cudaStream_t st);
cudaError_t launch_moe_route(int logits_dtype, const void* logits, const float* bias,
                             int32_t* indices, int scores_dtype, void* scores, int T, int E, int K,
                             int norm, bool overlap, cudaStream_t st);
size_t moe_sort_smem(int n, int E);
cudaError_t launch_moe_sort(const int32_t* idx, int n, int E, int32_t* order, int32_t* sorted,
                            int32_t* inverse, bool overlap, cudaStream_t st);
cudaError_t launch_decode_advance(int32_t* positions, int32_t* kv_lens, int32_t* slots,
                                  const int32_t* block_table, int max_blocks, int B, int page,
                                  bool overlap, cudaStream_t st);

}  // namespace mlxq
