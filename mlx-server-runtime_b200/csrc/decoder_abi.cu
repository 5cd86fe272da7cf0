// extern "C" entry points of the decoder-layer operators (declared in
// include/mlxq_b200.h): host-side validation, then one launch each.
#include <cmath>
#include <cstdio>

#include "../../include/mlxq_b200.h"
#include "decoder_ops.h"

namespace {

int fail(int code, const char* msg) { return mlxq::set_last_error(code, msg); }

int cuda_fail(cudaError_t e, const char* what) {
    char buf[256];
    snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
    return mlxq::set_last_error(MLXQ_ERR_CUDA, buf);
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool act_dtype(int dt) { return dt == MLXQ_BF16 || dt == MLXQ_F16; }

constexpr int64_t kIntMax = 0x7fffffffLL;

int check_heads(int Hq, int Hkv, int hd) {
    if (Hq <= 0 || Hkv <= 0 || Hq % Hkv || Hq / Hkv > 8)
        return fail(MLXQ_ERR_SHAPE, "heads: n_q_heads must be a multiple of n_kv_heads, at most "
                                    "8 query heads per kv head");
    if (hd != 64 && hd != 128) return fail(MLXQ_ERR_SHAPE, "head_dim must be 64 or 128");
    return MLXQ_OK;
}

int check_page(int page_size) {
    if (page_size != 8 && page_size != 16 && page_size != 32)
        return fail(MLXQ_ERR_SHAPE, "paged_attention: page_size must be 8, 16 or 32");
    return MLXQ_OK;
}

}  // namespace

extern "C" {

int mlxq_rms_norm(const void* x, const void* residual, const void* weight, void* out,
                  void* residual_out, int64_t rows, int64_t dim, float eps, int dtype,
                  void* stream) {
    if (!act_dtype(dtype)) return fail(MLXQ_ERR_DTYPE, "rms_norm: dtype must be bf16 or f16");
    if (rows < 0 || rows > kIntMax || dim <= 0 || dim % 8 || dim > 8192)
        return fail(MLXQ_ERR_SHAPE, "rms_norm: dim must be a multiple of 8 up to 8192");
    if (!x || !weight || !out) return fail(MLXQ_ERR_NULL, "rms_norm: NULL pointer");
    if (residual_out && !residual)
        return fail(MLXQ_ERR_NULL, "rms_norm: residual_out needs a residual");
    if (!a16(x) || !a16(weight) || !a16(out) || (residual && !a16(residual)) ||
        (residual_out && !a16(residual_out)))
        return fail(MLXQ_ERR_ALIGN, "rms_norm: pointers must be 16-byte aligned");
    if (!(eps >= 0.f)) return fail(MLXQ_ERR_SHAPE, "rms_norm: eps must be >= 0");
    if (rows == 0) return MLXQ_OK;
    cudaError_t e = mlxq::launch_rms_norm(dtype, x, residual, weight, out, residual_out,
                                          static_cast<int>(rows), static_cast<int>(dim), eps,
                                          mlxq::launch_overlap_enabled(),
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MLXQ_OK : cuda_fail(e, "rms_norm launch");
}

int mlxq_rope_kv_append(const void* qkv, int64_t ld, void* q_out, void* k_cache, void* v_cache,
                        const int32_t* positions, const int32_t* slots, int64_t tokens,
                        int n_q_heads, int n_kv_heads, int head_dim, float rope_base, int dtype,
                        void* stream) {
    if (!act_dtype(dtype)) return fail(MLXQ_ERR_DTYPE, "rope_kv_append: dtype must be bf16 or f16");
    int rc = check_heads(n_q_heads, n_kv_heads, head_dim);
    if (rc) return rc;
    if (tokens < 0 || tokens > kIntMax || ld < (n_q_heads + 2 * n_kv_heads) * head_dim ||
        ld % 8 || ld > kIntMax)
        return fail(MLXQ_ERR_SHAPE, "rope_kv_append: ld must hold q, k and v (a multiple of 8)");
    if (!(rope_base > 1.0f)) return fail(MLXQ_ERR_SHAPE, "rope_kv_append: rope_base must be > 1");
    if (!qkv || !q_out || !k_cache || !v_cache || !positions || !slots)
        return fail(MLXQ_ERR_NULL, "rope_kv_append: NULL pointer");
    if (!a16(qkv) || !a16(q_out) || !a16(k_cache) || !a16(v_cache))
        return fail(MLXQ_ERR_ALIGN, "rope_kv_append: pointers must be 16-byte aligned");
    if (tokens == 0) return MLXQ_OK;
    cudaError_t e = mlxq::launch_rope_append(
        dtype, qkv, static_cast<int>(ld), q_out, k_cache, v_cache, positions, slots,
        static_cast<int>(tokens), n_q_heads, n_kv_heads, head_dim,
        static_cast<float>(std::log2(static_cast<double>(rope_base))),
        mlxq::launch_overlap_enabled(), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MLXQ_OK : cuda_fail(e, "rope_kv_append launch");
}

size_t mlxq_paged_attention_workspace_size(int64_t batch, int n_kv_heads, int64_t max_kv_len,
                                           int head_dim) {
    if (batch <= 0 || n_kv_heads <= 0 || max_kv_len <= 0 || batch > kIntMax ||
        max_kv_len > kIntMax || (head_dim != 64 && head_dim != 128))
        return 0;
    return mlxq::attn_decode_workspace(static_cast<int>(batch), n_kv_heads,
                                       static_cast<int>(max_kv_len), head_dim);
}

int mlxq_paged_attention_decode(const void* q, const void* k_cache, const void* v_cache,
                                const int32_t* block_table, int64_t max_blocks,
                                const int32_t* kv_lens, int64_t max_kv_len, void* out,
                                int64_t batch, int n_q_heads, int n_kv_heads, int head_dim,
                                int page_size, float scale, int dtype, void* workspace,
                                size_t workspace_bytes, void* stream) {
    if (!act_dtype(dtype)) return fail(MLXQ_ERR_DTYPE, "paged_attention: dtype must be bf16 or f16");
    int rc = check_heads(n_q_heads, n_kv_heads, head_dim);
    if (rc || (rc = check_page(page_size))) return rc;
    if (batch < 0 || batch > 65535 || max_blocks <= 0 || max_blocks > kIntMax || max_kv_len <= 0 ||
        max_kv_len > max_blocks * page_size)
        return fail(MLXQ_ERR_SHAPE,
                    "paged_attention: max_kv_len must be in [1, max_blocks * page_size]");
    if (!q || !k_cache || !v_cache || !block_table || !kv_lens || !out)
        return fail(MLXQ_ERR_NULL, "paged_attention: NULL pointer");
    if (!a16(q) || !a16(k_cache) || !a16(v_cache) || !a16(out))
        return fail(MLXQ_ERR_ALIGN, "paged_attention: pointers must be 16-byte aligned");
    if (batch == 0) return MLXQ_OK;
    const size_t need = mlxq::attn_decode_workspace(static_cast<int>(batch), n_kv_heads,
                                                    static_cast<int>(max_kv_len), head_dim);
    if (need) {
        if (!workspace || workspace_bytes < need)
            return fail(MLXQ_ERR_WORKSPACE, "paged_attention: workspace missing or too small");
        if (reinterpret_cast<uintptr_t>(workspace) & 255u)
            return fail(MLXQ_ERR_ALIGN, "paged_attention: workspace must be 256-byte aligned");
    }
    cudaError_t e = mlxq::launch_attn_decode(
        dtype, q, k_cache, v_cache, block_table, static_cast<int>(max_blocks), kv_lens,
        static_cast<int>(max_kv_len), out, static_cast<int>(batch), n_q_heads, n_kv_heads,
        head_dim, page_size, scale, workspace, mlxq::launch_overlap_enabled(),
        static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MLXQ_OK : cuda_fail(e, "paged_attention_decode launch");
}

int mlxq_paged_attention_prefill(const void* q, const int32_t* cu_q, int64_t max_q_len,
                                 const void* k_cache, const void* v_cache,
                                 const int32_t* block_table, int64_t max_blocks,
                                 const int32_t* kv_lens, void* out, int64_t batch, int n_q_heads,
                                 int n_kv_heads, int head_dim, int page_size, float scale,
                                 int dtype, void* stream) {
    if (!act_dtype(dtype)) return fail(MLXQ_ERR_DTYPE, "paged_attention: dtype must be bf16 or f16");
    int rc = check_heads(n_q_heads, n_kv_heads, head_dim);
    if (rc || (rc = check_page(page_size))) return rc;
    if (batch < 0 || batch > 65535 || max_blocks <= 0 || max_blocks > kIntMax || max_q_len < 0 ||
        max_q_len > max_blocks * page_size)
        return fail(MLXQ_ERR_SHAPE, "paged_attention_prefill: bad batch, blocks or query length");
    if (!q || !cu_q || !k_cache || !v_cache || !block_table || !kv_lens || !out)
        return fail(MLXQ_ERR_NULL, "paged_attention_prefill: NULL pointer");
    if (!a16(q) || !a16(k_cache) || !a16(v_cache) || !a16(out))
        return fail(MLXQ_ERR_ALIGN, "paged_attention_prefill: pointers must be 16-byte aligned");
    if (batch == 0 || max_q_len == 0) return MLXQ_OK;
    cudaError_t e = mlxq::launch_attn_prefill(
        dtype, q, cu_q, static_cast<int>(max_q_len), k_cache, v_cache, block_table,
        static_cast<int>(max_blocks), kv_lens, out, static_cast<int>(batch), n_q_heads,
        n_kv_heads, head_dim, page_size, scale, mlxq::launch_overlap_enabled(),
        static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MLXQ_OK : cuda_fail(e, "paged_attention_prefill launch");
}

int mlxq_quantized_embedding(const int32_t* ids, int64_t n, const uint32_t* wq,
                             const void* scales, const void* biases, void* out, int64_t vocab,
                             int64_t dim, int group_size, int bits, int dtype, void* stream) {
    if (!act_dtype(dtype)) return fail(MLXQ_ERR_DTYPE, "quantized_embedding: dtype must be bf16 or f16");
    if (bits != 4 && bits != 8)
        return fail(MLXQ_ERR_UNSUPPORTED_BITS, "quantized_embedding: bits must be 4 or 8");
    if (group_size != 32 && group_size != 64 && group_size != 128)
        return fail(MLXQ_ERR_GROUP_SIZE, "quantized_embedding: group_size not in {32, 64, 128}");
    if (n < 0 || n > kIntMax || vocab <= 0 || vocab > kIntMax || dim <= 0 || dim > kIntMax ||
        dim % group_size)
        return fail(MLXQ_ERR_SHAPE, "quantized_embedding: bad n, vocab or dim");
    if (!ids || !wq || !scales || !biases || !out)
        return fail(MLXQ_ERR_NULL, "quantized_embedding: NULL pointer");
    if (!a16(wq) || !a16(out))
        return fail(MLXQ_ERR_ALIGN, "quantized_embedding: pointers must be 16-byte aligned");
    if (n == 0) return MLXQ_OK;
    cudaError_t e = mlxq::launch_embed(dtype, bits, ids, static_cast<int>(n), wq, scales, biases,
                                       out, static_cast<int>(vocab), static_cast<int>(dim),
                                       group_size, mlxq::launch_overlap_enabled(),
                                       static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MLXQ_OK : cuda_fail(e, "quantized_embedding launch");
}

int mlxq_moe_route(const void* logits, int logits_dtype, const float* expert_bias,
                   int32_t* indices, void* scores, int scores_dtype, int64_t tokens,
                   int num_experts, int top_k, int norm_topk_prob, void* stream) {
    auto ok_dt = [](int d) { return d == MLXQ_F32 || d == MLXQ_BF16 || d == MLXQ_F16; };
    if (!ok_dt(logits_dtype) || !ok_dt(scores_dtype))
        return fail(MLXQ_ERR_DTYPE, "moe_route: dtypes must be float32, bfloat16 or float16");
    if (tokens < 0 || tokens > kIntMax / 32 || num_experts < 1 || num_experts > 1024 ||
        top_k < 1 || top_k > 32 || top_k > num_experts)
        return fail(MLXQ_ERR_SHAPE, "moe_route: need 1 <= top_k <= min(32, num_experts), "
                                    "num_experts <= 1024");
    if (!logits || !indices || !scores) return fail(MLXQ_ERR_NULL, "moe_route: NULL pointer");
    if (tokens == 0) return MLXQ_OK;
    cudaError_t e = mlxq::launch_moe_route(logits_dtype, logits, expert_bias, indices,
                                           scores_dtype, scores, static_cast<int>(tokens),
                                           num_experts, top_k, norm_topk_prob ? 1 : 0,
                                           mlxq::launch_overlap_enabled(),
                                           static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MLXQ_OK : cuda_fail(e, "moe_route launch");
}

int mlxq_moe_sort(const int32_t* indices, int64_t n, int num_experts, int32_t* order,
                  int32_t* sorted_indices, int32_t* inverse, void* stream) {
    if (n < 0 || n > 16384 || num_experts < 1 || num_experts > 1024)
        return fail(MLXQ_ERR_SHAPE, "moe_sort: need n <= 16384 and 1 <= num_experts <= 1024");
    if (!indices || !order || !sorted_indices || !inverse)
        return fail(MLXQ_ERR_NULL, "moe_sort: NULL pointer");
    if (n == 0) return MLXQ_OK;
    cudaError_t e = mlxq::launch_moe_sort(indices, static_cast<int>(n), num_experts, order,
                                          sorted_indices, inverse,
                                          mlxq::launch_overlap_enabled(),
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MLXQ_OK : cuda_fail(e, "moe_sort launch");
}

int mlxq_decode_advance(int32_t* positions, int32_t* kv_lens, int32_t* slots,
                        const int32_t* block_table, int64_t max_blocks, int64_t batch,
                        int page_size, void* stream) {
    if (batch < 0 || batch > kIntMax || max_blocks <= 0 || max_blocks > kIntMax || page_size <= 0)
        return fail(MLXQ_ERR_SHAPE, "decode_advance: bad batch, blocks or page size");
    if (!positions || !kv_lens || !slots || !block_table)
        return fail(MLXQ_ERR_NULL, "decode_advance: NULL pointer");
    if (batch == 0) return MLXQ_OK;
    cudaError_t e = mlxq::launch_decode_advance(positions, kv_lens, slots, block_table,
                                                static_cast<int>(max_blocks),
                                                static_cast<int>(batch), page_size,
                                                mlxq::launch_overlap_enabled(),
                                                static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MLXQ_OK : cuda_fail(e, "decode_advance launch");
}

}  // extern "C"
