/*
 * mlxq_b200.h -- C ABI of the B200 group-wise affine quantized matmul library
 * (libmlxq_b200.so, built from mlx-server-runtime_b200/csrc).
 *
 * The reference (huydt84/mlx-server-runtime) reaches these operators through
 * the third-party MLX package (mlx 0.31.2, python/uv.lock:939-940), whose
 * Python surface the model graphs call:
 *   mx.quantize          python/mlx_worker/native_mlx/models/lfm2.py:112-117,142-151
 *   nn.quantize          python/mlx_worker/native_mlx/models/qwen2.py:318-324
 *   QuantizedLinear      python/mlx_worker/native_mlx/models/qwen2.py:58-61,123-134,227
 *   mx.gather_qmm        python/mlx_worker/native_mlx/models/lfm2.py:176-187
 * Each entry point below replaces one of those operators; the ctypes shim in
 * mlx-server-runtime_b200/core.py binds them under MLX's names.
 *
 * Conventions
 *  - All pointers are DEVICE pointers to contiguous row-major buffers owned by
 *    the caller. The library allocates no device memory; kernels that need
 *    scratch space take a caller-provided workspace.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream). Every call is
 *    stream-ordered and asynchronous; errors detected on the host are returned
 *    before anything is enqueued.
 *  - Return value: MLXQ_OK (0) or a negative MLXQ_ERR_* code; the message of
 *    the last failure on the calling thread is available from mlxq_last_error().
 *    The library never aborts the process.
 *  - dtype codes: MLXQ_F32, MLXQ_BF16, MLXQ_F16.
 *  - Storage layout (MLX "affine" mode): w_q uint32 [rows, K*bits/32] with code
 *    k of a row at bits [bits*(k % (32/bits)), +bits) of word k/(32/bits);
 *    scales/biases [rows, K/group_size]; w ~= scale*q + bias.
 *  - Supported: bits in {4, 8} for the matmuls, {2, 4, 8} for quantize and
 *    dequantize; group_size in {32, 64, 128}; K a multiple of group_size.
 */
#ifndef MLXQ_B200_H
#define MLXQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLXQ_ABI_VERSION 1

enum {
    MLXQ_F32 = 0,
    MLXQ_BF16 = 1,
    MLXQ_F16 = 2,
};

enum {
    MLXQ_OK = 0,
    MLXQ_ERR_SHAPE = -1,            /* inconsistent or unsupported shape */
    MLXQ_ERR_DTYPE = -2,            /* unsupported dtype */
    MLXQ_ERR_ALIGN = -3,            /* pointer not 16-byte aligned */
    MLXQ_ERR_UNSUPPORTED_BITS = -4, /* bits not supported by this operator */
    MLXQ_ERR_GROUP_SIZE = -5,       /* group_size not in {32, 64, 128} */
    MLXQ_ERR_CUDA = -6,             /* a CUDA runtime call failed */
    MLXQ_ERR_WORKSPACE = -7,        /* workspace missing or too small */
    MLXQ_ERR_NULL = -8,             /* a required pointer is NULL */
    MLXQ_ERR_INDEX = -9,            /* index array argument invalid */
};

/* ABI version of the loaded library (MLXQ_ABI_VERSION at build time). */
int mlxq_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* mlxq_last_error(void);

/*
 * Launch overlap for quantized_matmul (process-wide, default off; returns the
 * previous setting). When on, each quantized_matmul is launched with CUDA
 * programmatic stream serialization: it may start streaming its packed weights,
 * scales and biases while the kernel before it on the stream is still running,
 * and waits for that kernel before reading activations or writing anything.
 * This hides the launch and ramp time between the back-to-back projections of
 * a decode step. Turn it on only when those weight buffers are not being
 * written by work still executing on the stream (the normal case: weights are
 * loaded once). No counterpart in the reference (MLX schedules its own graph).
 */
int mlxq_set_launch_overlap(int enable);
int mlxq_get_launch_overlap(void);

/*
 * Reads and clears the current device's kernel error code (0 = none). Kernels
 * that wait on hardware barriers give up after a bounded number of polls
 * instead of hanging; they then record a nonzero code here, skip their output
 * and exit. Synchronous (reads device memory). No counterpart in the reference.
 * A kernel that gave up may have left tickets of its workspace nonzero: after a
 * nonzero code, zero-fill every workspace passed to the matmuls again before
 * reusing it (the Python layer's device_error() does this for its workspaces).
 */
int mlxq_device_error(int* code);

/*
 * Failure-path check: enqueues one bounded mbarrier wait that nothing completes
 * (`polls` in [1, 2^22] polls), which gives up and records the timeout code (2) in
 * the device error word, as a kernel whose barrier never completed would. The
 * context stays usable. Lets a caller test its handling of mlxq_device_error
 * without any device fault. No counterpart in the reference.
 */
int mlxq_check_bounded_wait(uint32_t polls, void* stream);

/*
 * quantize: replaces mx.quantize(w, group_size, bits, mode="affine")
 * (lfm2.py:112-117) and the per-layer quantization nn.quantize performs
 * (qwen2.py:318-324). w [rows, K] of dtype w_dtype; writes wq
 * [rows, K*bits/32] uint32 and scales/biases [rows, K/group_size] in w_dtype.
 */
int mlxq_quantize(const void* w, int w_dtype, uint32_t* wq, void* scales, void* biases,
                  int64_t rows, int64_t K, int group_size, int bits, void* stream);

/*
 * dequantize: replaces mx.dequantize(w, scales, biases, group_size, bits)
 * (north_star API; MLX public op). out [rows, K] in `dtype` (the dtype of
 * scales/biases), each element round(round(scale*q) + bias).
 */
int mlxq_dequantize(const uint32_t* wq, const void* scales, const void* biases, int dtype,
                    void* out, int64_t rows, int64_t K, int group_size, int bits,
                    void* stream);

/*
 * Bytes of workspace mlxq_quantized_matmul needs for this problem (0 if none).
 * The workspace must be zero-filled once when first allocated; the kernels
 * leave it zeroed again at exit, so it can be reused by later calls on the
 * same stream without clearing. Calls that overlap on the GPU must not share it.
 * Decode shapes whose row blocks are split over CTAs need it for their partial
 * sums; prefill shapes whose whole tiles would leave much of the GPU idle (few
 * output tiles: the q/o, k/v and down projections at a few thousand tokens)
 * use it for stream-K partial tiles (about 29 MB on 148 SMs). A prefill call
 * given no workspace, or too small a one, runs whole tiles instead.
 */
size_t mlxq_qmm_workspace_size(int64_t M, int64_t N, int64_t K, int group_size, int bits,
                               int dtype);

/*
 * quantized_matmul: replaces mx.quantized_matmul(x, w, scales, biases,
 * transpose=True, group_size, bits) as called by nn.QuantizedLinear
 * (qwen2.py:58-61,123-134,227), plus QuantizedLinear's optional bias add.
 * Up to 32 rows of x use the decode kernels (HBM-bound); more rows with K a
 * multiple of 64 use the tcgen05 prefill kernel (weights dequantized into
 * tensor memory as the MMA's A operand, rounded once to the activation dtype,
 * fp32 accumulation).
 * x [M, K], w [N, K*bits/32], scales/biases [N, K/group_size], bias [N] or
 * NULL, out [M, N]; x/scales/biases/bias/out all of `dtype` (bf16 or f16).
 * out = round(x @ dequant(w)^T) with float32 accumulation; with bias,
 * round(out + bias).
 */
int mlxq_quantized_matmul(const void* x, const uint32_t* w, const void* scales,
                          const void* biases, const void* bias, void* out, int64_t M,
                          int64_t N, int64_t K, int group_size, int bits, int dtype,
                          void* workspace, size_t workspace_bytes, void* stream);

/*
 * gather_qmm: replaces mx.gather_qmm(x, w, scales, biases, lhs_indices,
 * rhs_indices, transpose=True, group_size, bits, sorted_indices) as called by
 * QuantizedSwitchLinear (lfm2.py:169-190).
 *   x      [x_batches, M, K]
 *   w      [num_experts, N, K*bits/32]; scales/biases [num_experts, N, K/group_size]
 *   out    [batch, M, N], out[b] = x[xi(b)] @ dequant(w[rhs_indices[b]])^T
 *   xi(b)  = lhs_indices ? lhs_indices[b] : b / lhs_div   (lhs_div >= 1; the
 *            broadcast of x [T,1,1,K] against indices [T,k] is lhs_div = k)
 * sorted_indices != 0 promises rhs_indices is non-decreasing (MLX's hint); the
 * kernels then stream each expert's weights once for all its rows. Results
 * do not depend on the flag when the promise holds. Rows whose indices are out
 * of range are left unwritten.
 */
int mlxq_gather_qmm(const void* x, const uint32_t* w, const void* scales, const void* biases,
                    const int32_t* lhs_indices, int64_t lhs_div, const int32_t* rhs_indices,
                    void* out, int64_t batch, int64_t M, int64_t N, int64_t K,
                    int64_t num_experts, int64_t x_batches, int group_size, int bits,
                    int dtype, int sorted_indices, void* workspace, size_t workspace_bytes,
                    void* stream);

/*
 * gather_qmm with the SwiGLU activation in the epilogue, for the decode sizes of an
 * MoE layer: w, scales, biases hold every expert's gate and up projections interleaved
 * by 16-row tiles (tile j = gate rows 8j..8j+7, then up rows 8j..8j+7; N = 2 * the
 * hidden size, a multiple of 16), and out [batch, M, N/2] receives silu(gate) * up,
 * each projection rounded to dtype first (as SwitchGLU's separate up_proj, gate_proj
 * and element-wise ops compute it, lfm2.py:202-218). Other arguments as
 * mlxq_gather_qmm: decode sizes run the grouped decode kernel's epilogue (no workspace
 * used), sorted batches with enough rows per expert the grouped tensor-core kernel's
 * (workspace as mlxq_gather_qmm_workspace_size). MLXQ_ERR_SHAPE when neither takes the
 * shape: mlxq_gather_swiglu_supported says which do (lhs_given: lhs_indices will be
 * passed).
 */
int mlxq_gather_swiglu_supported(int64_t batch, int64_t M, int64_t N, int64_t K,
                                 int64_t num_experts, int64_t x_batches, int group_size, int bits,
                                 int dtype, int lhs_given, int sorted_indices);
int mlxq_gather_qmm_swiglu(const void* x, const uint32_t* w, const void* scales,
                           const void* biases, const int32_t* lhs_indices, int64_t lhs_div,
                           const int32_t* rhs_indices, void* out, int64_t batch, int64_t M,
                           int64_t N, int64_t K, int64_t num_experts, int64_t x_batches,
                           int group_size, int bits, int dtype, int sorted_indices,
                           void* workspace, size_t workspace_bytes, void* stream);

/*
 * quantized_matmul_argmax: greedy decoding's next token without the logits. The
 * reference computes the vocabulary logits with the lm_head (or the tied
 * embedding's as_linear) quantized_matmul, then takes their argmax per sequence
 * (qwen2.py:225-227, executor.py:406-414). Here each logit is rounded to `dtype`
 * (plus bias) exactly as mlxq_quantized_matmul would write it, and ids[t] (int32,
 * t < M) receives the index of the largest, the first one on ties. Decode shapes
 * only (M <= 16, K/group_size a multiple of 8). The workspace
 * (mlxq_argmax_workspace_size bytes, at least 64 KiB, zero-filled once) is left
 * zeroed again, like mlxq_quantized_matmul's; calls that overlap on the GPU must
 * not share it.
 */
size_t mlxq_argmax_workspace_size(int64_t M, int64_t N, int64_t K, int group_size, int bits,
                                  int dtype);
int mlxq_quantized_matmul_argmax(const void* x, const uint32_t* w, const void* scales,
                                 const void* biases, const void* bias, int32_t* ids, int64_t M,
                                 int64_t N, int64_t K, int group_size, int bits, int dtype,
                                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * quantized_matmul_swiglu: the gate and up projections of a SwiGLU MLP and the
 * activation between them, silu(gate_proj(x)) * up_proj(x), in one launch.
 * The reference computes it as two quantized_matmul calls, a silu and a multiply
 * (qwen2.py:133-134, lfm2.py:212).
 * w / scales / biases hold the gate and up matrices interleaved by 16-row tiles:
 * tile j = gate rows 8j..8j+7 then up rows 8j..8j+7 (quantized rows copied as they
 * are; mlx_server_runtime_b200.interleave_gate_up builds it). N = 2 * intermediate
 * (a multiple of 16); out [M, N/2] = silu(g) * u with g, u each rounded to `dtype`
 * first, as the two separate matmuls would be. Decode shapes (M <= 16, K/group_size
 * a multiple of 8) run the decode kernel's epilogue (workspace as
 * mlxq_qmm_workspace_size(M, N, K, ...)); prefill shapes (M > 32, K a multiple of 64)
 * the tensor-core kernel's, whole tiles, no workspace. mlxq_swiglu_supported says
 * which shapes one of them takes.
 */
int mlxq_swiglu_supported(int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype);
int mlxq_quantized_matmul_swiglu(const void* x, const uint32_t* w, const void* scales,
                                 const void* biases, void* out, int64_t M, int64_t N, int64_t K,
                                 int group_size, int bits, int dtype, void* workspace,
                                 size_t workspace_bytes, void* stream);

/*
 * quantized_matmul_noalloc: the same operation as mlxq_quantized_matmul, for
 * callers that cannot allocate device memory -- a host that binds this C ABI
 * without a device allocator of its own, or a plugin inside a serving engine
 * whose memory manager owns all device memory and where a cudaMalloc in the
 * middle of a decode step may synchronize the device. It takes no workspace:
 * the K-split scratch is a fixed MLXQ_NOALLOC_SCRATCH_BYTES (2 MiB) array
 * compiled into the library, held by every GPU that loads the library until the
 * process exits. Shapes whose scratch need exceeds it return MLXQ_ERR_WORKSPACE
 * with the required size. The first call on a device looks up the array's
 * device address and sets kernel attributes; make that first call before any
 * stream capture. All calls share the one array: calls that overlap on the GPU
 * (different streams, or concurrent host threads) race and must be serialized
 * by the caller. It calls no cudaMalloc, cudaFree or allocating routine.
 * No counterpart in the reference (MLX allocates its own buffers).
 */
#define MLXQ_NOALLOC_SCRATCH_BYTES (2u * 1024u * 1024u)
int mlxq_quantized_matmul_noalloc(const void* x, const uint32_t* w, const void* scales,
                                  const void* biases, const void* bias, void* out, int64_t M,
                                  int64_t N, int64_t K, int group_size, int bits, int dtype,
                                  void* stream);

/*
 * Bytes of workspace mlxq_gather_qmm needs (the per-expert segment table of
 * the sorted path; 0 when sorted_indices == 0). No zero-fill is required.
 */
size_t mlxq_gather_qmm_workspace_size(int64_t batch, int64_t M, int64_t N, int64_t K,
                                      int64_t num_experts, int group_size, int bits, int dtype,
                                      int sorted_indices);


/* ---------------------------------------------------------------------------------
 * Decoder-layer operators around the projections (the row after the matmul on
 * either side of it in every layer of the reference's Qwen2-style graphs). The
 * same conventions hold; with launch overlap on they take part in it like the
 * matmuls (they wait for the previous kernel before reading its outputs).
 * dtype: MLXQ_BF16 or MLXQ_F16 for every activation, weight and cache buffer.
 */

/*
 * RMSNorm: replaces nn.RMSNorm (models/qwen2.py:144-147,161-165, mx.fast.rms_norm).
 * h = x, or with `residual` h = round(x + residual) (written to residual_out when
 * not NULL: the decoder block's `hidden = x + attn_out`, qwen2.py:161-165);
 * out = round(round(h * rsqrt(mean(h^2) + eps)) * weight) per row of `dim` (a
 * multiple of 8, at most 8192).
 */
int mlxq_rms_norm(const void* x, const void* residual, const void* weight, void* out,
                  void* residual_out, int64_t rows, int64_t dim, float eps, int dtype,
                  void* stream);

/*
 * RoPE and the paged KV append: replaces the two mx.fast.rope calls of
 * Qwen2Attention (qwen2.py:91-105, traditional=False) and the cache staging of
 * PagedBatchReservation.stage_layer (cache.py:485-520). qkv [tokens, ld] holds each
 * token's q (n_q_heads * head_dim), k and v (n_kv_heads * head_dim each), as the
 * fused q/k/v projection writes them. Writes the rotated queries to q_out
 * [tokens, n_q_heads, head_dim]; the rotated keys and the values to row slots[t]
 * of k_cache / v_cache, pools of [pages * page_size, n_kv_heads, head_dim] (the
 * reference's [pages, page_size, kv_heads, head_dim] layout); a negative slot
 * skips the append. Angle of pair i at position p: p * rope_base^(-2i/head_dim).
 */
int mlxq_rope_kv_append(const void* qkv, int64_t ld, void* q_out, void* k_cache, void* v_cache,
                        const int32_t* positions, const int32_t* slots, int64_t tokens,
                        int n_q_heads, int n_kv_heads, int head_dim, float rope_base, int dtype,
                        void* stream);

/*
 * Paged attention: replaces PagedLayerAttentionContext.append_and_attend's SDPA
 * over the sequence's pages (attention.py:215-298, mask from _dense_causal_mask,
 * attention.py:404-427): softmax(q k^T * scale + causal mask) v per query head,
 * the kv head being q_head / (n_q_heads / n_kv_heads). block_table [batch,
 * max_blocks] holds each sequence's page ids; kv_lens[b] = keys cached for
 * sequence b, the new ones included. head_dim 64 or 128, page_size 8, 16 or 32.
 *
 * decode: one query per sequence, q [batch, n_q_heads, head_dim] at position
 * kv_lens[b] - 1, attending every cached key; max_kv_len bounds kv_lens and sizes
 * the launch. The workspace (mlxq_paged_attention_workspace_size bytes, 256-byte
 * aligned, zero-filled once; the kernel leaves it zeroed) holds the partial results
 * of sequences longer than 128 keys; calls that overlap on the GPU must not share it.
 */
size_t mlxq_paged_attention_workspace_size(int64_t batch, int n_kv_heads, int64_t max_kv_len,
                                           int head_dim);
int mlxq_paged_attention_decode(const void* q, const void* k_cache, const void* v_cache,
                                const int32_t* block_table, int64_t max_blocks,
                                const int32_t* kv_lens, int64_t max_kv_len, void* out,
                                int64_t batch, int n_q_heads, int n_kv_heads, int head_dim,
                                int page_size, float scale, int dtype, void* workspace,
                                size_t workspace_bytes, void* stream);

/*
 * prefill: the new tokens of every sequence, q [total, n_q_heads, head_dim] with
 * sequence b's queries at rows [cu_q[b], cu_q[b+1]) (cu_q [batch + 1], at most
 * max_q_len per sequence); query i of sequence b sits at position
 * kv_lens[b] - (cu_q[b+1] - cu_q[b]) + i and attends the keys at or before it
 * (chunked prefill over an existing cache included). out like q.
 */
int mlxq_paged_attention_prefill(const void* q, const int32_t* cu_q, int64_t max_q_len,
                                 const void* k_cache, const void* v_cache,
                                 const int32_t* block_table, int64_t max_blocks,
                                 const int32_t* kv_lens, void* out, int64_t batch, int n_q_heads,
                                 int n_kv_heads, int head_dim, int page_size, float scale,
                                 int dtype, void* stream);

/*
 * Quantized embedding lookup: replaces QuantizedEmbedding.__call__ (embed_tokens,
 * qwen2.py:185, once nn.quantize has converted the table): out [n, dim] row i =
 * dequantize(row ids[i] of wq / scales / biases), bit-identical to mlxq_dequantize
 * of that row; ids outside [0, vocab) give zero rows.
 */
int mlxq_quantized_embedding(const int32_t* ids, int64_t n, const uint32_t* wq,
                             const void* scales, const void* biases, void* out, int64_t vocab,
                             int64_t dim, int group_size, int bits, int dtype, void* stream);

/*
 * MoE routing: replaces the router of Lfm2MoE.__call__ (lfm2.py:366-375):
 * gates = softmax(logits as float32) (+ expert_bias [num_experts] float32 when not
 * NULL), the top_k experts per token and their gates, renormalised to sum to one
 * (with the reference's + 1e-20) when norm_topk_prob, written as indices [tokens,
 * top_k] int32 and scores [tokens, top_k] of scores_dtype. The reference takes an
 * argpartition, whose order within the k is unspecified; here experts come in
 * descending gate order, the lower index first on ties. num_experts <= 1024,
 * top_k <= 32. Logits of any float dtype.
 */
int mlxq_moe_route(const void* logits, int logits_dtype, const float* expert_bias,
                   int32_t* indices, void* scores, int scores_dtype, int64_t tokens,
                   int num_experts, int top_k, int norm_topk_prob, void* stream);

/*
 * Stable sort of MoE routing entries by expert: replaces the argsort pair of the
 * sorted SwitchGLU path (_gather_sort, lfm2.py:613-618: order = argsort(indices),
 * inv_order = argsort(order)). For entries i < n with expert indices[i]:
 * order[p] = the entry at sorted position p (equal experts keep entry order),
 * sorted_indices[p] = indices[order[p]], inverse[i] = the sorted position of entry i.
 * Negative values form one group before every expert and values >= num_experts one
 * after, each in entry order (argsort would also order them by value).
 * n <= 16384, num_experts <= 1024. One launch, nothing read back to the host.
 */
int mlxq_moe_sort(const int32_t* indices, int64_t n, int num_experts, int32_t* order,
                  int32_t* sorted_indices, int32_t* inverse, void* stream);

/*
 * Decode-loop bookkeeping on the device, so a captured decode step replays with no
 * host work: for each sequence, positions[b] += 1, kv_lens[b] = positions[b] + 1,
 * slots[b] = that position's cache row from block_table (-1 past its end). The
 * reference's executor gathers the cache lengths on the host before every step
 * (executor.py:272-293).
 */
int mlxq_decode_advance(int32_t* positions, int32_t* kv_lens, int32_t* slots,
                        const int32_t* block_table, int64_t max_blocks, int64_t batch,
                        int page_size, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MLXQ_B200_H */
