// The decoder-layer operators around the quantized projections (sm_100a):
// RMSNorm with a fused residual add, RoPE with the paged KV-cache append,
// attention over the paged cache (decode and prefill forms), the quantized
// embedding lookup, and the position advance of a decode loop.
//
// Reference (huydt84/mlx-server-runtime, python/mlx_worker/native_mlx/):
//   RMSNorm           models/qwen2.py:144-147,161-165 (nn.RMSNorm, eps 1e-6)
//   RoPE              models/qwen2.py:91-105 (mx.fast.rope, traditional=False, base 1e6)
//   KV append         cache.py:485-520 (PagedBatchReservation.stage_layer: new keys and
//                     values written to their slots of the [pages, page_size, kv_heads,
//                     head_dim] pools)
//   attention         attention.py:215-298 (append_and_attend: SDPA over the sequence's
//                     pages with a causal mask offset by the cached length)
//   embedding         models/qwen2.py:185 (embed_tokens(inputs), a QuantizedEmbedding
//                     once nn.quantize has run)
//
// Every kernel here takes part in launch overlap the way the matmuls do: it lets
// the next kernel on the stream start at once (griddepcontrol.launch_dependents)
// and waits for the previous one (griddepcontrol.wait) before it reads anything
// that kernel may have written. Launched without the overlap attribute, both
// instructions are no-ops.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "decoder_ops.h"
#include "sm100.cuh"

namespace mlxq {

namespace {

__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
    return make_float2(Elem<T>::lo(u), Elem<T>::hi(u));
}

template <typename T>
__device__ __forceinline__ uint16_t bits16(T v) {
    return *reinterpret_cast<const uint16_t*>(&v);
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    return static_cast<uint32_t>(bits16(Elem<T>::from_f(a))) |
           (static_cast<uint32_t>(bits16(Elem<T>::from_f(b))) << 16);
}

template <typename T>
__device__ __forceinline__ float round_t(float v) {
    return Elem<T>::to_f(Elem<T>::from_f(v));
}

// Launch with the overlap attribute when asked; the kernel's carveout is set to the
// whole shared-memory capacity once per device (see ensure_smem_attr).
cudaError_t launch_ex(const void* func, PerDevice& cache, dim3 grid, dim3 block, size_t smem,
                      cudaStream_t st, bool overlap, void** args) {
    int dev = 0;
    cudaError_t e = current_device(&dev);
    if (e != cudaSuccess) return e;
    e = ensure_smem_attr(func, cache, dev, smem > 0 ? static_cast<int>(smem) : 1);
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = overlap ? attr : nullptr;
    cfg.numAttrs = overlap ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, func, args);
}

}  // namespace

// ------------------------------------------------------------------------------------
// RMSNorm: h = x (+ delta, rounded to T, written to sum_out); y = rms_norm(h) * w.
// One CTA per row; thread i owns elements [8i, 8i + 8). The normalized value is
// rounded to T before the weight product, which is rounded again (one rounding
// per operation in the activation type).
template <typename T>
__global__ void rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ delta,
                                const T* __restrict__ w, T* __restrict__ y,
                                T* __restrict__ sum_out, int D, float eps) {
    __shared__ float red[32];
    pdl_launch_dependents();
    const int row = blockIdx.x;
    const int i = threadIdx.x;
    const bool on = 8 * i < D;
    // the weight is a parameter (not written by the kernels before this one): load
    // it before waiting for them
    uint4 wv = make_uint4(0u, 0u, 0u, 0u);
    if (on) wv = *reinterpret_cast<const uint4*>(w + 8 * i);
    pdl_wait();
    float h[8];
    float ss = 0.f;
    if (on) {
        const uint4 xv = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * D + 8 * i);
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
        if (delta) {
            const uint4 dv =
                *reinterpret_cast<const uint4*>(delta + static_cast<size_t>(row) * D + 8 * i);
            const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 a = unpack2<T>(xw[k]), b = unpack2<T>(dw[k]);
                h[2 * k] = round_t<T>(a.x + b.x);
                h[2 * k + 1] = round_t<T>(a.y + b.y);
            }
            if (sum_out) {
                uint4 o;
                o.x = pack2<T>(h[0], h[1]);
                o.y = pack2<T>(h[2], h[3]);
                o.z = pack2<T>(h[4], h[5]);
                o.w = pack2<T>(h[6], h[7]);
                *reinterpret_cast<uint4*>(sum_out + static_cast<size_t>(row) * D + 8 * i) = o;
            }
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 a = unpack2<T>(xw[k]);
                h[2 * k] = a.x;
                h[2 * k + 1] = a.y;
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) ss = fmaf(h[k], h[k], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int warps = (blockDim.x + 31) >> 5;
    if ((i & 31) == 0) red[i >> 5] = ss;
    __syncthreads();
    if (i < 32) {
        float v = i < warps ? red[i] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (i == 0) red[0] = v;
    }
    __syncthreads();
    const float r = rsqrtf(red[0] / static_cast<float>(D) + eps);
    if (on) {
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 g = unpack2<T>(ww[k]);
            o[k] = pack2<T>(round_t<T>(h[2 * k] * r) * g.x, round_t<T>(h[2 * k + 1] * r) * g.y);
        }
        *reinterpret_cast<uint4*>(y + static_cast<size_t>(row) * D + 8 * i) =
            make_uint4(o[0], o[1], o[2], o[3]);
    }
}

cudaError_t launch_rms_norm(int dtype, const void* x, const void* delta, const void* w, void* y,
                            void* sum_out, int rows, int D, float eps, bool overlap,
                            cudaStream_t st) {
    const int threads = ((D / 8) + 31) / 32 * 32;
    void* args[] = {&x, &delta, &w, &y, &sum_out, &D, &eps};
    static PerDevice cfg[2];
    const bool bf = dtype == kBF16;
    const void* f = bf ? reinterpret_cast<const void*>(&rms_norm_kernel<__nv_bfloat16>)
                       : reinterpret_cast<const void*>(&rms_norm_kernel<__half>);
    return launch_ex(f, cfg[bf ? 0 : 1], dim3(rows), dim3(threads), 0, st, overlap, args);
}

// ------------------------------------------------------------------------------------
// RoPE (half-rotation form, traditional=False) and the paged KV append. CTA (token t,
// head block y) rotates ROPE_HEADS heads, one (i, i + hd/2) pair per thread, so
// every thread has one load of each operand in flight; queries go to q_out
// [T, Hq, hd], keys and values to their cache slot (slot = page * page_size +
// offset; a negative slot skips the append). The values are copied by the CTAs
// of the token's first head block.
//   freq_i = base^(-2i/hd), angle = position * freq_i, for i < hd/2:
//   (a, b) = (x_i, x_{i+hd/2}) -> (a cos - b sin, a sin + b cos), rounded to T.
constexpr int ROPE_HEADS = 4;

template <typename T>
__global__ void rope_append_kernel(const T* __restrict__ qkv, int ld, T* __restrict__ q_out,
                                   T* __restrict__ k_cache, T* __restrict__ v_cache,
                                   const int32_t* __restrict__ positions,
                                   const int32_t* __restrict__ slots, int Hq, int Hkv, int hd,
                                   float log2_base) {
    pdl_launch_dependents();
    const int half = hd / 2;
    const int i = threadIdx.x % half;
    const int h = blockIdx.y * ROPE_HEADS + threadIdx.x / half;
    // the frequency depends on nothing the previous kernel writes
    const float freq =
        exp2f(-(2.0f * static_cast<float>(i) / static_cast<float>(hd)) * log2_base);
    pdl_wait();
    const int t = blockIdx.x;
    const T* src = qkv + static_cast<size_t>(t) * ld;
    const int slot = slots[t];
    if (h < Hq + Hkv) {
        const float pos = static_cast<float>(positions[t]);
        const float a = Elem<T>::to_f(src[h * hd + i]);
        const float b = Elem<T>::to_f(src[h * hd + i + half]);
        float sn, cs;
        sincosf(pos * freq, &sn, &cs);
        const T ra = Elem<T>::from_f(a * cs - b * sn);
        const T rb = Elem<T>::from_f(a * sn + b * cs);
        if (h < Hq) {
            T* dq = q_out + (static_cast<size_t>(t) * Hq + h) * hd;
            dq[i] = ra;
            dq[i + half] = rb;
        } else if (slot >= 0) {
            T* dk = k_cache + (static_cast<size_t>(slot) * Hkv + (h - Hq)) * hd;
            dk[i] = ra;
            dk[i + half] = rb;
        }
    }
    if (blockIdx.y == 0 && slot >= 0) {
        const int vchunks = Hkv * hd / 8;
        const uint4* vs = reinterpret_cast<const uint4*>(src + (Hq + Hkv) * hd);
        uint4* vd = reinterpret_cast<uint4*>(v_cache + static_cast<size_t>(slot) * Hkv * hd);
        for (int c = threadIdx.x; c < vchunks; c += blockDim.x) vd[c] = vs[c];
    }
}

cudaError_t launch_rope_append(int dtype, const void* qkv, int ld, void* q_out, void* k_cache,
                               void* v_cache, const int32_t* positions, const int32_t* slots,
                               int tokens, int Hq, int Hkv, int hd, float log2_base, bool overlap,
                               cudaStream_t st) {
    void* args[] = {&qkv, &ld, &q_out, &k_cache, &v_cache, &positions, &slots,
                    &Hq, &Hkv, &hd, &log2_base};
    static PerDevice cfg[2];
    const bool bf = dtype == kBF16;
    const void* f = bf ? reinterpret_cast<const void*>(&rope_append_kernel<__nv_bfloat16>)
                       : reinterpret_cast<const void*>(&rope_append_kernel<__half>);
    const int blocks_y = (Hq + Hkv + ROPE_HEADS - 1) / ROPE_HEADS;
    return launch_ex(f, cfg[bf ? 0 : 1], dim3(tokens, blocks_y), dim3(ROPE_HEADS * hd / 2), 0, st,
                     overlap, args);
}

// ------------------------------------------------------------------------------------
// Decode attention on the tensor cores: one query token per sequence. CTA (split s,
// kv head g, sequence b) takes a contiguous range of the sequence's L_b cached keys
// (tps tiles of 64 keys; at most 64 splits per sequence) and the G = Hq/Hkv <= 8 query
// heads sharing kv head g, which are the rows of the m16n8k16 MMAs (rows G..15 zero).
// Per tile, the key and value rows are gathered from the pages with cp.async into
// shared memory (16-byte chunks XOR-swizzled by row: ldmatrix reads are conflict
// free); warp w owns keys 16w..16w+15 of every tile:
//   S = Q K^T      2 n-tiles of 8 keys x 8 k-steps of 16 dimensions (fp32)
//   softmax        online per row over the warp's keys (running max, sum; exp2)
//   O += P V       P stays in registers as the A operand, V read transposed
// The 4 warps' (max, sum, O) are merged in shared memory. A sequence with one split
// writes its outputs; otherwise each split stores its (max, sum, unnormalised output)
// and the last split to finish (acquire-release ticket per (b, g), zero between
// calls) merges them in split order.
namespace attn {
constexpr int SK = 64;        // keys per tile
constexpr int THREADS = 128;  // 4 warps x 16 keys
constexpr int MAXG = 8;       // query heads per kv head
constexpr int MAXSPLIT = 64;  // splits per sequence
}  // namespace attn

template <int HD>
__device__ __forceinline__ uint32_t kv_swz(int row, int chunk) {
    return static_cast<uint32_t>(row * (HD * 2) + ((chunk ^ (row & 7)) << 4));
}

template <typename T, int HD>
__global__ void __launch_bounds__(attn::THREADS)
    attn_decode_kernel(const T* __restrict__ q, const T* __restrict__ k_cache,
                       const T* __restrict__ v_cache, const int32_t* __restrict__ block_table,
                       int max_blocks, const int32_t* __restrict__ kv_lens, T* __restrict__ out,
                       int Hq, int Hkv, int page, float scale_log2, float* __restrict__ ws_o,
                       float2* __restrict__ ws_ml, unsigned* __restrict__ tickets,
                       int max_splits, int max_kv, int tps) {
    using namespace attn;
    static_assert(HD == 64 || HD == 128, "head_dim");
    constexpr int CH = HD / 8;            // 16-byte chunks per row
    constexpr int NW = THREADS / 32;      // warps
    constexpr int DPT = HD / 16;          // dimensions per thread in the merges (8 or 4)
    __shared__ __align__(128) uint8_t qsm[16 * HD * 2];
    __shared__ __align__(128) uint8_t kv[2 * SK * HD * 2];  // keys, values; then warp O
    __shared__ float wm[NW][MAXG], wl[NW][MAXG];
    __shared__ int pid[SK / 8 + 2];
    __shared__ int s_last;
    static_assert(NW * MAXG * HD * 4 <= 2 * SK * HD * 2, "warp outputs fit the tile buffer");
    pdl_launch_dependents();
    pdl_wait();
    const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int G = Hq / Hkv;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int skeys = tps * SK;             // keys per split
    const int ks0 = split * skeys;
    const int32_t* bt = block_table + static_cast<size_t>(b) * max_blocks;
    // The sequence length, the first tile's page ids and the queries do not depend on
    // one another: their loads are issued together (page ids past the block table are
    // not read).
    constexpr int QPT = (16 * CH + THREADS - 1) / THREADS;  // query chunks per thread
    int pid0 = 0;
    const int p00 = ks0 / page;
    if (tid < SK / 8 + 2 && p00 + tid < max_blocks) pid0 = bt[p00 + tid];
    uint4 qv[QPT];
#pragma unroll
    for (int i = 0; i < QPT; ++i) {
        const int c = tid + i * THREADS;
        const int r = c / CH, ch = c % CH;
        qv[i] = make_uint4(0u, 0u, 0u, 0u);
        if (c < 16 * CH && r < G)
            qv[i] = *reinterpret_cast<const uint4*>(
                q + (static_cast<size_t>(b) * Hq + g * G + r) * HD + ch * 8);
    }
    const int L = min(kv_lens[b], max_kv);  // max_kv <= the block table's reach
    const int nsplit = (L + skeys - 1) / skeys;
    if (split >= nsplit) return;
    const int ke = min(L, ks0 + skeys);
    const int ntile = (ke - ks0 + SK - 1) / SK;
    uint8_t* ksm = kv;
    uint8_t* vsm = kv + SK * HD * 2;

    // queries: rows = the group's heads, rows G..15 zero
#pragma unroll
    for (int i = 0; i < QPT; ++i) {
        const int c = tid + i * THREADS;
        if (c < 16 * CH) *reinterpret_cast<uint4*>(qsm + kv_swz<HD>(c / CH, c % CH)) = qv[i];
    }
    if (tid < SK / 8 + 2) pid[tid] = pid0;  // page sizes >= 8: a tile spans <= SK/8 + 1 pages
    __syncthreads();
    uint32_t qa[HD / 16][4];
    {
        const uint32_t qb = smem_u32(qsm);
        const int r = lane & 15;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
            ldmatrix_x4(qb + kv_swz<HD>(r, 2 * kk + (lane >> 4)), qa[kk][0], qa[kk][1],
                        qa[kk][2], qa[kk][3]);
    }
    float o[HD / 8][4];
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float mrow = -INFINITY, lrow = 0.f;  // row lane/4 (a head); rows 8.. are padding

    for (int tile = 0; tile < ntile; ++tile) {
        const int k0 = ks0 + tile * SK;
        const int n = min(SK, ke - k0);
        const int p0 = k0 / page;
        const int np = (k0 + n - 1) / page - p0 + 1;
        if (tile > 0) {
            __syncthreads();  // the previous tile's buffers are free
            if (tid < np) pid[tid] = bt[p0 + tid];
            __syncthreads();
        }
#pragma unroll 4
        for (int c = tid; c < SK * CH; c += THREADS) {
            const int r = c / CH, ch = c % CH;
            const bool ok = r < n;
            const int key = ok ? k0 + r : k0;
            const size_t row = static_cast<size_t>(pid[key / page - p0]) * page + key % page;
            const size_t off = (row * Hkv + g) * HD + ch * 8;
            cp_async16(ksm + kv_swz<HD>(r, ch), k_cache + off, ok ? 16 : 0);
            cp_async16(vsm + kv_swz<HD>(r, ch), v_cache + off, ok ? 16 : 0);
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        // S = Q K^T over this warp's 16 keys
        float sc[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
        const uint32_t kb = smem_u32(ksm), vb = smem_u32(vsm);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
            const int r = warp * 16 + (lane & 7) + ((lane >> 4) << 3);
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4(kb + kv_swz<HD>(r, 2 * kk + ((lane >> 3) & 1)), b0, b1, b2, b3);
            mma16816<T>(sc[0], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
            mma16816<T>(sc[1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
        }
        // mask the tile's tail, scale (base 2), online softmax of row lane/4
        float mnew = mrow;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int key = warp * 16 + nt * 8 + 2 * (lane & 3) + e;
                sc[nt][e] = key < n ? sc[nt][e] * scale_log2 : -INFINITY;
                mnew = fmaxf(mnew, sc[nt][e]);
            }
        mnew = fmaxf(mnew, __shfl_xor_sync(0xffffffffu, mnew, 1));
        mnew = fmaxf(mnew, __shfl_xor_sync(0xffffffffu, mnew, 2));
        const float mref = mnew == -INFINITY ? 0.f : mnew;
        const float corr = exp2f(mrow - mref);
        mrow = mnew;
        lrow *= corr;
        uint32_t pa[4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            const float p0v = exp2f(sc[nt][0] - mref), p1v = exp2f(sc[nt][1] - mref);
            lrow += p0v + p1v;
            pa[2 * nt] = pack2<T>(p0v, p1v);
            pa[2 * nt + 1] = 0u;  // rows 8..15 (padding) carry nothing
        }
#pragma unroll
        for (int j = 0; j < HD / 8; ++j) {
            o[j][0] *= corr;
            o[j][1] *= corr;
        }
        // O += P V over this warp's 16 keys
#pragma unroll
        for (int dpp = 0; dpp < HD / 16; ++dpp) {
            const int r = warp * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4_trans(vb + kv_swz<HD>(r, 2 * dpp + (lane >> 4)), b0, b1, b2, b3);
            mma16816<T>(o[2 * dpp], pa[0], pa[1], pa[2], pa[3], b0, b1);
            mma16816<T>(o[2 * dpp + 1], pa[0], pa[1], pa[2], pa[3], b2, b3);
        }
    }
    // merge the warps: row sums, then (max, sum, O) of rows < G through shared memory
    lrow += __shfl_xor_sync(0xffffffffu, lrow, 1);
    lrow += __shfl_xor_sync(0xffffffffu, lrow, 2);
    const int hr = lane >> 2;  // this lane's head row
    if ((lane & 3) == 0 && hr < MAXG) {
        wm[warp][hr] = mrow;
        wl[warp][hr] = lrow;
    }
    __syncthreads();  // (the tile buffers are free from here: they hold the warps' O)
    float* wo = reinterpret_cast<float*>(kv);  // [NW][MAXG][HD]
    if (hr < G) {
#pragma unroll
        for (int j = 0; j < HD / 8; ++j)
            *reinterpret_cast<float2*>(&wo[(warp * MAXG + hr) * HD + 8 * j + 2 * (lane & 3)]) =
                make_float2(o[j][0], o[j][1]);
    }
    __syncthreads();
    // thread (head h, dimensions DPT*dd ..): the CTA's result for its slice
    const int h = tid / (HD / DPT), dd = tid % (HD / DPT);
    float res[DPT];
    float Mc = -INFINITY, Lc = 0.f;
    if (h < G) {
#pragma unroll
        for (int w = 0; w < NW; ++w) Mc = fmaxf(Mc, wm[w][h]);
#pragma unroll
        for (int e = 0; e < DPT; ++e) res[e] = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float c = wm[w][h] == -INFINITY ? 0.f : exp2f(wm[w][h] - Mc);
            Lc = fmaf(c, wl[w][h], Lc);
#pragma unroll
            for (int e = 0; e < DPT; ++e) res[e] = fmaf(c, wo[(w * MAXG + h) * HD + DPT * dd + e], res[e]);
        }
    }
    if (nsplit == 1) {
        if (h < G) {
            const float inv = 1.0f / Lc;
            T* dst = out + (static_cast<size_t>(b) * Hq + g * G + h) * HD + DPT * dd;
#pragma unroll
            for (int e = 0; e < DPT; e += 2)
                *reinterpret_cast<uint32_t*>(dst + e) = pack2<T>(res[e] * inv, res[e + 1] * inv);
        }
        return;
    }
    // this split's partials: [b][g][split][h][HD] and (m, l) per head
    const size_t base = (static_cast<size_t>(b) * Hkv + g) * max_splits;
    if (h < G) {
#pragma unroll
        for (int e = 0; e < DPT; ++e) ws_o[((base + split) * MAXG + h) * HD + DPT * dd + e] = res[e];
        if (dd == 0) ws_ml[(base + split) * MAXG + h] = make_float2(Mc, Lc);
    }
    // The barrier orders every thread's partials before thread 0's acq_rel ticket,
    // whose release publishes them GPU-wide and whose acquire (with the second barrier)
    // makes the other splits' partials visible to this CTA.
    __syncthreads();
    if (tid == 0)
        s_last = atom_add_acq_rel_gpu(tickets + b * Hkv + g, 1u) ==
                 static_cast<unsigned>(nsplit - 1);
    __syncthreads();
    if (!s_last) return;
    // The last split merges them in split order with a running maximum: each thread
    // reads every split's (max, sum) of its head and its slice of the split's outputs,
    // four splits' loads in flight together.
    if (h < G) {
        float acc[DPT];
#pragma unroll
        for (int e = 0; e < DPT; ++e) acc[e] = 0.f;
        float M = -INFINITY, den = 0.f;
#pragma unroll 4
        for (int sp = 0; sp < nsplit; ++sp) {
            const float2 ml = __ldcg(&ws_ml[(base + sp) * MAXG + h]);
            const float* src = &ws_o[((base + sp) * MAXG + h) * HD + DPT * dd];
            float v[DPT];
#pragma unroll
            for (int e = 0; e < DPT; e += 4) {
                const float4 t = __ldcg(reinterpret_cast<const float4*>(src + e));
                v[e] = t.x; v[e + 1] = t.y; v[e + 2] = t.z; v[e + 3] = t.w;
            }
            const float Mn = fmaxf(M, ml.x);
            const float co = M == -INFINITY ? 0.f : exp2f(M - Mn);
            const float cn = ml.x == -INFINITY ? 0.f : exp2f(ml.x - Mn);
            den = fmaf(cn, ml.y, den * co);
#pragma unroll
            for (int e = 0; e < DPT; ++e) acc[e] = fmaf(cn, v[e], acc[e] * co);
            M = Mn;
        }
        const float inv = 1.0f / den;
        T* dst = out + (static_cast<size_t>(b) * Hq + g * G + h) * HD + DPT * dd;
#pragma unroll
        for (int e = 0; e < DPT; e += 2)
            *reinterpret_cast<uint32_t*>(dst + e) = pack2<T>(acc[e] * inv, acc[e + 1] * inv);
    }
    if (tid == 0) tickets[b * Hkv + g] = 0u;
}

// ------------------------------------------------------------------------------------
// Prefill attention (flash-attention form on mma.sync m16n8k16, fp32 accumulation):
// CTA (query tile of 64 tokens, query head h, sequence b), 4 warps of 16 query rows.
// Query i of sequence b sits at position L_b - Lq_b + i and attends keys at positions
// <= its own (keys < L_b). Key and value tiles of 64 keys come from the pages through
// a two-stage cp.async ring, XOR-swizzled by 16-byte chunk so ldmatrix reads are
// conflict free; probabilities stay in registers as the A operand of P V.
namespace pf {
constexpr int QT = 64;   // queries per CTA
constexpr int KT = 64;   // keys per tile
constexpr int THREADS = 128;
}  // namespace pf

template <int HD>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
    return static_cast<uint32_t>(row * (HD * 2) + ((chunk ^ (row & 7)) << 4));
}

template <typename T, int HD>
__global__ void __launch_bounds__(pf::THREADS)
    attn_prefill_kernel(const T* __restrict__ q, const int32_t* __restrict__ cu_q,
                        const T* __restrict__ k_cache, const T* __restrict__ v_cache,
                        const int32_t* __restrict__ block_table, int max_blocks,
                        const int32_t* __restrict__ kv_lens, T* __restrict__ out, int Hq,
                        int Hkv, int page, float scale_log2) {
    using namespace pf;
    static_assert(HD == 64 || HD == 128, "head_dim");
    constexpr int CH = HD / 8;  // 16-byte chunks per row
    extern __shared__ __align__(128) uint8_t pf_smem[];
    uint8_t* qsm = pf_smem;                      // [QT][HD]
    uint8_t* ksm = qsm + QT * HD * 2;            // [2][KT][HD]
    uint8_t* vsm = ksm + 2 * KT * HD * 2;        // [2][KT][HD]
    pdl_launch_dependents();
    pdl_wait();
    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int q0 = cu_q[b], Lq = cu_q[b + 1] - q0;
    if (qt * QT >= Lq) return;
    const int L = min(kv_lens[b], max_blocks * page);
    const int g = h / (Hq / Hkv);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pos0 = L - Lq;  // position of query 0
    const int qlo = qt * QT, qhi = min(Lq, qlo + QT);
    const int kend = min(L, pos0 + qhi);  // keys [0, kend) are visible to some row
    const int ntiles = (kend + KT - 1) / KT;
    const int32_t* bt = block_table + static_cast<size_t>(b) * max_blocks;

    // queries (rows past Lq are zero)
    for (int c = tid; c < QT * CH; c += THREADS) {
        const int r = c / CH, ch = c % CH;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (qlo + r < Lq)
            v = *reinterpret_cast<const uint4*>(
                q + (static_cast<size_t>(q0 + qlo + r) * Hq + h) * HD + ch * 8);
        *reinterpret_cast<uint4*>(qsm + swz<HD>(r, ch)) = v;
    }
    auto load_tile = [&](int tile, int stage) {
        uint8_t* kd = ksm + stage * KT * HD * 2;
        uint8_t* vd = vsm + stage * KT * HD * 2;
        for (int c = tid; c < KT * CH; c += THREADS) {
            const int r = c / CH, ch = c % CH;
            const int key = tile * KT + r;
            const bool ok = key < kend;
            const int kk = ok ? key : 0;
            const size_t row = static_cast<size_t>(bt[kk / page]) * page + kk % page;
            const size_t off = (row * Hkv + g) * HD + ch * 8;
            cp_async16(kd + swz<HD>(r, ch), k_cache + off, ok ? 16 : 0);
            cp_async16(vd + swz<HD>(r, ch), v_cache + off, ok ? 16 : 0);
        }
        cp_async_commit();
    };
    if (ntiles > 0) load_tile(0, 0);
    __syncthreads();

    // this warp's 16 query rows as A fragments (k = head dims)
    uint32_t qa[HD / 16][4];
    {
        const uint32_t qb = smem_u32(qsm);
        const int r = warp * 16 + (lane & 15);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
            const int ch = 2 * kk + (lane >> 4);
            ldmatrix_x4(qb + swz<HD>(r, ch), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
        }
    }
    float o[HD / 8][4];
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    // positions of the two rows this lane holds (rows r and r + 8 of the warp's tile)
    const int qpos[2] = {pos0 + qlo + warp * 16 + (lane >> 2),
                         pos0 + qlo + warp * 16 + (lane >> 2) + 8};

    for (int tile = 0; tile < ntiles; ++tile) {
        const int stage = tile & 1;
        if (tile + 1 < ntiles) {
            load_tile(tile + 1, stage ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const uint32_t kb = smem_u32(ksm + stage * KT * HD * 2);
        const uint32_t vb = smem_u32(vsm + stage * KT * HD * 2);
        // S = Q K^T for 64 keys: 8 n-tiles of 8 keys
        float s[KT / 8][4];
#pragma unroll
        for (int nt = 0; nt < KT / 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
            for (int np = 0; np < KT / 16; ++np) {
                // keys 16np..16np+15, dims 16kk..16kk+15: x4 gives two n-tiles' B
                const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int ch = 2 * kk + ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldmatrix_x4(kb + swz<HD>(r, ch), b0, b1, b2, b3);
                mma16816<T>(s[2 * np], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
                mma16816<T>(s[2 * np + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
            }
        }
        // mask, scale (base 2), online softmax
        float mnew[2] = {mrow[0], mrow[1]};
#pragma unroll
        for (int nt = 0; nt < KT / 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = tile * KT + nt * 8 + 2 * (lane & 3) + (e & 1);
                const int rr = e >> 1;
                const bool ok = key < kend && key <= qpos[rr];
                s[nt][e] = ok ? s[nt][e] * scale_log2 : -INFINITY;
                mnew[rr] = fmaxf(mnew[rr], s[nt][e]);
            }
        }
        float corr[2];
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            mnew[rr] = fmaxf(mnew[rr], __shfl_xor_sync(0xffffffffu, mnew[rr], 1));
            mnew[rr] = fmaxf(mnew[rr], __shfl_xor_sync(0xffffffffu, mnew[rr], 2));
            const float mref = mnew[rr] == -INFINITY ? 0.f : mnew[rr];
            corr[rr] = exp2f(mrow[rr] - mref);
            mrow[rr] = mnew[rr];
            lrow[rr] *= corr[rr];
        }
        uint32_t pa[KT / 16][4];
#pragma unroll
        for (int nt = 0; nt < KT / 8; ++nt) {
            float p[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int rr = e >> 1;
                const float mref = mrow[rr] == -INFINITY ? 0.f : mrow[rr];
                p[e] = exp2f(s[nt][e] - mref);
                lrow[rr] += p[e];
            }
            // C fragment of n-tile nt = half of the A fragment of k-step nt/2
            pa[nt >> 1][(nt & 1) * 2 + 0] = pack2<T>(p[0], p[1]);
            pa[nt >> 1][(nt & 1) * 2 + 1] = pack2<T>(p[2], p[3]);
        }
#pragma unroll
        for (int j = 0; j < HD / 8; ++j) {
            o[j][0] *= corr[0];
            o[j][1] *= corr[0];
            o[j][2] *= corr[1];
            o[j][3] *= corr[1];
        }
        // O += P V: k = keys, n = head dims; V rows are [key][dim], read transposed
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
#pragma unroll
            for (int dp = 0; dp < HD / 16; ++dp) {
                const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
                const int ch = 2 * dp + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldmatrix_x4_trans(vb + swz<HD>(r, ch), b0, b1, b2, b3);
                mma16816<T>(o[2 * dp], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
                mma16816<T>(o[2 * dp + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
            }
        }
        __syncthreads();  // the stage is refilled next iteration
    }
    // normalise and store rows r, r + 8
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        float l = lrow[rr];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        const int qi = qlo + warp * 16 + (lane >> 2) + 8 * rr;
        if (qi >= Lq) continue;
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        T* dst = out + (static_cast<size_t>(q0 + qi) * Hq + h) * HD;
#pragma unroll
        for (int j = 0; j < HD / 8; ++j) {
            const int d = j * 8 + 2 * (lane & 3);
            *reinterpret_cast<uint32_t*>(dst + d) =
                pack2<T>(o[j][2 * rr] * inv, o[j][2 * rr + 1] * inv);
        }
    }
}

// Tiles of SK keys per split: one until a sequence would need more than MAXSPLIT splits.
static int attn_tiles_per_split(int max_kv_len) {
    const int tiles = (max_kv_len + attn::SK - 1) / attn::SK;
    return (tiles + attn::MAXSPLIT - 1) / attn::MAXSPLIT;
}
static int attn_splits(int max_kv_len) {
    const int keys = attn_tiles_per_split(max_kv_len) * attn::SK;
    return (max_kv_len + keys - 1) / keys;
}

size_t attn_decode_workspace(int B, int Hkv, int max_kv_len, int head_dim) {
    const int splits = attn_splits(max_kv_len);
    if (splits <= 1) return 0;
    const size_t tickets = (static_cast<size_t>(B) * Hkv * 4 + 255) / 256 * 256;
    const size_t parts = static_cast<size_t>(B) * Hkv * splits * attn::MAXG;
    return tickets + parts * head_dim * 4 + parts * 8;
}

cudaError_t launch_attn_decode(int dtype, const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* block_table, int max_blocks, const int32_t* kv_lens,
                               int max_kv_len, void* out, int B, int Hq, int Hkv, int hd, int page,
                               float scale, void* workspace, bool overlap, cudaStream_t st) {
    const int splits = attn_splits(max_kv_len);
    int tps = attn_tiles_per_split(max_kv_len);
    float scale_log2 = scale * 1.4426950408889634f;
    unsigned* tickets = nullptr;
    float* ws_o = nullptr;
    float2* ws_ml = nullptr;
    if (splits > 1) {
        char* base = static_cast<char*>(workspace);
        const size_t tb = (static_cast<size_t>(B) * Hkv * 4 + 255) / 256 * 256;
        const size_t parts = static_cast<size_t>(B) * Hkv * splits * attn::MAXG;
        tickets = reinterpret_cast<unsigned*>(base);
        ws_o = reinterpret_cast<float*>(base + tb);
        ws_ml = reinterpret_cast<float2*>(base + tb + parts * hd * 4);
    }
    int max_splits = splits;
    void* args[] = {&q, &k_cache, &v_cache, &block_table, &max_blocks, &kv_lens, &out,
                    &Hq, &Hkv, &page, &scale_log2, &ws_o, &ws_ml, &tickets, &max_splits,
                    &max_kv_len, &tps};
    const void* f = nullptr;
    if (dtype == kBF16)
        f = hd == 128 ? reinterpret_cast<const void*>(&attn_decode_kernel<__nv_bfloat16, 128>)
                      : reinterpret_cast<const void*>(&attn_decode_kernel<__nv_bfloat16, 64>);
    else
        f = hd == 128 ? reinterpret_cast<const void*>(&attn_decode_kernel<__half, 128>)
                      : reinterpret_cast<const void*>(&attn_decode_kernel<__half, 64>);
    static PerDevice cfg[4];
    const int which = (dtype == kBF16 ? 0 : 2) + (hd == 128 ? 0 : 1);
    return launch_ex(f, cfg[which], dim3(splits, Hkv, B), dim3(attn::THREADS), 0, st, overlap,
                     args);
}

size_t attn_prefill_smem(int hd) { return static_cast<size_t>(pf::QT + 4 * pf::KT) * hd * 2; }

cudaError_t launch_attn_prefill(int dtype, const void* q, const int32_t* cu_q, int max_q_len,
                                const void* k_cache, const void* v_cache,
                                const int32_t* block_table, int max_blocks,
                                const int32_t* kv_lens, void* out, int B, int Hq, int Hkv, int hd,
                                int page, float scale, bool overlap, cudaStream_t st) {
    float scale_log2 = scale * 1.4426950408889634f;
    const size_t smem = attn_prefill_smem(hd);
    const void* f = nullptr;
    if (dtype == kBF16)
        f = hd == 128 ? reinterpret_cast<const void*>(&attn_prefill_kernel<__nv_bfloat16, 128>)
                      : reinterpret_cast<const void*>(&attn_prefill_kernel<__nv_bfloat16, 64>);
    else
        f = hd == 128 ? reinterpret_cast<const void*>(&attn_prefill_kernel<__half, 128>)
                      : reinterpret_cast<const void*>(&attn_prefill_kernel<__half, 64>);
    static PerDevice cfg[4];
    const int which = (dtype == kBF16 ? 0 : 2) + (hd == 128 ? 0 : 1);
    void* args[] = {&q, &cu_q, &k_cache, &v_cache, &block_table, &max_blocks, &kv_lens, &out,
                    &Hq, &Hkv, &page, &scale_log2};
    const int qtiles = (max_q_len + pf::QT - 1) / pf::QT;
    return launch_ex(f, cfg[which], dim3(qtiles, Hq, B), dim3(pf::THREADS), smem, st, overlap,
                     args);
}

// ------------------------------------------------------------------------------------
// Quantized embedding lookup: out[i] = dequantize(row ids[i]) with MLX's rounding,
// round(round(scale * q) + bias) in T (bit-identical to mlxq_dequantize of that row).
// One CTA per id, one thread per packed word; ids outside [0, vocab) give zeros.
template <typename T, int BITS>
__global__ void embed_kernel(const int32_t* __restrict__ ids, const uint32_t* __restrict__ wq,
                             const T* __restrict__ scales, const T* __restrict__ biases,
                             T* __restrict__ out, int vocab, int K, int gs) {
    constexpr int EPW = 32 / BITS;
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.x;
    const int id = ids[i];
    const int words = K / EPW;
    T* dst = out + static_cast<size_t>(i) * K;
    for (int wi = threadIdx.x; wi < words; wi += blockDim.x) {
        uint32_t packed[EPW / 2];
        if (id >= 0 && id < vocab) {
            const uint32_t wv = wq[static_cast<size_t>(id) * words + wi];
            const int g = wi * EPW / gs;
            const float s = Elem<T>::to_f(scales[static_cast<size_t>(id) * (K / gs) + g]);
            const float b = Elem<T>::to_f(biases[static_cast<size_t>(id) * (K / gs) + g]);
#pragma unroll
            for (int e = 0; e < EPW; e += 2) {
                const float q0 = static_cast<float>((wv >> (BITS * e)) & ((1u << BITS) - 1u));
                const float q1 = static_cast<float>((wv >> (BITS * (e + 1))) & ((1u << BITS) - 1u));
                packed[e / 2] = pack2<T>(round_t<T>(s * q0) + b, round_t<T>(s * q1) + b);
            }
        } else {
#pragma unroll
            for (int e = 0; e < EPW / 2; ++e) packed[e] = 0u;
        }
        if constexpr (EPW == 8) {
            *reinterpret_cast<uint4*>(dst + wi * EPW) =
                make_uint4(packed[0], packed[1], packed[2], packed[3]);
        } else {
            *reinterpret_cast<uint2*>(dst + wi * EPW) = make_uint2(packed[0], packed[1]);
        }
    }
}

cudaError_t launch_embed(int dtype, int bits, const int32_t* ids, int n, const uint32_t* wq,
                         const void* scales, const void* biases, void* out, int vocab, int K,
                         int gs, bool overlap, cudaStream_t st) {
    void* args[] = {&ids, &wq, &scales, &biases, &out, &vocab, &K, &gs};
    const void* f = nullptr;
    if (dtype == kBF16)
        f = bits == 4 ? reinterpret_cast<const void*>(&embed_kernel<__nv_bfloat16, 4>)
                      : reinterpret_cast<const void*>(&embed_kernel<__nv_bfloat16, 8>);
    else
        f = bits == 4 ? reinterpret_cast<const void*>(&embed_kernel<__half, 4>)
                      : reinterpret_cast<const void*>(&embed_kernel<__half, 8>);
    const int words = K * bits / 32;
    const int threads = words >= 256 ? 256 : (words + 31) / 32 * 32;
    static PerDevice cfg[4];
    const int which = (dtype == kBF16 ? 0 : 2) + (bits == 4 ? 0 : 1);
    return launch_ex(f, cfg[which], dim3(n), dim3(threads), 0, st, overlap, args);
}

// ------------------------------------------------------------------------------------
// MoE routing (lfm2.py:366-375): per token, gates = softmax(logits in float32)
// (+ expert_bias), the top_k experts by gate (their order is not part of the
// reference's contract, which takes an argpartition; here: descending gate, the
// lower index first on ties), their gates, renormalised to sum to one with the
// reference's 1e-20 guard when norm_topk, rounded to the scores' dtype. One warp per
// token; lane l holds experts l, l + 32, ...
template <typename TL, typename TS>
__global__ void moe_route_kernel(const TL* __restrict__ logits, const float* __restrict__ bias,
                                 int32_t* __restrict__ indices, TS* __restrict__ scores, int T,
                                 int E, int K, int norm) {
    constexpr int MAXE = 1024 / 32;
    pdl_launch_dependents();
    pdl_wait();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const TL* row = logits + static_cast<size_t>(warp) * E;
    float v[MAXE];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < MAXE; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < E ? static_cast<float>(Elem<TL>::to_f(row[e])) : -INFINITY;
        m = fmaxf(m, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < MAXE; ++i) {
        v[i] = lane + 32 * i < E ? expf(v[i] - m) : 0.f;
        sum += v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.0f / sum;
#pragma unroll
    for (int i = 0; i < MAXE; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < E ? v[i] * inv + (bias ? bias[e] : 0.f) : -INFINITY;
    }
    float picked = 0.f;   // lane k (< K) keeps the k-th pick
    int picked_idx = 0;
    float total = 0.f;
    for (int k = 0; k < K; ++k) {
        float best = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < MAXE; ++i) {
            const int e = lane + 32 * i;
            if (v[i] > best || (v[i] == best && e < bi)) {
                best = v[i];
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob > best || (ob == best && oi < bi)) {
                best = ob;
                bi = oi;
            }
        }
#pragma unroll
        for (int i = 0; i < MAXE; ++i)
            if (lane + 32 * i == bi) v[i] = -INFINITY;
        if (lane == k) {
            picked = best;
            picked_idx = bi;
        }
        total += best;
    }
    if (lane < K) {
        const float sc = norm ? picked / (total + 1e-20f) : picked;
        indices[static_cast<size_t>(warp) * K + lane] = picked_idx;
        scores[static_cast<size_t>(warp) * K + lane] = Elem<TS>::from_f(sc);
    }
}

cudaError_t launch_moe_route(int logits_dtype, const void* logits, const float* bias,
                             int32_t* indices, int scores_dtype, void* scores, int T, int E, int K,
                             int norm, bool overlap, cudaStream_t st) {
    void* args[] = {&logits, &bias, &indices, &scores, &T, &E, &K, &norm};
    static PerDevice cfg[9];
    const void* f = nullptr;
    int which = 0;
#define MLXQ_ROUTE_CASE(LD, LT, SD, STY, W)                                             \
    if (logits_dtype == LD && scores_dtype == SD) {                                    \
        f = reinterpret_cast<const void*>(&moe_route_kernel<LT, STY>);                 \
        which = W;                                                                      \
    }
    MLXQ_ROUTE_CASE(kF32, float, kBF16, __nv_bfloat16, 0)
    MLXQ_ROUTE_CASE(kF32, float, kF16, __half, 1)
    MLXQ_ROUTE_CASE(kF32, float, kF32, float, 2)
    MLXQ_ROUTE_CASE(kBF16, __nv_bfloat16, kBF16, __nv_bfloat16, 3)
    MLXQ_ROUTE_CASE(kBF16, __nv_bfloat16, kF16, __half, 4)
    MLXQ_ROUTE_CASE(kBF16, __nv_bfloat16, kF32, float, 5)
    MLXQ_ROUTE_CASE(kF16, __half, kBF16, __nv_bfloat16, 6)
    MLXQ_ROUTE_CASE(kF16, __half, kF16, __half, 7)
    MLXQ_ROUTE_CASE(kF16, __half, kF32, float, 8)
#undef MLXQ_ROUTE_CASE
    if (!f) return cudaErrorInvalidValue;
    const int warps_per_cta = 4;
    return launch_ex(f, cfg[which], dim3((T + warps_per_cta - 1) / warps_per_cta),
                     dim3(32 * warps_per_cta), 0, st, overlap, args);
}

// ------------------------------------------------------------------------------------
// Stable sort of MoE routing entries by expert (the argsort pair of _gather_sort,
// lfm2.py:613-618): order[p] = entry at sorted position p, sorted[p] = its expert,
// inverse[i] = sorted position of entry i. One CTA, a counting sort: entries are
// bucketed by clamp(v, -1, E) + 1 (values outside [0, E) form a bucket before and one
// after the experts, each in entry order); warp w owns the contiguous slice w of the
// entries and counts its buckets (shared-memory atomics), an exclusive scan over
// (bucket, warp) gives each warp's first position per bucket, and the warp then
// places its slice 32 entries at a time in order: lanes with the same bucket
// (match_any) take consecutive positions by lane.
constexpr int kMoeSortThreads = 1024;
constexpr int kMoeSortWarps = kMoeSortThreads / 32;

__global__ void __launch_bounds__(kMoeSortThreads) moe_sort_kernel(
    const int32_t* __restrict__ idx, int n, int E, int32_t* __restrict__ order,
    int32_t* __restrict__ sorted, int32_t* __restrict__ inverse) {
    extern __shared__ int ms_smem[];
    const int nb = E + 2;
    int* cnt = ms_smem;                       // [nb][warps]: counts, then first positions
    int* key = cnt + nb * kMoeSortWarps;      // [n] bucket of each entry
    __shared__ int wsum[kMoeSortWarps];
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int L = nb * kMoeSortWarps;
    for (int i = tid; i < L; i += kMoeSortThreads) cnt[i] = 0;
    __syncthreads();
    const int per = (n + kMoeSortWarps - 1) / kMoeSortWarps;
    const int lo = min(n, warp * per), hi = min(n, lo + per);
    for (int i = lo + lane; i < hi; i += 32) {
        const int k = max(-1, min(idx[i], E)) + 1;
        key[i] = k;
        atomicAdd(cnt + k * kMoeSortWarps + warp, 1);
    }
    __syncthreads();
    // exclusive scan of cnt in (bucket, warp) order: thread t scans a contiguous run
    {
        const int run = (L + kMoeSortThreads - 1) / kMoeSortThreads;
        const int r0 = min(L, tid * run), r1 = min(L, r0 + run);
        int sum = 0;
        for (int i = r0; i < r1; ++i) sum += cnt[i];
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) wsum[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int w = wsum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += v;
            }
            wsum[lane] = w;  // inclusive over warps
        }
        __syncthreads();
        int pos = incl - sum + (warp > 0 ? wsum[warp - 1] : 0);
        for (int i = r0; i < r1; ++i) {
            const int c = cnt[i];
            cnt[i] = pos;
            pos += c;
        }
    }
    __syncthreads();
    const unsigned below = (1u << lane) - 1u;
    for (int base = lo; base < hi; base += 32) {
        const int i = base + lane;
        const bool live = i < hi;
        const int k = live ? key[i] : -1 - lane;  // dead lanes match no one
        const unsigned same = __match_any_sync(0xffffffffu, k);
        if (live) {
            int* slot = cnt + k * kMoeSortWarps + warp;
            const int r = *slot + __popc(same & below);
            order[r] = i;
            sorted[r] = idx[i];
            inverse[i] = r;
        }
        __syncwarp();
        // the lowest lane of each bucket moves the warp's position on past its members
        if (live && (same & below) == 0) cnt[k * kMoeSortWarps + warp] += __popc(same);
        __syncwarp();
    }
}

size_t moe_sort_smem(int n, int E) {
    return static_cast<size_t>(n + (E + 2) * kMoeSortWarps) * sizeof(int);
}

cudaError_t launch_moe_sort(const int32_t* idx, int n, int E, int32_t* order, int32_t* sorted,
                            int32_t* inverse, bool overlap, cudaStream_t st) {
    void* args[] = {&idx, &n, &E, &order, &sorted, &inverse};
    static PerDevice cfg;
    return launch_ex(reinterpret_cast<const void*>(&moe_sort_kernel), cfg, dim3(1),
                     dim3(kMoeSortThreads), moe_sort_smem(n, E), st, overlap, args);
}

// ------------------------------------------------------------------------------------
// One decode step further for every sequence: the next token sits at position
// p + 1, the cache then holds p + 2 keys, and its slot is that position's place in
// the sequence's pages (-1 past the block table).
__global__ void decode_advance_kernel(int32_t* __restrict__ positions,
                                      int32_t* __restrict__ kv_lens, int32_t* __restrict__ slots,
                                      const int32_t* __restrict__ block_table, int max_blocks,
                                      int B, int page) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int p = positions[b] + 1;
    positions[b] = p;
    kv_lens[b] = p + 1;
    const int blk = p / page;
    slots[b] = blk < max_blocks
                   ? block_table[static_cast<size_t>(b) * max_blocks + blk] * page + p % page
                   : -1;
}

cudaError_t launch_decode_advance(int32_t* positions, int32_t* kv_lens, int32_t* slots,
                                  const int32_t* block_table, int max_blocks, int B, int page,
                                  bool overlap, cudaStream_t st) {
    void* args[] = {&positions, &kv_lens, &slots, &block_table, &max_blocks, &B, &page};
    static PerDevice cfg;
    return launch_ex(reinterpret_cast<const void*>(&decode_advance_kernel), cfg, dim3((B + 127) / 128),
                     dim3(128), 0, st, overlap, args);
}

}  // namespace mlxq
