// quantize / dequantize kernels (MLX affine layout), bit-exact with the CPU
// restatement of MLX's algorithm.
//
// Layout: one thread owns one packed uint32 word (32/bits consecutive codes of
// a row); the group_size/(32/bits) threads of a group sit in adjacent lanes of
// one warp, so group min/max is a shuffle reduction and every load and store
// is coalesced. Both kernels are pure HBM streams (load-time work in the
// reference: mx.quantize at lfm2.py:112-117, nn.quantize at qwen2.py:318-324).
#include "common.cuh"
#include "launch.h"

namespace mlxq {

template <typename T, int BITS>
__global__ void __launch_bounds__(256) quantize_kernel(const T* __restrict__ w,
                                                       uint32_t* __restrict__ wq,
                                                       T* __restrict__ scales,
                                                       T* __restrict__ biases,
                                                       long long total_words, int lanes_per_group) {
    constexpr int EPW = 32 / BITS;
    const float n_bins = static_cast<float>((1 << BITS) - 1);
    const long long wi = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const bool live = wi < total_words;

    float v[EPW];
    float lmax = -INFINITY, lmin = INFINITY;
    if (live) {
        const T* src = w + wi * EPW;
#pragma unroll
        for (int e = 0; e < EPW; ++e) {
            v[e] = Elem<T>::to_f(src[e]);
            lmax = fmaxf(lmax, v[e]);
            lmin = fminf(lmin, v[e]);
        }
    }
    // Reduce over the lanes of this group (an aligned power-of-two segment of
    // the warp). Lanes past the end form whole segments of their own.
    for (int off = lanes_per_group >> 1; off > 0; off >>= 1) {
        lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, off));
        lmin = fminf(lmin, __shfl_xor_sync(0xffffffffu, lmin, off));
    }
    if (!live) return;

    const bool mask = fabsf(lmin) > fabsf(lmax);
    float scale = __fdiv_rn(__fsub_rn(lmax, lmin), n_bins);
    scale = fmaxf(scale, 1e-7f);
    scale = mask ? scale : -scale;
    const float edge = mask ? lmin : lmax;
    const float q0 = rintf(__fdiv_rn(edge, scale));
    float bias = 0.0f;
    if (q0 != 0.0f) {
        scale = __fdiv_rn(edge, q0);
        bias = edge;
    }
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < EPW; ++e) {
        float q = rintf(__fdiv_rn(__fsub_rn(v[e], bias), scale));
        q = fminf(fmaxf(q, 0.0f), n_bins);
        word |= static_cast<uint32_t>(q) << (BITS * e);
    }
    wq[wi] = word;
    if ((threadIdx.x & (lanes_per_group - 1)) == 0) {
        const long long g = wi / lanes_per_group;
        scales[g] = Elem<T>::from_f(scale);
        biases[g] = Elem<T>::from_f(bias);
    }
}

template <typename T, int BITS>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t* __restrict__ wq,
                                                         const T* __restrict__ scales,
                                                         const T* __restrict__ biases,
                                                         T* __restrict__ out,
                                                         long long total_words,
                                                         int words_per_group) {
    constexpr int EPW = 32 / BITS;
    const long long wi = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (wi >= total_words) return;
    const long long g = wi / words_per_group;
    const float s = Elem<T>::to_f(scales[g]);
    const float b = Elem<T>::to_f(biases[g]);
    const uint32_t word = wq[wi];
    T res[EPW];
#pragma unroll
    for (int e = 0; e < EPW; ++e) {
        const float q = static_cast<float>((word >> (BITS * e)) & ((1u << BITS) - 1u));
        // One rounding per operation, in the storage type: round(round(s*q) + b).
        const float t = Elem<T>::to_f(Elem<T>::from_f(__fmul_rn(s, q)));
        res[e] = Elem<T>::from_f(__fadd_rn(t, b));
    }
    T* dst = out + wi * EPW;
#pragma unroll
    for (int e = 0; e < EPW; ++e) dst[e] = res[e];
}

template <typename T>
static cudaError_t launch_quantize_t(const void* w, uint32_t* wq, void* s, void* b, long long rows,
                                     long long K, int gs, int bits, cudaStream_t st) {
    const long long words = rows * K * bits / 32;
    const int lanes = gs / (32 / bits);
    const unsigned blocks = static_cast<unsigned>((words + 255) / 256);
    if (words == 0) return cudaSuccess;
    const T* wt = static_cast<const T*>(w);
    T* st_ = static_cast<T*>(s);
    T* bt = static_cast<T*>(b);
    switch (bits) {
        case 2: quantize_kernel<T, 2><<<blocks, 256, 0, st>>>(wt, wq, st_, bt, words, lanes); break;
        case 4: quantize_kernel<T, 4><<<blocks, 256, 0, st>>>(wt, wq, st_, bt, words, lanes); break;
        case 8: quantize_kernel<T, 8><<<blocks, 256, 0, st>>>(wt, wq, st_, bt, words, lanes); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_dequantize_t(const uint32_t* wq, const void* s, const void* b, void* out,
                                       long long rows, long long K, int gs, int bits,
                                       cudaStream_t st) {
    const long long words = rows * K * bits / 32;
    const int wpg = gs * bits / 32;
    const unsigned blocks = static_cast<unsigned>((words + 255) / 256);
    if (words == 0) return cudaSuccess;
    const T* stt = static_cast<const T*>(s);
    const T* bt = static_cast<const T*>(b);
    T* o = static_cast<T*>(out);
    switch (bits) {
        case 2: dequantize_kernel<T, 2><<<blocks, 256, 0, st>>>(wq, stt, bt, o, words, wpg); break;
        case 4: dequantize_kernel<T, 4><<<blocks, 256, 0, st>>>(wq, stt, bt, o, words, wpg); break;
        case 8: dequantize_kernel<T, 8><<<blocks, 256, 0, st>>>(wq, stt, bt, o, words, wpg); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_quantize(const void* w, int dtype, uint32_t* wq, void* s, void* b,
                            long long rows, long long K, int gs, int bits, cudaStream_t st) {
    switch (dtype) {
        case kF32: return launch_quantize_t<float>(w, wq, s, b, rows, K, gs, bits, st);
        case kBF16: return launch_quantize_t<__nv_bfloat16>(w, wq, s, b, rows, K, gs, bits, st);
        case kF16: return launch_quantize_t<__half>(w, wq, s, b, rows, K, gs, bits, st);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_dequantize(const uint32_t* wq, const void* s, const void* b, int dtype,
                              void* out, long long rows, long long K, int gs, int bits,
                              cudaStream_t st) {
    switch (dtype) {
        case kF32: return launch_dequantize_t<float>(wq, s, b, out, rows, K, gs, bits, st);
        case kBF16:
            return launch_dequantize_t<__nv_bfloat16>(wq, s, b, out, rows, K, gs, bits, st);
        case kF16: return launch_dequantize_t<__half>(wq, s, b, out, rows, K, gs, bits, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace mlxq
