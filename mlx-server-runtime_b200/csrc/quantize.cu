// quantize / dequantize kernels (MLX affine layout), bit-exact with the CPU
// restatement of MLX's algorithm.
//
// quantize: one thread owns one packed uint32 word (32/bits consecutive codes of a
// row), loaded as one or two 16-byte vectors; the group_size/(32/bits) threads of a
// group sit in adjacent lanes of one warp, so group min/max is a shuffle reduction.
// dequantize: each lane expands four words strided by 32, so a warp's loads and its
// vector stores cover contiguous spans. Both kernels are HBM streams (load-time work
// in the reference: mx.quantize at lfm2.py:112-117, nn.quantize at qwen2.py:318-324).
#include "common.cuh"
#include "launch.h"

namespace mlxq {

// 32-bit words of packed elements: two 16-bit values (low half first) or one float.
template <typename T>
struct Packed {
    static constexpr int kPerWord = sizeof(T) == 2 ? 2 : 1;
    static __device__ __forceinline__ float get(uint32_t u, int i) {
        if constexpr (sizeof(T) == 4) {
            return __uint_as_float(u);
        } else {
            return i == 0 ? Elem<T>::lo(u) : Elem<T>::hi(u);
        }
    }
    static __device__ __forceinline__ uint32_t bits(T v) {
        if constexpr (sizeof(T) == 4) {
            return __float_as_uint(v);
        } else {
            return static_cast<uint32_t>(*reinterpret_cast<const unsigned short*>(&v));
        }
    }
};

// N consecutive 32-bit words (N in {2, 4, 8, 16}) from / to an address aligned to
// min(4 N, 16) bytes, as 8- or 16-byte accesses with the streaming cache hint: the
// data is touched once.
template <int N>
__device__ __forceinline__ void load_words(const void* p, uint32_t (&r)[N]) {
    if constexpr (N == 2) {
        const uint2 v = __ldcs(reinterpret_cast<const uint2*>(p));
        r[0] = v.x;
        r[1] = v.y;
    } else {
#pragma unroll
        for (int i = 0; i < N / 4; ++i) {
            const uint4 v = __ldcs(reinterpret_cast<const uint4*>(p) + i);
            r[4 * i] = v.x;
            r[4 * i + 1] = v.y;
            r[4 * i + 2] = v.z;
            r[4 * i + 3] = v.w;
        }
    }
}

template <int N>
__device__ __forceinline__ void store_words(void* p, const uint32_t (&r)[N]) {
    if constexpr (N == 2) {
        __stcs(reinterpret_cast<uint2*>(p), make_uint2(r[0], r[1]));
    } else {
#pragma unroll
        for (int i = 0; i < N / 4; ++i)
            __stcs(reinterpret_cast<uint4*>(p) + i,
                   make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]));
    }
}

// The code of one element, clamp(rint(RN(d / s)), 0, n_bins) with RN the IEEE
// quotient, from r = RN(1 / s): q = RN(d * r) is within (2^-23 + 2^-48) |d / s| of
// d / s, and RN(d / s) within 2^-24 |d / s|, so for |q| <= 1024 the two differ by
// less than 2e-4. When q is more than 1e-3 from every half-integer, both round to
// the same integer; otherwise (or when q is outside [-1024, 1024], not a number, or
// r is not a normal float: `fast` false) the IEEE quotient is taken.
// Rounding to an integer adds and subtracts 1.5 * 2^23 (a float in [2^23, 2^24) has
// unit spacing, and the add rounds to nearest even like rintf for |q| < 2^22), and the
// clamped integer is read from the low mantissa bits of the same sum: no conversion
// instructions on the common path.
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23
constexpr uint32_t kRoundMagicBits = 0x4B400000u;

__device__ __forceinline__ uint32_t quant_code(float d, float s, float r, float n_bins, bool fast) {
    const float q = __fmul_rn(d, r);
    float k = __fsub_rn(__fadd_rn(q, kRoundMagic), kRoundMagic);
    if (!fast || !(fabsf(q) <= 1024.0f) || fabsf(__fsub_rn(q, k)) > 0.499f)
        k = rintf(__fdiv_rn(d, s));
    k = fminf(fmaxf(k, 0.0f), n_bins);
    return __float_as_uint(__fadd_rn(k, kRoundMagic)) - kRoundMagicBits;
}

// One thread quantizes WPT consecutive packed words (WPT * 32/bits elements, all in
// one group); the group_size / (WPT * 32/bits) threads of a group sit in adjacent
// lanes, so group min/max is a shuffle reduction over them, and the group's scale
// and bias (three IEEE divisions) are worked out once per WPT words.
template <typename T, int BITS, int WPT>
__global__ void __launch_bounds__(256) quantize_kernel(const T* __restrict__ w,
                                                       uint32_t* __restrict__ wq,
                                                       T* __restrict__ scales,
                                                       T* __restrict__ biases,
                                                       long long total_words, int lanes_per_group,
                                                       int log2_lanes) {
    constexpr int EPW = 32 / BITS;
    constexpr int NW = EPW / Packed<T>::kPerWord;  // input words per packed word
    const float n_bins = static_cast<float>((1 << BITS) - 1);
    const long long ti = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long wi = ti * WPT;  // first packed word (total_words is a multiple of WPT)
    const bool live = wi < total_words;

    float v[WPT][EPW];
    float lmax = -INFINITY, lmin = INFINITY;
    if (live) {
        uint32_t raw[WPT][NW];
#pragma unroll
        for (int j = 0; j < WPT; ++j) load_words<NW>(w + (wi + j) * EPW, raw[j]);
#pragma unroll
        for (int j = 0; j < WPT; ++j)
#pragma unroll
            for (int e = 0; e < EPW; ++e) {
                v[j][e] = Packed<T>::get(raw[j][e / Packed<T>::kPerWord], e % Packed<T>::kPerWord);
                lmax = fmaxf(lmax, v[j][e]);
                lmin = fminf(lmin, v[j][e]);
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
    const float r = __frcp_rn(scale);
    const float ar = fabsf(r);
    const bool fast = ar >= 0x1p-126f && ar <= 0x1p126f;
#pragma unroll
    for (int j = 0; j < WPT; ++j) {
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < EPW; ++e) {
            word |= quant_code(__fsub_rn(v[j][e], bias), scale, r, n_bins, fast) << (BITS * e);
        }
        __stcs(wq + wi + j, word);
    }
    if ((threadIdx.x & (lanes_per_group - 1)) == 0) {
        const long long g = ti >> log2_lanes;
        scales[g] = Elem<T>::from_f(scale);
        biases[g] = Elem<T>::from_f(bias);
    }
}

// Each warp expands 32 * WPT consecutive packed words; lane l takes words
// l, l + 32, ... of that run, so every load (4 bytes a lane) and every store
// (EPW elements a lane) of the warp covers one contiguous span.
constexpr int kDequantWPT = 4;

template <typename T, int BITS>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t* __restrict__ wq,
                                                         const T* __restrict__ scales,
                                                         const T* __restrict__ biases,
                                                         T* __restrict__ out,
                                                         long long total_words,
                                                         int log2_words_per_group) {
    constexpr int EPW = 32 / BITS;
    constexpr int NW = EPW / Packed<T>::kPerWord;  // output words per packed word
    const int lane = threadIdx.x & 31;
    const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const long long base = warp * (32 * kDequantWPT) + lane;
    uint32_t word[kDequantWPT];
    float s[kDequantWPT], b[kDequantWPT];
#pragma unroll
    for (int j = 0; j < kDequantWPT; ++j) {
        const long long wi = base + 32 * j;
        if (wi < total_words) {
            const long long g = wi >> log2_words_per_group;
            word[j] = __ldcs(wq + wi);
            s[j] = Elem<T>::to_f(scales[g]);
            b[j] = Elem<T>::to_f(biases[g]);
        }
    }
#pragma unroll
    for (int j = 0; j < kDequantWPT; ++j) {
        const long long wi = base + 32 * j;
        if (wi >= total_words) break;
        uint32_t res[NW];
#pragma unroll
        for (int i = 0; i < NW; ++i) res[i] = 0;
#pragma unroll
        for (int e = 0; e < EPW; ++e) {
            const float q = static_cast<float>((word[j] >> (BITS * e)) & ((1u << BITS) - 1u));
            // One rounding per operation, in the storage type: round(round(s*q) + b).
            const float t = Elem<T>::to_f(Elem<T>::from_f(__fmul_rn(s[j], q)));
            const uint32_t r = Packed<T>::bits(Elem<T>::from_f(__fadd_rn(t, b[j])));
            res[e / Packed<T>::kPerWord] |= r << (16 * (e % Packed<T>::kPerWord));
        }
        store_words<NW>(out + wi * EPW, res);
    }
}

static int log2_exact(int v) {
    int l = 0;
    while ((1 << l) < v) ++l;
    return l;
}

// Packed words per quantize thread: four (one 64-byte span of bf16 weights at 4 bits)
// unless a group has fewer.
constexpr int kQuantWPT = 4;

template <typename T, int BITS>
static cudaError_t launch_quantize_b(const T* w, uint32_t* wq, T* s, T* b, long long words,
                                     int gs, cudaStream_t st) {
    const int wpg = gs / (32 / BITS);  // packed words per group
    if (wpg >= kQuantWPT) {
        const int lanes = wpg / kQuantWPT;
        const long long threads = words / kQuantWPT;
        const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
        quantize_kernel<T, BITS, kQuantWPT>
            <<<blocks, 256, 0, st>>>(w, wq, s, b, words, lanes, log2_exact(lanes));
    } else {
        const unsigned blocks = static_cast<unsigned>((words + 255) / 256);
        quantize_kernel<T, BITS, 1><<<blocks, 256, 0, st>>>(w, wq, s, b, words, wpg,
                                                            log2_exact(wpg));
    }
    return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_quantize_t(const void* w, uint32_t* wq, void* s, void* b, long long rows,
                                     long long K, int gs, int bits, cudaStream_t st) {
    const long long words = rows * K * bits / 32;
    if (words == 0) return cudaSuccess;
    const T* wt = static_cast<const T*>(w);
    T* st_ = static_cast<T*>(s);
    T* bt = static_cast<T*>(b);
    switch (bits) {
        case 2: return launch_quantize_b<T, 2>(wt, wq, st_, bt, words, gs, st);
        case 4: return launch_quantize_b<T, 4>(wt, wq, st_, bt, words, gs, st);
        case 8: return launch_quantize_b<T, 8>(wt, wq, st_, bt, words, gs, st);
        default: return cudaErrorInvalidValue;
    }
}

template <typename T>
static cudaError_t launch_dequantize_t(const uint32_t* wq, const void* s, const void* b, void* out,
                                       long long rows, long long K, int gs, int bits,
                                       cudaStream_t st) {
    const long long words = rows * K * bits / 32;
    const int lw = log2_exact(gs * bits / 32);
    const long long per_block = 256LL * kDequantWPT;
    const unsigned blocks = static_cast<unsigned>((words + per_block - 1) / per_block);
    if (words == 0) return cudaSuccess;
    const T* stt = static_cast<const T*>(s);
    const T* bt = static_cast<const T*>(b);
    T* o = static_cast<T*>(out);
    switch (bits) {
        case 2: dequantize_kernel<T, 2><<<blocks, 256, 0, st>>>(wq, stt, bt, o, words, lw); break;
        case 4: dequantize_kernel<T, 4><<<blocks, 256, 0, st>>>(wq, stt, bt, o, words, lw); break;
        case 8: dequantize_kernel<T, 8><<<blocks, 256, 0, st>>>(wq, stt, bt, o, words, lw); break;
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
