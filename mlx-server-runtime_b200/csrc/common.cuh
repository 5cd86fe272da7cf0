// Shared device helpers for the sm_100a quantized-matmul kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mlxq {

// ---- element types -----------------------------------------------------------------------
// Per activation type: conversion helpers and the extraction that turns packed
// codes into exact 16-bit MMA operands without integer-to-float conversion. A
// field OR'ed into the mantissa of a 16-bit float with a fixed exponent gives
// offset + field exactly:
//   bf16 (7 mantissa bits): a nibble must sit at bits 0-3 of a half, so every
//     nibble position is shifted there first:  0x4300 | q = 128 + q,
//     0x4500 | q = 2048 + 16*q  (the high nibble of an 8-bit code).
//   f16 (10 mantissa bits): bits 0-3 and 4-7 both fit:  0x6400 | q = 1024 + q,
//     0x5400 | (q << 4) = 64 + q,  0x6400 | (q << 4) = 1024 + 16*q.
// extract<BITS>(w) returns four operands, each holding a pair of codes, in a
// fixed order the activation fragments mirror:
//   4-bit: nibble pairs (0,4) (1,5) (2,6) (3,7)
//   8-bit: (low nibbles of bytes 0,2) (high nibbles of bytes 0,2)
//          (low nibbles of bytes 1,3) (high nibbles of bytes 1,3)
// and the matmul over them equals sum x*q plus offsets times activation sums:
//   kUniform: every operand carries the same offset kOff (per code);
//   otherwise even code positions carry kOffE and odd positions kOffO.
// (a & MASK) | c as one LOP3 with the mask as its immediate and c a register.
template <uint32_t MASK>
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "n"(MASK), "r"(c));
    return r;
}

// A value the compiler cannot treat as a constant, so it stays in one register
// instead of being rebuilt from an immediate before every use.
__device__ __forceinline__ uint32_t opaque(uint32_t v) {
    asm volatile("" : "+r"(v));
    return v;
}

template <typename T>
struct Elem;

template <>
struct Elem<__nv_bfloat16> {
    // magic operands for extract(): kept in registers by the caller (see opaque())
    template <int BITS>
    struct Magic {
        static constexpr uint32_t kA = 0x43004300u;
        static constexpr uint32_t kB = (BITS == 4) ? 0x43004300u : 0x45004500u;
    };
    template <int BITS>
    static __device__ __forceinline__ void extract(uint32_t w, uint32_t (&t)[4], uint32_t ma,
                                                   uint32_t mb) {
        t[0] = lop_and_or<0x000F000Fu>(w, ma);
        t[1] = lop_and_or<0x000F000Fu>(w >> 4, mb);
        t[2] = lop_and_or<0x000F000Fu>(w >> 8, ma);
        t[3] = lop_and_or<0x000F000Fu>(w >> 12, mb);
    }
    template <int BITS>
    struct Off {
        static constexpr bool kUniform = true;
        static constexpr float kOff = (BITS == 4) ? 128.0f : 2176.0f;  // 128 + 2048
        static constexpr float kOffE = kOff, kOffO = kOff;
    };
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) {
        return __float2bfloat16_rn(v);
    }
    // the low / high 16-bit halves of a packed pair, as float
    static __device__ __forceinline__ float lo(uint32_t u) { return __uint_as_float(u << 16); }
    static __device__ __forceinline__ float hi(uint32_t u) {
        return __uint_as_float(u & 0xffff0000u);
    }
};

template <>
struct Elem<__half> {
    template <int BITS>
    struct Magic {
        static constexpr uint32_t kA = 0x64006400u;
        static constexpr uint32_t kB = (BITS == 4) ? 0x54005400u : 0x64006400u;
    };
    template <int BITS>
    static __device__ __forceinline__ void extract(uint32_t w, uint32_t (&t)[4], uint32_t ma,
                                                   uint32_t mb) {
        const uint32_t h = w >> 8;
        t[0] = lop_and_or<0x000F000Fu>(w, ma);
        t[1] = lop_and_or<0x00F000F0u>(w, mb);
        t[2] = lop_and_or<0x000F000Fu>(h, ma);
        t[3] = lop_and_or<0x00F000F0u>(h, mb);
    }
    template <int BITS>
    struct Off {
        static constexpr bool kUniform = (BITS == 8);
        static constexpr float kOffE = 1024.0f;
        static constexpr float kOffO = (BITS == 4) ? 64.0f : 1024.0f;
        static constexpr float kOff = (BITS == 4) ? 1024.0f : 2048.0f;  // uniform case only
    };
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
    static __device__ __forceinline__ float lo(uint32_t u) {
        return __half2float(__ushort_as_half(static_cast<unsigned short>(u & 0xffffu)));
    }
    static __device__ __forceinline__ float hi(uint32_t u) {
        return __half2float(__ushort_as_half(static_cast<unsigned short>(u >> 16)));
    }
};

template <>
struct Elem<float> {
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
};

// ---- tensor-core fragment MMA (m16n8k16, fp32 accumulate) -------------------------------
// Plain (non-volatile) asm: the instructions have no side effects beyond their
// outputs, so the compiler may interleave independent accumulation chains.
// mma16816z starts from a zero accumulator.
#define MLXQ_MMA_ASM(TY)                                                                         \
    "mma.sync.aligned.m16n8k16.row.col.f32." TY "." TY ".f32 "

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    if constexpr (__is_same(T, __nv_bfloat16)) {
        asm(MLXQ_MMA_ASM("bf16") "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm(MLXQ_MMA_ASM("f16") "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

template <typename T>
__device__ __forceinline__ void mma16816z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    const float z = 0.0f;
    if constexpr (__is_same(T, __nv_bfloat16)) {
        asm(MLXQ_MMA_ASM("bf16") "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
            : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
    } else {
        asm(MLXQ_MMA_ASM("f16") "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
            : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
    }
}

// ---- async copies (LDGSTS) ----------------------------------------------------------------
// src_bytes == 0 zero-fills the destination without reading global memory; the
// caller still passes an in-bounds source address.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, int src_bytes) {
    uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16, %2;\n" ::"r"(d), "l"(gsrc),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gsrc, int src_bytes) {
    uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(d), "l"(gsrc),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc, int src_bytes) {
    uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(gsrc),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Two floats rounded to f16, a in the low half.
__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// silu(gate) * up of the SwiGLU epilogues from the fp32 accumulators of a gate row and
// its up row: each projection rounded to T first (as two separate matmuls would write
// them), the activation in fp32, one more rounding.
template <typename T>
__device__ __forceinline__ T swiglu_out(float g, float u) {
    using ET = Elem<T>;
    const float gr = ET::to_f(ET::from_f(g)), ur = ET::to_f(ET::from_f(u));
    return ET::from_f(gr / (1.0f + expf(-gr)) * ur);
}

}  // namespace mlxq
