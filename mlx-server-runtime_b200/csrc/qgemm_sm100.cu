// Prefill-shaped group-wise affine quantized matmul on sm_100a: dequantize into
// shared memory, multiply with tcgen05 (5th-generation tensor cores, fp32
// accumulator in tensor memory).
//
//   out[m, n] = sum_k x[m, k] * (scale[n, k/g] * q[n, k] + bias[n, k/g])
//
// for M > 32 tokens (MLX's quantized_matmul as QuantizedLinear calls it during
// prefill, qwen2.py:58-61,123-134 of the reference).
//
// CTA tile: BM = 128 tokens x BN = 256 weight rows, K blocks of BK = 64, a
// 3-stage pipeline, 256 threads:
//   * x tiles [128 x 64] bf16 arrive by 16-byte cp.async into the canonical
//     K-major 128-byte-swizzled layout (8-row x 128-byte atoms, chunk c of row r
//     stored at chunk c ^ (r % 8)).
//   * Packed weight rows arrive by cp.async; thread t dequantizes row t of the
//     block: codes become exact 16-bit values with byte permutes and a magic
//     exponent (no integer-to-float conversion), then w = scale*q + bias with one
//     packed FMA (one rounding, like MLX's dequantize-in-kernel), stored in the
//     same swizzled layout.
//   * One thread issues tcgen05.mma (M=128, N=256, K=16) x 4 per K block from
//     shared-memory descriptors into a 128 x 256 fp32 accumulator in tensor
//     memory, then tcgen05.commit arrives on the stage's mbarrier; a stage is
//     refilled only after that barrier shows its MMAs finished.
//   * Epilogue: tcgen05.ld (32 lanes x 32 columns per warp) -> bf16/f16 ->
//     global, optional per-row bias added as a second rounding.
// Every mbarrier wait is bounded: on timeout the CTA records an error in
// g_qgemm_error, stops issuing work, waits (bounded) for what is in flight,
// frees its tensor memory and returns.
#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"

namespace mlxq {

__device__ int g_qgemm_error;  // 0, or the first error code a kernel recorded

namespace qg {
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 3, THREADS = 256;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kSpinLimit = 1u << 20;
constexpr int kErrTimeout = 1;
template <int BITS>
constexpr int raw_row_bytes() { return BK * BITS / 8; }  // 32 (4-bit) / 64 (8-bit)
template <int BITS>
constexpr int stage_bytes() { return A_BYTES + B_BYTES + BN * raw_row_bytes<BITS>(); }
template <int BITS>
constexpr int smem_bytes() { return STAGES * stage_bytes<BITS>() + 1024 + 128; }
}  // namespace qg

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address (16-byte units)
    d |= static_cast<uint64_t>(1) << 16;                   // leading byte offset (unused here)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;           // stride byte offset
    d |= static_cast<uint64_t>(1) << 46;                   // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;                   // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, A/B bf16 or f16, both K-major.
template <typename T>
__host__ __device__ constexpr uint32_t qgemm_idesc() {
    constexpr uint32_t ab = __is_same(T, __nv_bfloat16) ? 1u : 0u;
    return (1u << 4) | (ab << 7) | (ab << 10) | (static_cast<uint32_t>(qg::BN >> 3) << 17) |
           (static_cast<uint32_t>(qg::BM >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                     bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// Packed-pair helpers for the dequantization (T = bf16 or f16).
template <typename T>
struct Pair;
template <>
struct Pair<__nv_bfloat16> {
    static constexpr uint32_t kMagicLo = 0x43434343u;  // bytes 0x43: 0x43|q -> 128 + q
    static constexpr uint32_t kMagicHi = 0x45454545u;  // 0x45|q -> 2048 + 16*q
    static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
        __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a),
                                   *reinterpret_cast<__nv_bfloat162*>(&b));
        return *reinterpret_cast<uint32_t*>(&r);
    }
    static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
        __nv_bfloat162 r = __hadd2(*reinterpret_cast<__nv_bfloat162*>(&a),
                                   *reinterpret_cast<__nv_bfloat162*>(&b));
        return *reinterpret_cast<uint32_t*>(&r);
    }
    static __device__ __forceinline__ uint32_t fma(uint32_t a, uint32_t b, uint32_t c) {
        __nv_bfloat162 r = __hfma2(*reinterpret_cast<__nv_bfloat162*>(&a),
                                   *reinterpret_cast<__nv_bfloat162*>(&b),
                                   *reinterpret_cast<__nv_bfloat162*>(&c));
        return *reinterpret_cast<uint32_t*>(&r);
    }
    static constexpr uint32_t kOffLo = 0x43004300u;  // (128, 128)
    static constexpr uint32_t kOffHi = 0x45004500u;  // (2048, 2048)
};
template <>
struct Pair<__half> {
    static constexpr uint32_t kMagicLo = 0x64646464u;  // 0x64|q -> 1024 + q
    static constexpr uint32_t kMagicHi = 0x74747474u;  // 0x74|q -> 16384 + 16*q
    static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
        __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
        return *reinterpret_cast<uint32_t*>(&r);
    }
    static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
        __half2 r = __hadd2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
        return *reinterpret_cast<uint32_t*>(&r);
    }
    static __device__ __forceinline__ uint32_t fma(uint32_t a, uint32_t b, uint32_t c) {
        __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b),
                            *reinterpret_cast<__half2*>(&c));
        return *reinterpret_cast<uint32_t*>(&r);
    }
    static constexpr uint32_t kOffLo = 0x64006400u;  // (1024, 1024)
    static constexpr uint32_t kOffHi = 0x74007400u;  // (16384, 16384)
};

template <typename T>
__device__ __forceinline__ uint32_t splat(T v) {
    const uint16_t h = *reinterpret_cast<const uint16_t*>(&v);
    return static_cast<uint32_t>(h) | (static_cast<uint32_t>(h) << 16);
}

// 8 dequantized values (k0..k7 in order) from the 8 codes of one chunk.
// 4-bit: one word holds k0..k7 (nibble j = code k_j). 8-bit: two words, byte j = code.
template <typename T, int BITS>
__device__ __forceinline__ uint4 dequant_chunk(const uint32_t* wds, uint32_t s2, uint32_t b2,
                                               uint32_t mlo, uint32_t mhi) {
    using P = Pair<T>;
    uint32_t q[4];  // (k0,k1) (k2,k3) (k4,k5) (k6,k7) as exact 16-bit integers
    if constexpr (BITS == 4) {
        const uint32_t w = wds[0];
        const uint32_t t = w & 0x0F0F0F0Fu;         // nibbles 0,2,4,6 in bytes 0..3
        const uint32_t u = (w >> 4) & 0x0F0F0F0Fu;  // nibbles 1,3,5,7
        const uint32_t lo = prmt(t, u, 0x5140);     // bytes: n0 n1 n2 n3
        const uint32_t hi = prmt(t, u, 0x7362);     // bytes: n4 n5 n6 n7
        q[0] = P::sub(prmt(lo, mlo, 0x4140), P::kOffLo);  // (magic|n0, magic|n1) - offset
        q[1] = P::sub(prmt(lo, mlo, 0x4342), P::kOffLo);
        q[2] = P::sub(prmt(hi, mlo, 0x4140), P::kOffLo);
        q[3] = P::sub(prmt(hi, mlo, 0x4342), P::kOffLo);
    } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t w = wds[h];                 // bytes k(4h+0..3)
            const uint32_t t = w & 0x0F0F0F0Fu;        // low nibbles
            const uint32_t u = (w >> 4) & 0x0F0F0F0Fu; // high nibbles
            const uint32_t l01 = P::sub(prmt(t, mlo, 0x4140), P::kOffLo);
            const uint32_t l23 = P::sub(prmt(t, mlo, 0x4342), P::kOffLo);
            const uint32_t h01 = P::sub(prmt(u, mhi, 0x4140), P::kOffHi);
            const uint32_t h23 = P::sub(prmt(u, mhi, 0x4342), P::kOffHi);
            q[2 * h + 0] = P::add(l01, h01);  // ql + 16*qh, exact (<= 255)
            q[2 * h + 1] = P::add(l23, h23);
        }
    }
    uint4 r;
    r.x = P::fma(q[0], s2, b2);
    r.y = P::fma(q[1], s2, b2);
    r.z = P::fma(q[2], s2, b2);
    r.w = P::fma(q[3], s2, b2);
    return r;
}

template <typename T, int BITS, int GS>
__global__ void __launch_bounds__(qg::THREADS, 1) qgemm_kernel(const QgemmParams p) {
    using namespace qg;
    constexpr int SB = stage_bytes<BITS>();
    constexpr int RAWB = raw_row_bytes<BITS>();
    constexpr int WPR = RAWB / 4;  // packed words per row per K block
    constexpr uint32_t IDESC = qgemm_idesc<T>();

    extern __shared__ uint8_t qg_smem_raw[];
    const uint32_t raw_base = smem_u32(qg_smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* smem = qg_smem_raw + (base - raw_base);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * SB);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + STAGES);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const int M = p.M, N = p.N, K = p.K;
    const long long kw = static_cast<long long>(K) * BITS / 32;
    const int KB = K / BK;
    const int G = K / GS;
    const T* xg = static_cast<const T*>(p.x);
    const T* sg = static_cast<const T*>(p.s);
    const T* bg = static_cast<const T*>(p.b);

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
    }
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(smem_u32(bars + s), 1);
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    // this thread's weight row
    const int wn = n0 + tid;
    const bool wrow_ok = wn < N;
    const uint32_t* wrow = p.w + (wrow_ok ? static_cast<long long>(wn) * kw : 0);

    auto load_stage = [&](int kb, int s) {
        uint8_t* st = smem + s * SB;
        // x tile: 1024 16-byte units, 4 per thread, swizzled
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int u = tid + THREADS * i;
            const int row = u >> 3, c = u & 7;
            const int tok = m0 + row;
            const bool ok = tok < M;
            const T* src = ok ? xg + static_cast<long long>(tok) * K + kb * BK + c * 8 : xg;
            cp_async16(st + (row >> 3) * 1024 + (row & 7) * 128 + ((c ^ (row & 7)) << 4), src,
                       ok ? 16 : 0);
        }
        // packed weights of this thread's row
        uint8_t* rdst = st + A_BYTES + B_BYTES + tid * RAWB;
        const uint32_t* rsrc = wrow + static_cast<long long>(kb) * WPR;
#pragma unroll
        for (int j = 0; j < RAWB / 16; ++j)
            cp_async16(rdst + 16 * j, wrow_ok ? rsrc + 4 * j : p.w, wrow_ok ? 16 : 0);
        cp_async_commit();
    };

    // scales / biases of this thread's row for K block kb (one or two groups)
    auto load_sb = [&](int kb, uint32_t (&s2)[2], uint32_t (&b2)[2]) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int g = (kb * BK + h * 32) / GS;
            T sv = T(0.0f), bv = T(0.0f);
            if (wrow_ok && kb < KB) {
                sv = sg[static_cast<long long>(wn) * G + g];
                bv = bg[static_cast<long long>(wn) * G + g];
            }
            s2[h] = splat(sv);
            b2[h] = splat(bv);
        }
    };

#pragma unroll
    for (int i = 0; i < STAGES - 1; ++i) {
        if (i < KB) load_stage(i, i);
        else cp_async_commit();
    }
    uint32_t s2[2], b2[2];
    load_sb(0, s2, b2);
    const uint32_t mlo = opaque(Pair<T>::kMagicLo), mhi = opaque(Pair<T>::kMagicHi);
    bool aborted = false;

    for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % STAGES;
        uint8_t* st = smem + s * SB;
        uint32_t ns2[2], nb2[2];
        load_sb(kb + 1, ns2, nb2);  // next block's scales, hidden behind this block

        cp_async_wait<STAGES - 2>();
        // dequantize this thread's row into the swizzled B tile
        {
            uint32_t raw[WPR];
            const uint4* rsrc = reinterpret_cast<const uint4*>(st + A_BYTES + B_BYTES + tid * RAWB);
#pragma unroll
            for (int j = 0; j < WPR / 4; ++j) {
                const uint4 v = rsrc[j];
                raw[4 * j] = v.x; raw[4 * j + 1] = v.y; raw[4 * j + 2] = v.z; raw[4 * j + 3] = v.w;
            }
            uint8_t* bdst = st + A_BYTES + (tid >> 3) * 1024 + (tid & 7) * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int h = (c * 8 >= 32) ? 1 : 0;  // which half of the block (group for g32)
                const uint4 v = dequant_chunk<T, BITS>(&raw[c * (BITS == 4 ? 1 : 2)], s2[h], b2[h],
                                                      mlo, mhi);
                *reinterpret_cast<uint4*>(bdst + ((c ^ (tid & 7)) << 4)) = v;
            }
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
        __syncthreads();
        if (*s_abort) {
            aborted = true;
            break;
        }
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const uint64_t adesc = sw128_kmajor_desc(smem_u32(st));
            const uint64_t bdesc = sw128_kmajor_desc(smem_u32(st + A_BYTES));
#pragma unroll
            for (int j = 0; j < BK / 16; ++j)  // advance 32 bytes (16 elements) per step
                umma_f16(tmem, adesc + 2 * j, bdesc + 2 * j, IDESC, (kb > 0 || j > 0) ? 1u : 0u);
            umma_commit(smem_u32(bars + s));
        }
        // refill the stage MMA(kb-1) used with K block kb + STAGES - 1
        if (kb + STAGES - 1 < KB) {
            if (kb >= 1) {
                const int ps = (kb - 1) % STAGES;
                if (!mbar_wait_bounded(smem_u32(bars + ps), ((kb - 1) / STAGES) & 1, kSpinLimit)) {
                    *s_abort = 1;
                    atomicCAS(&g_qgemm_error, 0, kErrTimeout);
                }
            }
            load_stage(kb + STAGES - 1, (kb + STAGES - 1) % STAGES);
        } else {
            cp_async_commit();
        }
        s2[0] = ns2[0]; s2[1] = ns2[1];
        b2[0] = nb2[0]; b2[1] = nb2[1];
    }

    // wait for the last MMA, then read the accumulator out of tensor memory
    bool done = !aborted && KB > 0;
    if (done) {
        const int ls = (KB - 1) % STAGES;
        if (!mbar_wait_bounded(smem_u32(bars + ls), ((KB - 1) / STAGES) & 1, kSpinLimit)) {
            atomicCAS(&g_qgemm_error, 0, kErrTimeout);
            done = false;
        }
    }
    cp_async_wait<0>();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    done = __syncthreads_and(done ? 1 : 0) != 0;
    if (done) {
        const int quarter = warp & 3, half = warp >> 2;
        const int tok = m0 + quarter * 32 + lane;
        T* og = static_cast<T*>(p.out);
        const T* biasg = static_cast<const T*>(p.bias);
#pragma unroll 1
        for (int i = 0; i < 4; ++i) {
            const int col = half * 128 + i * 32;
            uint32_t r[32];
            tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + col, r);
            const int n = n0 + col;
            if (tok < M && n < N) {
                T y[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    y[e] = Elem<T>::from_f(__uint_as_float(r[e]));
                    if (biasg && n + e < N)
                        y[e] = Elem<T>::from_f(Elem<T>::to_f(y[e]) + Elem<T>::to_f(biasg[n + e]));
                }
                T* dst = og + static_cast<long long>(tok) * N + n;
                if ((N & 7) == 0 && n + 32 <= N) {
#pragma unroll
                    for (int v = 0; v < 4; ++v)
                        reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(y)[v];
                } else {
                    for (int e = 0; e < 32 && n + e < N; ++e) dst[e] = y[e];
                }
            }
        }
    } else if (!aborted) {
        // nothing to read (K == 0 is rejected on the host) or the last wait timed out
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                     "r"(kTmemCols));
    }
}

template <typename T, int BITS, int GS>
static cudaError_t qgemm_launch_t(const QgemmParams& p, cudaStream_t st) {
    auto kern = qgemm_kernel<T, BITS, GS>;
    constexpr int smem = qg::smem_bytes<BITS>();
    static int configured[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    dim3 grid((p.M + qg::BM - 1) / qg::BM, (p.N + qg::BN - 1) / qg::BN, 1);
    kern<<<grid, qg::THREADS, smem, st>>>(p);
    return cudaGetLastError();
}

template <typename T>
static cudaError_t qgemm_dtype(int bits, int gs, const QgemmParams& p, cudaStream_t st) {
    if (bits == 4) {
        if (gs == 32) return qgemm_launch_t<T, 4, 32>(p, st);
        if (gs == 64) return qgemm_launch_t<T, 4, 64>(p, st);
        if (gs == 128) return qgemm_launch_t<T, 4, 128>(p, st);
    } else if (bits == 8) {
        if (gs == 32) return qgemm_launch_t<T, 8, 32>(p, st);
        if (gs == 64) return qgemm_launch_t<T, 8, 64>(p, st);
        if (gs == 128) return qgemm_launch_t<T, 8, 128>(p, st);
    }
    return cudaErrorInvalidValue;
}

bool qgemm_supported(int M, int N, int K, int bits, int gs) {
    (void)N;
    return M > 32 && K % qg::BK == 0 && (bits == 4 || bits == 8) &&
           (gs == 32 || gs == 64 || gs == 128);
}

cudaError_t qgemm_launch(int dtype, int bits, int gs, const QgemmParams& p, cudaStream_t st) {
    if (dtype == kBF16) return qgemm_dtype<__nv_bfloat16>(bits, gs, p, st);
    if (dtype == kF16) return qgemm_dtype<__half>(bits, gs, p, st);
    return cudaErrorInvalidValue;
}

cudaError_t qgemm_read_error(int* out_code) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_qgemm_error, sizeof(int));
    if (e != cudaSuccess) return e;
    if (v != 0) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_qgemm_error, &zero, sizeof(int));
    }
    *out_code = v;
    return e;
}

}  // namespace mlxq
