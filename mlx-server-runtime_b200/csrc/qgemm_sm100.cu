// Prefill-shaped group-wise affine quantized matmul on sm_100a: dequantize into
// shared memory, multiply with tcgen05 (5th-generation tensor cores, fp32
// accumulator in tensor memory).
//
//   out[m, n] = sum_k x[m, k] * (scale[n, k/g] * q[n, k] + bias[n, k/g])
//
// for M > 32 tokens (MLX's quantized_matmul as QuantizedLinear calls it during
// prefill, qwen2.py:58-61,123-134 of the reference).
//
// Output tiles BW = 128 weight rows x BT = 192 tokens (128 for experts' row segments),
// K blocks of BK = 64; one
// persistent CTA per SM with specialized warps (see qgemm_kernel):
//   * TMA brings the activation tile in the canonical K-major 128-byte-swizzled
//     layout (8-row x 128-byte atoms, chunk c of row r at chunk c ^ (r % 8)) that the
//     MMA reads as its B operand, and the raw packed codes of the 128 weight rows.
//   * DQ warps per tensor-memory lane quarter take turns by K block (one K block each,
//     all 64 codes of a row per thread, so DQ K blocks are dequantized at once): codes
//     become exact 16-bit
//     values with byte permutes and a magic exponent (no integer-to-float
//     conversion), then w = scale*q + bias with one packed FMA (one rounding, like
//     MLX's dequantize-in-kernel), stored straight into tensor memory as the MMA's
//     A operand (weight row = lane).
//   * One thread issues tcgen05.mma (M=128, N=192, K=16; A from tensor memory, B
//     from a shared-memory descriptor) into one of two 128 x 192 fp32 accumulators.
//   * Epilogue warps read the finished accumulator (tcgen05.ld; thread = weight row,
//     32 tokens per load) while the other one fills: bf16/f16, optional bias added
//     as a second rounding.
// Every mbarrier wait is bounded: on timeout the CTA records an error in
// g_qgemm_error, its roles stop issuing work, the loads and MMAs in flight are
// waited for (bounded), tensor memory is freed and the kernel returns.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"

namespace mlxq {

__device__ int g_qgemm_error;  // 0, or the first error code a kernel recorded

namespace qg {
constexpr int BW = 128;  // weight rows per tile: MMA M, tensor-memory lanes
constexpr int BT_DENSE = 192, BT_GROUPED = 128;  // tokens per tile (MMA N): dense / experts
constexpr int BK = 64;
constexpr int ASTAGES = 4;                      // dequantized weight tiles in tensor memory
constexpr int DQ = 2;                           // dequant warps per tensor-memory lane quarter
constexpr int NDEQ = 4 * DQ, NEPI = 4;          // dequant / epilogue warps
constexpr int WARP_TMA = 0, WARP_MMA = 1, WARP_EPI0 = 2, WARP_DEQ0 = WARP_EPI0 + NEPI;
constexpr int THREADS = (WARP_DEQ0 + NDEQ) * 32;
static_assert(DQ == 1 || DQ == 2 || DQ == 4, "dequant warps per lane quarter (a K block each)");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kACols = BK / 2;     // 32-bit columns per A stage (two 16-bit values each)
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr int kErrTimeout = 1;
// suspending barrier waits: up to kParkLimit waits of about kParkNs each (~4 s)
constexpr uint32_t kParkNs = 2000, kParkLimit = 1u << 21;
template <int BITS>
constexpr int raw_bytes() { return BW * BK * BITS / 8; }  // 4 KB (4-bit) / 8 KB (8-bit)
template <int BITS>
constexpr int load_stages() { return 6; }
// A dequant warp waits on the load stages (and A stages) of its own K blocks only
// (K block index % DQ == its turn); with both rings multiples of DQ, the stage of its
// next K block last held one of its own, whose phase it has seen complete, so its
// parity wait can never match an older phase.
static_assert(load_stages<4>() % DQ == 0 && load_stages<8>() % DQ == 0 && ASTAGES % DQ == 0,
              "load and A rings must be multiples of DQ");
template <int BITS, int BT>
constexpr int smem_bytes() {
    return load_stages<BITS>() * (BT * BK * 2 + raw_bytes<BITS>()) +
           (2 * load_stages<BITS>() + 2 * ASTAGES + 7) * 8 + 16 + 1024;
}
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

// Instruction descriptor, kind::f16: fp32 accumulate, A/B bf16 or f16, both K-major,
// M = BW, N = BT.
template <typename T, int BT>
__host__ __device__ constexpr uint32_t qgemm_idesc() {
    constexpr uint32_t ab = __is_same(T, __nv_bfloat16) ? 1u : 0u;
    return (1u << 4) | (ab << 7) | (ab << 10) | (static_cast<uint32_t>(BT >> 3) << 17) |
           (static_cast<uint32_t>(qg::BW >> 4) << 24);
}

// D (tensor memory) (+)= A (tensor memory) * B (shared-memory descriptor)
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// 8 consecutive 32-bit columns of this thread's tensor-memory lane
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
        : "memory");
}

// 16 consecutive 32-bit columns of this thread's tensor-memory lane
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15])
        : "memory");
}

// 32 consecutive 32-bit columns of this thread's tensor-memory lane
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
        "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
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

// 16-byte read-only global load issued exactly here (volatile asm: the compiler
// may not sink it to the first use, so a prefetch made a whole chunk ahead keeps
// its distance).
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
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

// Persistent, warp-specialized prefill kernel. One CTA per SM walks its share of
// the output tiles (BW = 128 weight rows x BT tokens); per K block of 64:
//   warp 0  (TMA)      the activation tile [BT tokens x 64] (128-byte swizzle: the
//                      MMA's K-major B layout) and the raw packed codes of the tile's
//                      128 weight rows, into a ring of load stages;
//   dequant warps      thread = weight row: DQ warps share each tensor-memory lane
//                      quarter (w % 4) and take its K blocks in turn (warp j: blocks
//                      j, j + DQ, ...), so DQ K blocks are in flight at once; w =
//                      scale*q + bias goes straight into a ring of A tiles in tensor
//                      memory (tcgen05.st), never through shared memory;
//   warp 1  (MMA)      one thread issues tcgen05.mma M=128 N=BT K=16 x 4 with A from
//                      tensor memory into one of two accumulators and commits the load
//                      stage and the A tile back to their producers;
//   warps 2-5 (epilogue) drain the other accumulator (thread = weight row, columns =
//                      tokens) while the next tile accumulates; optional bias as a
//                      second rounding.
// EPI 1: SwiGLU over gate/up rows interleaved by 16-row tiles (whole tiles only): the
// gate row r and up row r + 8 of a tile are tensor-memory lanes l and l ^ 8 of one warp;
// the gate lane writes silu(gate) * up to column 8 j + r of the N / 2 outputs.
template <typename T, int BITS, int GS, int BT, bool SK, int EPI = 0>
__global__ void __launch_bounds__(qg::THREADS, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw,
                 const QgemmParams p) {
    using namespace qg;
    constexpr int LS = load_stages<BITS>();
    constexpr int RAW = raw_bytes<BITS>();
    constexpr int X_BYTES = BT * BK * 2;  // activation tile
    constexpr int LSB = X_BYTES + RAW;    // bytes of one load stage
    constexpr uint32_t kACol0 = 2 * BT;   // first A stage column (after two accumulators)
    static_assert(kACol0 + ASTAGES * kACols <= kTmemCols, "tensor memory budget");
    constexpr int WPR = BK * BITS / 32;   // packed words per row per K block
    constexpr uint32_t IDESC = qgemm_idesc<T, BT>();

    extern __shared__ uint8_t qg_smem_raw[];
    uint8_t* smem = qg_smem_raw + ((1024u - (smem_u32(qg_smem_raw) & 1023u)) & 1023u);
    uint64_t* load_full = reinterpret_cast<uint64_t*>(smem + LS * LSB);
    uint64_t* load_empty = load_full + LS;
    uint64_t* a_full = load_empty + LS;
    uint64_t* a_empty = a_full + ASTAGES;
    uint64_t* acc_full = a_empty + ASTAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* mma_done = acc_empty + 2;
    uint64_t* epi_done = mma_done + 1;  // stream-K: the epilogue warps stored a partial
    uint64_t* tk_done = epi_done + 1;   // stream-K: the tile's ticket was taken
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tk_done + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* s_last = s_abort + 1;  // stream-K: this CTA finishes the tile

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = p.M, N = p.N, K = p.K;
    const int KB = K / BK;
    const int MB = (M + BT - 1) / BT, NB = (N + BW - 1) / BW;
    const bool grouped = p.E > 0;
    const int tiles = grouped ? p.tile_start[p.E] : MB * NB;
    // Output tile t: expert, first token row, end of the expert's rows, weight block.
    struct Tile {
        int e, row0, row_end, nb;
    };
    auto tile_of = [&](int t) -> Tile {
        // dense whole tiles: weight block fastest (CTA b keeps weight block b when the
        // blocks match the grid, and the CTAs sweep the token blocks together, so the
        // activations in use stay in L2); stream-K: token block fastest (a share then
        // covers consecutive tiles of one weight block)
        if (!grouped)
            return SK ? Tile{0, (t % MB) * BT, M, t / MB} : Tile{0, (t / NB) * BT, M, t % NB};
        int lo = 0, hi = p.E - 1;  // last expert whose first tile is <= t
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.tile_start[mid] <= t) lo = mid;
            else hi = mid - 1;
        }
        const int lt = t - p.tile_start[lo];
        const int r0 = p.seg[lo] * p.rpe;
        const int rows = max(0, p.seg[lo + 1] * p.rpe - r0);
        const int mbe = max(1, (rows + BT - 1) / BT);
        return Tile{lo, r0 + (lt % mbe) * BT, r0 + rows, lt / mbe};
    };
    // This CTA's work as segments: tile t, K blocks [kb0, kb1). Data-parallel: whole
    // tiles blockIdx.x, + gridDim.x, ...; stream-K: an equal contiguous share of the
    // tiles x K blocks, so its first and last tiles may be partial. (32-bit: the host
    // runs stream-K only while units x CTAs stays below 2^31.)
    const unsigned U = static_cast<unsigned>(tiles) * static_cast<unsigned>(KB);
    const unsigned P = gridDim.x;
    const unsigned u_lo = SK ? U * blockIdx.x / P : 0u;
    const unsigned u_hi = SK ? U * (blockIdx.x + 1) / P : 0u;
    struct Seg {
        int t, kb0, kb1;
        unsigned u;  // stream-K: index of the segment's first K block
    };
    auto sk_seg = [&](unsigned u) -> Seg {
        const int kb0 = static_cast<int>(u % static_cast<unsigned>(KB));
        const unsigned left = u_hi - u;
        return Seg{static_cast<int>(u / static_cast<unsigned>(KB)), kb0,
                   left < static_cast<unsigned>(KB - kb0) ? kb0 + static_cast<int>(left) : KB, u};
    };
    auto seg_first = [&]() -> Seg {
        return SK ? sk_seg(u_lo) : Seg{static_cast<int>(blockIdx.x), 0, KB, 0u};
    };
    auto seg_valid = [&](const Seg& g) -> bool { return SK ? g.u < u_hi : g.t < tiles; };
    auto seg_next = [&](const Seg& g) -> Seg {
        return SK ? sk_seg(g.u + static_cast<unsigned>(g.kb1 - g.kb0))
                    : Seg{g.t + static_cast<int>(P), 0, KB, 0u};
    };
    // stream-K: the CTA that owns K block u of the tiles x K blocks sequence
    auto owner = [&](unsigned u) -> int { return static_cast<int>(((u + 1) * P - 1) / U); };

    if (warp == WARP_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
    }
    if (tid == 0) {
        for (int s = 0; s < LS; ++s) {
            mbar_init(smem_u32(load_full + s), 1);
            mbar_init(smem_u32(load_empty + s), 4 + 1);  // its K block's 4 dequant warps + MMA
        }
        for (int a = 0; a < ASTAGES; ++a) {
            mbar_init(smem_u32(a_full + a), 4);  // one dequant warp per lane quarter
            mbar_init(smem_u32(a_empty + a), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(acc_full + a), 1);
            mbar_init(smem_u32(acc_empty + a), NEPI);
        }
        mbar_init(smem_u32(mma_done), 1);
        mbar_init(smem_u32(epi_done), NEPI);
        mbar_init(smem_u32(tk_done), 1);
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    // (a suspending wait: the hardware parks the thread until the phase completes)
    auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        if (*s_abort) return false;
        if (mbar_wait_park(smem_u32(bar), parity, kParkLimit, kParkNs)) return true;
        atomicCAS(&g_qgemm_error, 0, kErrTimeout);
        *s_abort = 1;
        return false;
    };

    if (warp == WARP_TMA) {
        // ------------------------------ loads -------------------------------------
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tx)) : "memory");
            asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tw)) : "memory");
            uint32_t li = 0;
            bool ok = true;
            for (Seg wk = seg_first(); seg_valid(wk) && ok; wk = seg_next(wk)) {
                const Tile tl = tile_of(wk.t);
                for (int kb = wk.kb0; kb < wk.kb1; ++kb, ++li) {
                    const int s = li % LS;
                    if (li >= LS && !wait(load_empty + s, (li / LS - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = smem_u32(smem + s * LSB);
                    const uint32_t bar = smem_u32(load_full + s);
                    mbar_arrive_expect_tx(bar, LSB);
                    tma_load_2d(dst, &tx, bar, kb * BK, tl.row0);
                    tma_load_2d(dst + X_BYTES, &tw, bar, kb * WPR, tl.e * N + tl.nb * BW);
                }
            }
            if (!ok) {
                // let the copies already issued land before the CTA can exit
                const uint32_t n = li < static_cast<uint32_t>(LS) ? li : LS;
                for (uint32_t j = li - n; j < li; ++j)
                    mbar_wait_bounded(smem_u32(load_full + j % LS), (j / LS) & 1, kSpinLimit);
            }
        }
    } else if (warp == WARP_MMA) {
        // ------------------------------ MMA issue ---------------------------------
        if (lane == 0) {
            uint32_t li = 0, ai_k = 0, ai = 0;
            bool ok = true;
            for (Seg wk = seg_first(); seg_valid(wk) && ok; wk = seg_next(wk), ++ai) {
                const uint32_t a = ai & 1;
                if (ai >= 2 && !wait(acc_empty + a, (ai / 2 - 1) & 1)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
                for (int kb = wk.kb0; kb < wk.kb1; ++kb, ++li, ++ai_k) {
                    const int s = li % LS, as = ai_k % ASTAGES;
                    // (the single MMA thread polls without parking: it wakes fastest)
                    if (!mbar_wait_bounded(smem_u32(load_full + s), (li / LS) & 1, kSpinLimit) ||
                        !mbar_wait_bounded(smem_u32(a_full + as), (ai_k / ASTAGES) & 1, kSpinLimit)) {
                        atomicCAS(&g_qgemm_error, 0, kErrTimeout);
                        *s_abort = 1;
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
                    const uint64_t bdesc = sw128_kmajor_desc(smem_u32(smem + s * LSB));
                    const uint32_t acol = tmem + kACol0 + as * kACols;
#pragma unroll
                    for (int j = 0; j < BK / 16; ++j)  // 16 elements: 8 A columns, 32 B of B
                        umma_f16_ts(tmem + a * BT, acol + 8 * j, bdesc + 2 * j, IDESC,
                                    (kb > wk.kb0 || j > 0) ? 1u : 0u);
                    umma_commit(smem_u32(load_empty + s));
                    umma_commit(smem_u32(a_empty + as));
                }
                if (ok) umma_commit(smem_u32(acc_full + a));
            }
            // every MMA issued so far has finished before tensor memory is freed
            umma_commit(smem_u32(mma_done));
            mbar_wait_bounded(smem_u32(mma_done), 0, kSpinLimit);
        }
    } else if (warp >= WARP_DEQ0) {
        // ------------------------------ dequantize ---------------------------------
        const int q = warp & 3;                       // tensor-memory lane quarter
        const int r = q * 32 + lane;                  // weight row within the tile
        const int ph = (warp - WARP_DEQ0) / 4;        // this warp's K blocks: index % DQ == ph
        constexpr int TCOLS = BK / 2;                 // tensor-memory columns per thread
        constexpr int NGK = BK >= GS ? BK / GS : 1;   // quantization groups per K block
        const int G = K / GS;
        const T* sg = static_cast<const T*>(p.s);
        const T* bg = static_cast<const T*>(p.b);
        const uint32_t mlo = opaque(Pair<T>::kMagicLo), mhi = opaque(Pair<T>::kMagicHi);
        const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16) + kACol0;
        // Scales and biases by 16-byte chunks of 8 groups (rows 16-byte aligned):
        // `cur` is the chunk in use, `nxt` the next one this thread will need along its
        // (tile, chunk) sequence, loaded a whole chunk (4-16 K blocks) early.
        const bool vec = (G % 8) == 0;
        const int nch = G / 8;
        auto load_chunk = [&](int tt, int cc, uint4& sv, uint4& bv) {
            sv = make_uint4(0u, 0u, 0u, 0u);
            bv = sv;
            if (tt >= tiles) return;
            const Tile tl = tile_of(tt);
            const int n = tl.nb * BW + r;
            if (n < N) {
                const long long off = (static_cast<long long>(tl.e) * N + n) * G + cc * 8;
                sv = ldg_nc_v4(sg + off);
                bv = ldg_nc_v4(bg + off);
            }
        };
        uint4 sc = make_uint4(0u, 0u, 0u, 0u), bc = sc, sn = sc, bn = sc;
        // the chunk sequence follows the segments: (tile, chunk) in order, the first
        // chunk being the one of the first segment's first K block
        const Seg wk0 = seg_first();
        int cur_t = wk0.t, cur_c = 0, tn = wk0.t, cn = (wk0.kb0 * BK / GS) >> 3;
        auto advance = [&]() {  // nxt becomes cur; fetch the chunk after it
            sc = sn;
            bc = bn;
            cur_t = tn;
            cur_c = cn;
            if (++cn == nch) {
                cn = 0;
                tn += SK ? 1 : static_cast<int>(P);
            }
            load_chunk(tn, cn, sn, bn);
        };
        if (vec) {
            load_chunk(tn, cn, sn, bn);
            advance();
        }
        auto pick = [](const uint4& v, int g) -> uint32_t {  // halfword g % 8, splatted
            const int w4 = (g >> 1) & 3;
            const uint32_t w = (w4 & 2) ? ((w4 & 1) ? v.w : v.z) : ((w4 & 1) ? v.y : v.x);
            const uint32_t h = (g & 1) ? (w >> 16) : (w & 0xffffu);
            return h | (h << 16);
        };
        uint32_t lb = 0;  // K blocks of this CTA's earlier segments
        bool ok = true;
        for (Seg wk = seg_first(); seg_valid(wk) && ok; lb += wk.kb1 - wk.kb0, wk = seg_next(wk)) {
            const int t = wk.t;
            const Tile tl = tile_of(t);
            const int n = tl.nb * BW + r;  // row within expert tl.e (n >= N: none)
            // K blocks are dealt by their index along the CTA's whole sequence, so a
            // stage's previous K block (LS back, LS a multiple of DQ) was this warp's too
            for (int kb = wk.kb0 + static_cast<int>((ph + DQ - lb % DQ) % DQ); kb < wk.kb1;
                 kb += DQ) {
                const uint32_t li = lb + (kb - wk.kb0);  // K block index along the CTA's work
                const int s = li % LS, as = li % ASTAGES;
                uint32_t s2[NGK], b2[NGK];
#pragma unroll
                for (int j = 0; j < NGK; ++j) {
                    const int g = (kb * BK) / GS + j;  // this row's groups in the K block
                    if (vec) {
                        // a warp meets every chunk of 8 groups (a chunk spans at least 4
                        // K blocks, DQ <= 4) except perhaps the tail of a stream-K share's
                        // first chunk: at most one extra step, bounded all the same
#pragma unroll 1
                        for (int k = 0; k < 4 && ((g >> 3) != cur_c || t != cur_t); ++k)
                            advance();
                        s2[j] = pick(sc, g);
                        b2[j] = pick(bc, g);
                    } else {
                        T sv = T(0.0f), bv = T(0.0f);
                        if (n < N) {
                            sv = sg[(static_cast<long long>(tl.e) * N + n) * G + g];
                            bv = bg[(static_cast<long long>(tl.e) * N + n) * G + g];
                        }
                        s2[j] = splat(sv);
                        b2[j] = splat(bv);
                    }
                }
                if (!wait(load_full + s, (li / LS) & 1) ||
                    (li >= ASTAGES && !wait(a_empty + as, (li / ASTAGES - 1) & 1))) {
                    ok = false;
                    break;
                }
                // row r's codes of the K block (TMA 32-/64-byte swizzle: 16-byte chunk c
                // of row r sits at chunk c ^ (r >> 2 & 1) / c ^ (r >> 1 & 3))
                uint32_t raw[WPR];
                const uint8_t* rrow = smem + s * LSB + X_BYTES + r * (WPR * 4);
#pragma unroll
                for (int c = 0; c < WPR / 4; ++c) {
                    const int pc = (BITS == 4) ? (c ^ ((r >> 2) & 1)) : (c ^ ((r >> 1) & 3));
                    const uint4 v = *reinterpret_cast<const uint4*>(rrow + pc * 16);
                    raw[4 * c] = v.x; raw[4 * c + 1] = v.y; raw[4 * c + 2] = v.z; raw[4 * c + 3] = v.w;
                }
                uint32_t outv[TCOLS];
#pragma unroll
                for (int c = 0; c < BK / 8; ++c) {
                    const int j = NGK > 1 ? (c * 8) / GS : 0;
                    const uint4 v = dequant_chunk<T, BITS>(&raw[c * (BITS == 4 ? 1 : 2)], s2[j],
                                                          b2[j], mlo, mhi);
                    outv[4 * c] = v.x; outv[4 * c + 1] = v.y;
                    outv[4 * c + 2] = v.z; outv[4 * c + 3] = v.w;
                }
                tmem_st32(tq + as * kACols, outv);
                asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
                asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(smem_u32(a_full + as));
                    mbar_arrive(smem_u32(load_empty + s));
                }
            }
        }
    } else {
        // ------------------------------ epilogue -----------------------------------
        const int q = warp & 3;  // tensor-memory lanes this warp may read
        T* og = static_cast<T*>(p.out);
        const T* biasg = static_cast<const T*>(p.bias);
        const int row = q * 32 + lane;  // this thread's weight row in the tile
        uint32_t ai = 0, np = 0;  // np: partial tiles handled so far (handshake parity)
        for (Seg wk = seg_first(); seg_valid(wk); wk = seg_next(wk), ++ai) {
            const uint32_t a = ai & 1;
            if (!wait(acc_full + a, (ai / 2) & 1)) break;
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const Tile tl = tile_of(wk.t);
            const int n = tl.nb * BW + row;  // this thread's output column
            const bool col_ok = n < N;
            const float bsum = (biasg && col_ok) ? Elem<T>::to_f(biasg[n]) : 0.f;
            const uint32_t tacc = tmem + (static_cast<uint32_t>(q * 32) << 16) + a * BT;
            if (wk.kb0 == 0 && wk.kb1 == KB) {
                // the whole tile: straight to the output
#pragma unroll 1
                for (int i = 0; i < BT / 32; ++i) {
                    uint32_t v[32];
                    tmem_ld32(tacc + i * 32, v);
                    const int tok0 = tl.row0 + i * 32;
                    if constexpr (EPI == 1) {
                        // gate lanes (row r < 8 of their 16-row tile) pair with lane ^ 8
                        const bool gate_lane = (lane & 8) == 0;
                        const int nh = (tl.nb * BW + q * 32 + (lane & 16)) / 2 + (lane & 7);
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float mine = __uint_as_float(v[j]);
                            const float other = __shfl_xor_sync(0xffffffffu, mine, 8);
                            const int tok = tok0 + j;
                            if (gate_lane && col_ok && tok < tl.row_end)
                                og[static_cast<long long>(tok) * (N / 2) + nh] =
                                    swiglu_out<T>(mine, other);
                        }
                    } else if (col_ok) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const int tok = tok0 + j;
                            if (tok < tl.row_end) {
                                T y = Elem<T>::from_f(__uint_as_float(v[j]));
                                if (biasg) y = Elem<T>::from_f(Elem<T>::to_f(y) + bsum);
                                og[static_cast<long long>(tok) * N + n] = y;
                            }
                        }
                    }
                }
                asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(acc_empty + a));
                continue;
            }
            // Stream-K, part of a tile: the fp32 partial goes to this CTA's slot (0: its
            // first segment, 1: its last); the last of the tile's contributors (atomic
            // ticket) adds all partials in CTA order and writes the tile.
            // (token-major: a warp writes, and later reads, 32 consecutive rows of a token)
            float* mine = p.partial +
                          static_cast<size_t>(blockIdx.x * 2 + (wk.u == u_lo ? 0 : 1)) * BT * BW + row;
#pragma unroll 1
            for (int i = 0; i < BT / 32; ++i) {
                uint32_t v[32];
                tmem_ld32(tacc + i * 32, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) mine[(i * 32 + j) * BW] = __uint_as_float(v[j]);
            }
            asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(smem_u32(acc_empty + a));  // the accumulator is free
                mbar_arrive(smem_u32(epi_done));       // this warp's partials are stored
            }
            const unsigned ub = static_cast<unsigned>(wk.t) * static_cast<unsigned>(KB);
            const int first = owner(ub), nc = owner(ub + KB - 1) - first + 1;
            // Once all epilogue warps have stored (epi_done: release/acquire at CTA scope),
            // one thread takes the acq_rel ticket: its release publishes them GPU-wide
            // (cumulatively), its acquire, passed on through tk_done, orders the other
            // contributors' partials before the reads below. Bounded waits and no named
            // barrier: a warp that stops early cannot leave the others blocked.
            const uint32_t par = np & 1u;
            ++np;
            if (row == 0) {
                int last = 0;
                if (!mbar_wait_park(smem_u32(epi_done), par, kParkLimit, kParkNs)) {
                    atomicCAS(&g_qgemm_error, 0, kErrTimeout);
                    *s_abort = 1;
                } else if (!*s_abort) {
                    last = atom_add_acq_rel_gpu(p.counter + wk.t, 1u) ==
                           static_cast<unsigned>(nc - 1);
                }
                *s_last = last;
                mbar_arrive(smem_u32(tk_done));
            }
            if (!mbar_wait_park(smem_u32(tk_done), par, kParkLimit, kParkNs)) {
                atomicCAS(&g_qgemm_error, 0, kErrTimeout);
                *s_abort = 1;
                break;
            }
            if (!*s_last) continue;
            if (row == 0) p.counter[wk.t] = 0u;  // re-armed (every contributor has ticked)
            if (!col_ok) continue;
#pragma unroll 1
            for (int i = 0; i < BT / 32; ++i) {
                float f[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) f[j] = 0.f;
#pragma unroll 1
                for (int c = 0; c < nc; ++c) {
                    const unsigned b = static_cast<unsigned>(first + c);
                    // slot 0 if this tile is where CTA b's share starts, else slot 1
                    const int slot = static_cast<int>(U * b / P / static_cast<unsigned>(KB)) == wk.t ? 0 : 1;
                    const float* src = p.partial +
                                       static_cast<size_t>(b * 2 + slot) * BT * BW + i * 32 * BW + row;
                    float w[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) w[j] = __ldcg(src + j * BW);
#pragma unroll
                    for (int j = 0; j < 32; ++j) f[j] += w[j];
                }
                const int tok0 = tl.row0 + i * 32;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int tok = tok0 + j;
                    if (tok < tl.row_end) {
                        T y = Elem<T>::from_f(f[j]);
                        if (biasg) y = Elem<T>::from_f(Elem<T>::to_f(y) + bsum);
                        og[static_cast<long long>(tok) * N + n] = y;
                    }
                }
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == WARP_MMA) {
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                     "r"(kTmemCols));
    }
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 qg_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

bool qg_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize,
            unsigned long long cols, unsigned long long rows, unsigned box_cols, unsigned box_rows,
            CUtensorMapSwizzle swz) {
    auto fn = qg_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * static_cast<cuuint64_t>(esize)};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

// SK: the stream-K instance (a separate kernel, so the whole-tile one keeps its
// registers and schedule).
template <typename T, int BITS, int GS, int BT, bool SK, int EPI = 0>
static cudaError_t qgemm_launch_bt(const QgemmParams& p, cudaStream_t st) {
    auto kern = qgemm_kernel<T, BITS, GS, BT, SK, EPI>;
    constexpr int smem = qg::smem_bytes<BITS, BT>();
    static_assert(smem <= 232448, "at most 227 KB of dynamic shared memory per CTA");
    static PerDevice configured;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    e = ensure_smem_attr(kern, configured, dev, smem);
    if (e != cudaSuccess) return e;
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    CUtensorMap tx, tw;
    const unsigned long long kw = static_cast<unsigned long long>(p.K) * BITS / 32;
    if (!qg_map(&tx, p.x, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, p.K, p.M, qg::BK, BT,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
        !qg_map(&tw, p.w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, kw,
                static_cast<unsigned long long>(p.N) * (p.E > 0 ? p.E : 1), qg::BK * BITS / 32, qg::BW,
                BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B))
        return cudaErrorInvalidValue;
    // grouped: the tile count lives on the device; ceil(rows_e / BT) summed over experts
    // is at most ceil(M / BT) + E
    const long long mblocks = (p.M + BT - 1) / BT + (p.E > 0 ? p.E : 0);
    const long long tiles = mblocks * ((p.N + qg::BW - 1) / qg::BW);
    const int grid = SK ? (p.grid > 0 && p.grid < sms ? p.grid : sms)
                        : static_cast<int>(tiles < sms ? tiles : sms);
    kern<<<grid, qg::THREADS, smem, st>>>(tx, tw, p);
    return cudaGetLastError();
}

// Experts' row segments are short (a few hundred rows): 128-token tiles waste less; a
// dense shape with few tiles (see qgemm_plan) also gets more of them at 128 tokens.
template <typename T, int BITS, int GS>
static cudaError_t qgemm_launch_t(const QgemmParams& p, cudaStream_t st) {
    if (p.epi == 1) {  // whole tiles only
        if (p.sk) return cudaErrorInvalidValue;
        if (p.E > 0) return qgemm_launch_bt<T, BITS, GS, qg::BT_GROUPED, false, 1>(p, st);
        return qgemm_launch_bt<T, BITS, GS, qg::BT_DENSE, false, 1>(p, st);
    }
    if (p.E > 0 || p.narrow) return qgemm_launch_bt<T, BITS, GS, qg::BT_GROUPED, false>(p, st);
    if (p.sk) return qgemm_launch_bt<T, BITS, GS, qg::BT_DENSE, true>(p, st);
    return qgemm_launch_bt<T, BITS, GS, qg::BT_DENSE, false>(p, st);
}

// tile_start[e + 1] = tile_start[e] + ceil(rows_e / BT_GROUPED) * NB, one block, E in chunks
__global__ void group_tiles_kernel(const int32_t* __restrict__ seg, int E, int rpe, int NB,
                                   int32_t* __restrict__ tile_start) {
    __shared__ int scan[1024];
    __shared__ int carry;
    if (threadIdx.x == 0) {
        carry = 0;
        tile_start[0] = 0;
    }
    __syncthreads();
    for (int base = 0; base < E; base += 1024) {
        const int e = base + threadIdx.x;
        int c = 0;
        if (e < E) {
            const int rows = max(0, (seg[e + 1] - seg[e]) * rpe);
            c = (rows + qg::BT_GROUPED - 1) / qg::BT_GROUPED * NB;
        }
        scan[threadIdx.x] = c;
        __syncthreads();
        for (int off = 1; off < 1024; off <<= 1) {  // inclusive scan
            const int v = threadIdx.x >= off ? scan[threadIdx.x - off] : 0;
            __syncthreads();
            scan[threadIdx.x] += v;
            __syncthreads();
        }
        if (e < E) tile_start[e + 1] = carry + scan[threadIdx.x];
        __syncthreads();
        if (threadIdx.x == 0) carry += scan[1023];
        __syncthreads();
    }
}

cudaError_t launch_group_tiles(const int32_t* seg, int E, int rpe, int N, int32_t* tile_start,
                               cudaStream_t st) {
    group_tiles_kernel<<<1, 1024, 0, st>>>(seg, E, rpe, (N + qg::BW - 1) / qg::BW, tile_start);
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

// Stream-K is used when whole tiles would fill less than this share of the CTA slots
// of their waves (q/o and down projections at a few thousand tokens), as long as each
// CTA's share is at least a third of a tile: more contributors per tile make the last
// one's pass over their partials cost more than the idle SMs (k/v at 512 tokens: 12
// tiles split 12 ways ran at 32 TFLOP/s).
constexpr double kStreamKBelow = 0.85;
constexpr long long kStreamKShare = 3;

bool qgemm_plan(int M, int N, int K, int num_sms, QgemmPlan* plan) {
    QgemmPlan pl{};
    const long long tiles = static_cast<long long>((M + qg::BT_DENSE - 1) / qg::BT_DENSE) *
                            ((N + qg::BW - 1) / qg::BW);
    const long long KB = K / qg::BK;
    const long long waves = (tiles + num_sms - 1) / num_sms;
    const double fill = static_cast<double>(tiles) / static_cast<double>(waves * num_sms);
    const long long units = tiles * KB;
    const long long tiles128 = static_cast<long long>((M + qg::BT_GROUPED - 1) /
                                                      qg::BT_GROUPED) *
                               ((N + qg::BW - 1) / qg::BW);
    // Stream-K CTAs: each takes at least KB / kStreamKShare K blocks, so at most about
    // that many CTAs add partials to one tile (the last one reads them all, which is
    // what bounds a short-K stream-K); one per SM when the K blocks allow, else fewer,
    // as long as they outnumber the whole 128-token tiles (k/v at 512-2048 tokens:
    // 36-132 CTAs instead of 16-64 tiles, 32.1 against 34.8 µs at 512 tokens).
    const long long sk_grid =
        num_sms > 0 ? std::min<long long>(num_sms, kStreamKShare * units / KB) : 0;
    if (num_sms > 0 && fill < kStreamKBelow && (sk_grid == num_sms || sk_grid > tiles128) &&
        units >= sk_grid && sk_grid > 0 &&
        tiles * 4 <= static_cast<long long>(kArgmaxOffset) &&
        units * (num_sms + 1) < (1LL << 31)) {
        pl.stream_k = true;
        pl.grid = static_cast<int>(sk_grid);
        pl.ws_bytes = kTicketBytes + static_cast<size_t>(num_sms) * 2 * qg::BW *
                                         qg::BT_DENSE * sizeof(float);
    } else if (fill < kStreamKBelow) {
        // too few tiles and too short a K for stream-K: 128-token tiles give the SMs
        // more of them (a tile's pipeline, not its width, sets its time)
        pl.narrow = tiles128 > tiles && tiles < num_sms;
    }
    *plan = pl;
    return true;
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
