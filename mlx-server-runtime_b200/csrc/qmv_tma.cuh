// Decode-shaped group-wise affine quantized matmul fed by TMA (sm_100a):
//
//   out[t, n] = sum_k x[t, k] * (scale[n, k/g] * q[n, k] + bias[n, k/g]),  t < M <= 8
//
// MLX's quantized_matmul with transpose=True as QuantizedLinear calls it at
// decode (qwen2.py:58-61,123-134 of the reference).
//
// Work: the weight matrix is cut into units of BR rows x 8 quantization groups
// (one pipeline stage), BR = 64, or 16 for matrices with few, short rows. Units
// are numbered row-block-major and each CTA takes a contiguous, equal share
// (stream-K): every SM streams the same number of bytes whatever N and K are. A
// row block whose units span several CTAs is finished by the last of them (atomic
// ticket, no waiting), which adds the fp32 partials in CTA order, so results are
// deterministic. When every row block fits on the SMs, each CTA takes one whole
// row block instead and no ticket is needed.
//
// Per CTA: one producer warp and 8 consumer warps (plus, in kernels built with
// HEADS, a ticket warp: a share that starts inside a row block stores that head
// row block's partials and goes on at once, while the ticket warp takes its
// ticket; whether the CTA came last to it is read when the share is done).
//   * Producer (one thread): for every unit, 2-D TMA loads of the packed
//     weights [BR rows x 128 B] per box (128-byte swizzle) plus one box each of
//     scales and biases [BR rows x 8 groups], into a ring of `stages` slots with
//     full/empty mbarriers. The ring holds most of the CTA's share, so nearly
//     all of it is requested from HBM at kernel start.
//   * Consumers: warp (rt, kq) owns row tile rt (16 rows) and GPW groups, GPW*kq..,
//     of every stage (64-row units: 4 row tiles x 2 warps of 4 groups; 16-row
//     units: 1 row tile x 8 warps of 1 group). ldmatrix reads the swizzled tiles
//     without bank conflicts and hands lane (r, c) words c, c+4, ... of the group
//     for rows r and r+8. Codes become exact f16 MMA operands with one LOP3 per
//     pair (see Elem<__half>::extract); one m16n8k16 MMA covers 16 codes x 8
//     token slots into a fresh fp32 accumulator per group.
//   * Activations: x[M, K] is staged once as f16 MMA B fragments. Each (group,
//     token) slice is multiplied by a power of two 2^e that brings its largest
//     magnitude into [2^14, 2^15), which makes the bf16 (or f16) values exact in
//     f16, so bf16 activations use the cheaper f16 extraction too. A record
//     {sum x, sum offset * x 2^e, 2^-e} per slice turns the MMA result D into
//       acc += (scale * 2^-e) * (D - sum offset * x 2^e) + bias * sum x.
//     The token count is a compile-time slot count TM in {1, 2, 4, 8, 16} (M
//     rounded up; absent tokens are zero; 16 slots are two MMA n-tiles of 8), so
//     every shared-memory address in the main loop is a per-lane base plus a constant.
// Every wait is bounded: a timeout records an error in *p.err, sets a CTA-wide
// abort flag that turns the remaining waits and all global writes off, and
// lets every warp run to the end (so the named barriers still meet).
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"

namespace mlxq {

namespace qt {
constexpr int SG = 8;                    // quantization groups per unit (stage)
constexpr int CWARPS = 8;                // consumer warps
constexpr int CTHREADS = CWARPS * 32;
// + producer warp (+ ticket warp in the kernels that hand off head tickets)
__host__ __device__ constexpr int threads(bool heads) { return CTHREADS + (heads ? 64 : 32); }
// Split of the 8 consumer warps over a unit of BR weight rows (64 or 16): RT
// row tiles of 16 rows times KSW warps along K, each warp taking GPW of the
// stage's 8 groups. Shorter units put more CTAs on a matrix with few rows and
// shorten each CTA's chain of stages when its row blocks are not split.
template <int BR>
struct Rows {
    static_assert(BR == 16 || BR == 64, "unit rows");
    static constexpr int RT = BR / 16;
    static constexpr int KSW = CWARPS / RT;
    static constexpr int GPW = SG / KSW;
};
constexpr int MAXM = 16;                 // tokens per launch
constexpr int MAX_STAGES = 16;
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr int kErrTimeout = 2;
// The ticket warp parks (suspend-time hint) while the consumers finish a head row block.
constexpr uint32_t kTicketParkNs = 1000;
constexpr uint32_t kTicketParkLimit = 1u << 20;

// Token slots a kernel instance is compiled for; M is rounded up to one of them.
// An MMA covers 8 token slots: 16 slots take two MMA n-tiles per weight fragment.
__host__ __device__ constexpr int token_slots(int M) {
    return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16;
}
__host__ __device__ constexpr int n_tiles(int TM) { return TM > 8 ? TM / 8 : 1; }

// Bytes one stage's TMA copies deliver (packed codes, scales, biases) and the
// stage's stride in the ring (rounded up to the 1024-byte period of the 128-byte
// swizzle, so every stage's boxes start on it).
__host__ __device__ constexpr int stage_tx(int bits, int gs, int br) {
    return (SG * gs * bits / 32 / 32) * br * 128 + 2 * br * SG * 2;
}
__host__ __device__ constexpr int stage_stride(int bits, int gs, int br) {
    return (stage_tx(bits, gs, br) + 1023) / 1024 * 1024;
}

template <int BITS, int GS, int BR>
struct Geo {
    static constexpr int WPG = GS * BITS / 32;     // packed words per group per row
    static constexpr int CPG = WPG / 4;            // 16-byte chunks per group per row
    static constexpr int BOXES = SG * WPG / 32;    // 128-byte TMA boxes per stage
    static constexpr int W_BYTES = BOXES * BR * 128;
    static constexpr int SB_BYTES = BR * SG * 2;   // scales (or biases) of one stage
    static constexpr int STAGE_TX = W_BYTES + 2 * SB_BYTES;
    static constexpr int STAGE = stage_stride(BITS, GS, BR);
    static constexpr int FR = (BITS == 4) ? 4 * CPG : 2 * CPG;  // B-fragment words per lane
    static constexpr int XG = GS * 2;              // fragment bytes per (group, token slot)
    static_assert(CPG >= 1 && BOXES >= 1 && STAGE_TX == stage_tx(BITS, GS, BR),
                  "unsupported geometry");
};

// Shared-memory layout (from a 1024-byte aligned base), in bytes; rt = row tiles
// per unit (the cross-warp reduction holds (KSW - 1) * RT = 8 - rt warp tiles).
struct Layout {
    int ring, xf, rec, red, bars, flags, best, total;
};
__host__ __device__ inline Layout layout(int stage_bytes, int stages, int G, int TM, int xg,
                                         int rt) {
    Layout L;
    L.ring = 0;
    L.xf = stages * stage_bytes;               // [G][FR/4][TM][4 lanes] x 16 B
    L.rec = L.xf + G * TM * xg;                // [G][TM] float4 records
    L.red = L.rec + G * TM * 16;               // cross-warp reduction
    L.bars = (L.red + (CWARPS - rt) * n_tiles(TM) * 4 * 32 * 4 + 7) & ~7;
    // full[stages], empty[stages], head_done, ticket_done
    L.flags = (L.bars + (2 * stages + 2) * 8 + 15) & ~15;  // abort, last, head_last
    L.best = L.flags + 16;                                  // argmax: best key per token
    L.total = L.best + MAXM * 8;
    return L;
}

// Owner CTA of unit u when U units are split in P contiguous shares
// [floor(U*i/P), floor(U*(i+1)/P)).
__host__ __device__ inline int owner(long long u, long long U, int P) {
    return static_cast<int>(((u + 1) * P - 1) / U);
}

// 2^e as a float for integer e in [-126, 127] (exact).
__device__ __forceinline__ float pow2i(int e) {
    return __uint_as_float(static_cast<uint32_t>(127 + e) << 23);
}

// The e that brings a finite m > 0 into [2^14, 2^15) (clamped so 2^e and 2^-e
// stay normal floats); 0 for zero, infinite or NaN m.
__device__ __forceinline__ int slice_exponent(float m) {
    const uint32_t bits = __float_as_uint(m);
    const int ef = static_cast<int>((bits >> 23) & 0xffu);
    if (!(m > 0.f) || ef == 0xff) return 0;
    const int e = 14 - (ef - 127);  // subnormal m (ef == 0) gives the clamp below
    return e > 126 ? 126 : (e < -126 ? -126 : e);
}

// Slow path of a full-barrier wait (the first poll usually succeeds).
static __device__ __noinline__ bool wait_slow(uint32_t bar, uint32_t parity) {
    return mbar_wait_bounded(bar, parity, kSpinLimit);
}
}  // namespace qt

// 2-D tiled tensor map over a row-major [rows, cols] array of `esize`-byte elements
// with box [box_rows, box_cols] (qmv_tma.cu); false when the driver's encoder is
// missing or rejects the map.
bool qt_make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize,
                 unsigned long long cols, unsigned long long rows, unsigned box_cols,
                 unsigned box_rows, CUtensorMapSwizzle swz);
bool qt_maps_available();
// Device address of the decode kernels' error word (qmv_tma.cu).
int* qmv_tma_error_flag();

struct QtParams {
    const void* x;
    const void* bias;
    void* out;
    int M, N, K, G;
    int GL;         // most K groups one CTA's units use (activation fragments staged)
    int S;          // stages (units) per row block = G / 8
    int RB;         // row blocks
    long long U;    // units
    int stages;     // ring depth
    int maxc;       // most CTAs contributing to one row block
    unsigned* counter;  // [RB], zero at entry and exit
    float* partial;     // [RB][maxc][M][64]
    int* err;           // device error flag
    unsigned* am_done;            // argmax epilogue: CTAs done (zero at entry and exit)
    unsigned long long* am_keys;  // argmax epilogue: best key per token (likewise)
};

// Epilogues (EPI):
// 0  the outputs out[t, n].
// 1  SwiGLU: w holds a gate/up pair per 16-row tile (rows 0-7 gate rows 8j.., rows 8-15
//    the matching up rows), which are exactly the rows r and r + 8 one MMA lane holds;
//    the kernel writes silu(gate) * up, out[t, 8j + r], N / 2 columns, each projection
//    rounded to T first as two separate matmuls would be.
// 2  greedy argmax: no outputs; each output value (rounded to T, plus bias) becomes a
//    key (order-preserving bits of the value, then the complement of n, so ties go to
//    the first n); the CTA keeps its best key per token in shared memory, then one
//    global atomicMax per token; the last CTA to finish (a done counter) writes the
//    winning n per token to int32 out[t] and re-arms the keys and the counter.

__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(n));
}

// x -> f16 MMA B fragments and per-slice records in shared memory, for nj group
// positions j (a multiple of 8) and TM token slots. xrow(t) is token slot t's row of x
// (nullptr: an absent slot, staged as zeros), grp(j) the K group staged at position j
// (-1: padding past K, zeros). Item i = ((j * TM + t) * 4 + c): lane c of token slot t
// holds words c, c+4, ... of the group (the words ldmatrix gives that lane). The item
// count is a multiple of 32, so every warp runs whole iterations and the 4 lanes of an
// item share a warp. Fragments and records are stored by position j.
template <typename T, int BITS, int GS, int TM, typename XRow, typename Grp>
__device__ __forceinline__ void qt_stage_activations(uint8_t* xf, float4* rec, int nj, XRow xrow,
                                                     Grp grp, int ctid) {
    using namespace qt;
    using ET = Elem<T>;
    using EH = Elem<__half>;
    using OFF = typename EH::template Off<BITS>;
    using GEO = Geo<BITS, GS, 16>;
    constexpr int CPG = GEO::CPG, FR = GEO::FR, XG = GEO::XG;
    constexpr int XW = BITS == 4 ? 8 : 4;  // activations per packed word
    constexpr int PB = (CPG * XW / 2 <= 8) ? 4 : 2;  // items with loads in flight together
    const int total = nj * TM * 4;
    for (int i0 = ctid; i0 < total; i0 += PB * CTHREADS) {
      uint32_t raw[PB][CPG][XW / 2];
#pragma unroll
      for (int b = 0; b < PB; ++b) {
        const int i = i0 + b * CTHREADS;
        const int cc = i & 3, t = (i >> 2) % TM, j = (i >> 2) / TM;
        const T* row = i < total ? xrow(t) : nullptr;
        const int g = i < total ? grp(j) : -1;
#pragma unroll
        for (int w = 0; w < CPG; ++w) {
            const int off = g * GS + (4 * w + cc) * XW;
            if constexpr (BITS == 4) {
                uint4 q = make_uint4(0u, 0u, 0u, 0u);
                if (row && g >= 0) q = *reinterpret_cast<const uint4*>(row + off);
                raw[b][w][0] = q.x; raw[b][w][1] = q.y; raw[b][w][2] = q.z; raw[b][w][3] = q.w;
            } else {
                uint2 q = make_uint2(0u, 0u);
                if (row && g >= 0) q = *reinterpret_cast<const uint2*>(row + off);
                raw[b][w][0] = q.x; raw[b][w][1] = q.y;
            }
        }
      }
#pragma unroll
      for (int b = 0; b < PB; ++b) {
        const int i = i0 + b * CTHREADS;
        if (i >= total) break;  // warp-uniform: total and CTHREADS are multiples of 32
        const int cc = i & 3, t = (i >> 2) % TM, j = (i >> 2) / TM;
        float v[CPG][XW];
        float m = 0.f;
#pragma unroll
        for (int w = 0; w < CPG; ++w) {
#pragma unroll
            for (int k = 0; k < XW / 2; ++k) {
                v[w][2 * k] = ET::lo(raw[b][w][k]);
                v[w][2 * k + 1] = ET::hi(raw[b][w][k]);
                m = fmaxf(m, fmaxf(fabsf(v[w][2 * k]), fabsf(v[w][2 * k + 1])));
            }
        }
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        // fmaxf drops NaN, and an infinite maximum keeps e = 0: NaN and inf
        // activations reach D unchanged and propagate to the output.
        const int e = slice_exponent(m);
        const float sc = pow2i(e);
        uint32_t fr[FR];
        float s_all = 0.f, s_even = 0.f, s_odd = 0.f;
#pragma unroll
        for (int w = 0; w < CPG; ++w) {
            float y[XW];
#pragma unroll
            for (int k = 0; k < XW; ++k) {
                y[k] = v[w][k] * sc;
                s_all += v[w][k];
                if (k & 1) s_odd += y[k]; else s_even += y[k];
            }
            if constexpr (BITS == 4) {
                // operands pair nibbles (0,4) (1,5) (2,6) (3,7) of the word
                fr[4 * w + 0] = pack_half2(y[0], y[4]);
                fr[4 * w + 1] = pack_half2(y[1], y[5]);
                fr[4 * w + 2] = pack_half2(y[2], y[6]);
                fr[4 * w + 3] = pack_half2(y[3], y[7]);
            } else {
                // operands pair bytes (0,2) and (1,3) of the word
                fr[2 * w + 0] = pack_half2(y[0], y[2]);
                fr[2 * w + 1] = pack_half2(y[1], y[3]);
            }
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
            s_all += __shfl_xor_sync(0xffffffffu, s_all, o);
            s_even += __shfl_xor_sync(0xffffffffu, s_even, o);
            s_odd += __shfl_xor_sync(0xffffffffu, s_odd, o);
        }
        uint4* dst = reinterpret_cast<uint4*>(xf + static_cast<size_t>(j) * TM * XG);
#pragma unroll
        for (int f = 0; f < FR / 4; ++f)
            dst[(f * TM + t) * 4 + cc] =
                make_uint4(fr[4 * f], fr[4 * f + 1], fr[4 * f + 2], fr[4 * f + 3]);
        if (cc == 0) {
            // 4-bit: even code positions carry offset kOffE, odd ones kOffO (per
            // MMA slot); 8-bit: every activation meets both nibble operands.
            const float toff = (BITS == 4) ? OFF::kOffE * s_even + OFF::kOffO * s_odd
                                           : OFF::kOff * (s_even + s_odd);
            rec[j * TM + t] = make_float4(s_all, toff, pow2i(-e), 0.f);
        }
      }
    }
}

// One consumer warp's view of the ring: warp (rt, kq) owns row tile rt (16 rows) and
// groups GPW*kq.. of every stage. The constructor fixes the per-lane offsets; stage()
// folds one stage's groups into acc (token slots 8 nt + 2c, 8 nt + 2c + 1 of rows r and
// r + 8 of the row tile), reading the staged activations of the stage's first group at
// xs / rs (as returned by x_at / rec_at for the stage's position in the staged groups).
template <typename T, int BITS, int GS, int TM, int BR>
struct QtConsumer {
    using ET = Elem<T>;
    using EH = Elem<__half>;
    using GEO = qt::Geo<BITS, GS, BR>;
    static constexpr int WPG = GEO::WPG, CPG = GEO::CPG, FR = GEO::FR, XG = GEO::XG;
    static constexpr int W_BYTES = GEO::W_BYTES, SB_BYTES = GEO::SB_BYTES;
    static constexpr int RT = qt::Rows<BR>::RT, KSW = qt::Rows<BR>::KSW, GPW = qt::Rows<BR>::GPW;
    static constexpr bool ODD = TM > 1;
    static constexpr int NT = qt::n_tiles(TM);  // MMA n-tiles of 8 token slots
    static constexpr int TS = TM < 8 ? TM : 8;  // token slots of one n-tile
    static constexpr int NLD = CPG > 1 ? CPG / 2 : 1;
    static constexpr int SBW = GPW >= 2 ? GPW / 2 : 1;

    int rt, kq, r, c;
    uint32_t lmo[GPW][NLD];  // ldmatrix row addresses (relative to the stage) per group/chunk
    int so0, so1, sb_sh;     // packed (scale, scale) words of rows r, r+8; shift for GPW == 1
    uint32_t magic_a, magic_b;
    const uint8_t* xl;       // B fragments of token slot r (lanes past the last slot repeat one)
    const float4* rl;        // records of tokens 2c, 2c+1 (wrapped into the slots likewise)

    __device__ __forceinline__ QtConsumer(int warp, int lane, const uint8_t* xf, const float4* rec) {
        rt = warp % RT;
        kq = warp / RT;
        r = lane >> 2;
        c = lane & 3;
        const int row = 16 * rt + (lane & 15);
#pragma unroll
        for (int h = 0; h < GPW; ++h) {
            const int gi = GPW * kq + h;
            const int box = (gi * WPG) >> 5;
            const int cbase = ((gi * WPG) & 31) >> 2;
#pragma unroll
            for (int j = 0; j < NLD; ++j) {
                const int ch = cbase + 2 * j + (CPG > 1 ? (lane >> 4) : 0);
                lmo[h][j] = box * (BR * 128) + row * 128 + ((ch ^ (row & 7)) << 4);
            }
        }
        const int rr = 16 * rt + r;
        so0 = W_BYTES + rr * 16 + ((GPW * kq) & ~1) * 2;
        so1 = so0 + 8 * 16;
        sb_sh = GPW == 1 ? 16 * (kq & 1) : 0;
        magic_a = opaque(EH::template Magic<BITS>::kA);
        magic_b = opaque(EH::template Magic<BITS>::kB);
        // (n-tile nt's slots are 8 nt.. : its fragments sit 8 * 64 bytes further)
        const int tr = r & (TS - 1);
        xl = xf + (tr * 4 + c) * 16 + GPW * kq * TM * XG;
        rl = rec + ((2 * c) & (TS - 1)) + GPW * kq * TM;
    }
    // staged activations of the stage at position lst (8 groups each) of the staged groups
    __device__ __forceinline__ const uint8_t* x_at(int lst) const {
        return xl + static_cast<size_t>(lst) * qt::SG * TM * XG;
    }
    __device__ __forceinline__ const float4* rec_at(int lst) const {
        return rl + lst * qt::SG * TM;
    }

    __device__ __forceinline__ void stage(const uint8_t* stg, const uint8_t* xs, const float4* rs,
                                          float (&acc)[NT][4]) const {
        const uint32_t stg_s = smem_u32(stg);
        uint32_t s_r0[SBW], s_r1[SBW], b_r0[SBW], b_r1[SBW];
#pragma unroll
        for (int q = 0; q < SBW; ++q) {
            s_r0[q] = *reinterpret_cast<const uint32_t*>(stg + so0 + 4 * q);
            s_r1[q] = *reinterpret_cast<const uint32_t*>(stg + so1 + 4 * q);
            b_r0[q] = *reinterpret_cast<const uint32_t*>(stg + so0 + 4 * q + SB_BYTES);
            b_r1[q] = *reinterpret_cast<const uint32_t*>(stg + so1 + 4 * q + SB_BYTES);
        }
        if constexpr (GPW == 1) {
            s_r0[0] >>= sb_sh; s_r1[0] >>= sb_sh;
            b_r0[0] >>= sb_sh; b_r1[0] >>= sb_sh;
        }
#pragma unroll
        for (int h = 0; h < GPW; ++h) {
            uint32_t wa[CPG], wb[CPG];
            if constexpr (CPG == 1) {
                ldmatrix_x2(stg_s + lmo[h][0], wa[0], wb[0]);
            } else {
#pragma unroll
                for (int j = 0; j < NLD; ++j)
                    ldmatrix_x4(stg_s + lmo[h][j], wa[2 * j], wb[2 * j], wa[2 * j + 1],
                                wb[2 * j + 1]);
            }
            const int hq = h >> 1;
            const float s0 = (h & 1) ? ET::hi(s_r0[hq]) : ET::lo(s_r0[hq]);
            const float s1 = (h & 1) ? ET::hi(s_r1[hq]) : ET::lo(s_r1[hq]);
            const float b0 = (h & 1) ? ET::hi(b_r0[hq]) : ET::lo(b_r0[hq]);
            const float b1 = (h & 1) ? ET::hi(b_r1[hq]) : ET::lo(b_r1[hq]);
            uint32_t ta[CPG][4], tb[CPG][4];
#pragma unroll
            for (int w = 0; w < CPG; ++w) {
                EH::template extract<BITS>(wa[w], ta[w], magic_a, magic_b);
                EH::template extract<BITS>(wb[w], tb[w], magic_a, magic_b);
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
            uint32_t X[FR];
#pragma unroll
            for (int f = 0; f < FR / 4; ++f) {
                const uint4 v = *reinterpret_cast<const uint4*>(xs + h * TM * XG + f * TM * 64 +
                                                                nt * 8 * 64);
                X[4 * f + 0] = v.x; X[4 * f + 1] = v.y;
                X[4 * f + 2] = v.z; X[4 * f + 3] = v.w;
            }
            float d[4];
#pragma unroll
            for (int w = 0; w < CPG; ++w) {
                if constexpr (BITS == 4) {
                    if (w == 0)
                        mma16816z<__half>(d, ta[w][0], tb[w][0], ta[w][1], tb[w][1],
                                          X[4 * w + 0], X[4 * w + 1]);
                    else
                        mma16816<__half>(d, ta[w][0], tb[w][0], ta[w][1], tb[w][1],
                                         X[4 * w + 0], X[4 * w + 1]);
                    mma16816<__half>(d, ta[w][2], tb[w][2], ta[w][3], tb[w][3], X[4 * w + 2],
                                     X[4 * w + 3]);
                } else {
                    if (w == 0)
                        mma16816z<__half>(d, ta[w][0], tb[w][0], ta[w][1], tb[w][1],
                                          X[2 * w + 0], X[2 * w + 0]);
                    else
                        mma16816<__half>(d, ta[w][0], tb[w][0], ta[w][1], tb[w][1],
                                         X[2 * w + 0], X[2 * w + 0]);
                    mma16816<__half>(d, ta[w][2], tb[w][2], ta[w][3], tb[w][3], X[2 * w + 1],
                                     X[2 * w + 1]);
                }
            }
            // fold this group into tokens 8 nt + 2c, 8 nt + 2c + 1 of rows r, r+8
            const float4 q0 = rs[h * TM + 8 * nt];
            acc[nt][0] = fmaf(s0 * q0.z, d[0] - q0.y, fmaf(b0, q0.x, acc[nt][0]));
            acc[nt][2] = fmaf(s1 * q0.z, d[2] - q0.y, fmaf(b1, q0.x, acc[nt][2]));
            if constexpr (ODD) {
                const float4 q1 = rs[h * TM + 8 * nt + 1];
                acc[nt][1] = fmaf(s0 * q1.z, d[1] - q1.y, fmaf(b0, q1.x, acc[nt][1]));
                acc[nt][3] = fmaf(s1 * q1.z, d[3] - q1.y, fmaf(b1, q1.x, acc[nt][3]));
            }
            }
        }
    }

    // Adds the KSW group-interleaved warps of each row tile into warp kq == 0's acc
    // (fixed order). Starts and ends with a barrier of the consumer threads.
    __device__ __forceinline__ void combine(float* red, int lane, float (&acc)[NT][4]) const {
        named_bar_sync(1, qt::CTHREADS);
        if (kq > 0) {
            float* dst = red + ((kq - 1) * RT + rt) * NT * 4 * 32 + lane;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) dst[(nt * 4 + e) * 32] = acc[nt][e];
        }
        named_bar_sync(1, qt::CTHREADS);
        if (kq == 0) {
#pragma unroll
            for (int h = 1; h < KSW; ++h) {
                const float* src = red + ((h - 1) * RT + rt) * NT * 4 * 32 + lane;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[nt][e] += src[(nt * 4 + e) * 32];
            }
        }
    }
};

template <typename T, int BITS, int GS, int TM, int BR, bool HEADS, int EPI>
__global__ void __launch_bounds__(qt::threads(HEADS), 1)
    qmv_tma_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap ts,
                   const __grid_constant__ CUtensorMap tb, const QtParams p) {
    using namespace qt;
    using ET = Elem<T>;        // activation / output type
    using EH = Elem<__half>;   // MMA operand type
    using OFF = typename EH::template Off<BITS>;
    using GEO = Geo<BITS, GS, BR>;
    constexpr int WPG = GEO::WPG, CPG = GEO::CPG, FR = GEO::FR, XG = GEO::XG;
    constexpr int STAGE = GEO::STAGE, W_BYTES = GEO::W_BYTES, SB_BYTES = GEO::SB_BYTES;
    constexpr int RT = Rows<BR>::RT, KSW = Rows<BR>::KSW, GPW = Rows<BR>::GPW;
    constexpr bool ODD = TM > 1;
    constexpr int NT = n_tiles(TM);           // MMA n-tiles of 8 token slots
    constexpr int TS = TM < 8 ? TM : 8;       // token slots of one n-tile

    extern __shared__ __align__(16) uint8_t qt_smem_raw[];
    // 1024-byte aligned base (128-byte swizzled TMA boxes), derived from the shared
    // array by pointer arithmetic so every access stays a shared-memory access
    uint8_t* base = qt_smem_raw + ((1024u - (smem_u32(qt_smem_raw) & 1023u)) & 1023u);
    const int M = p.M, N = p.N, G = p.G, S = p.S, stages = p.stages;
    const Layout L = layout(STAGE, stages, p.GL, TM, XG, RT);
    uint8_t* ring = base + L.ring;
    uint8_t* xf = base + L.xf;
    float4* rec = reinterpret_cast<float4*>(base + L.rec);
    float* red = reinterpret_cast<float*>(base + L.red);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bars);
    uint64_t* empty = full + stages;
    uint64_t* head_done = empty + stages;
    uint64_t* ticket_done = head_done + 1;
    volatile int* s_abort = reinterpret_cast<volatile int*>(base + L.flags);
    volatile int* s_last = s_abort + 1;
    volatile int* s_head_last = s_abort + 2;
    unsigned long long* s_best = reinterpret_cast<unsigned long long*>(base + L.best);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long U = p.U;
    const int P = gridDim.x;
    const long long u_lo = U * blockIdx.x / P, u_hi = U * (blockIdx.x + 1) / P;
    // A share that starts inside a row block and runs past its end has a head row
    // block shared with the previous CTA(s). Its ticket is taken by the ticket warp
    // while the consumers go on with the rest of the share; whether this CTA came
    // last to it (and so reduces it) is looked at once the share is done.
    const int head_rb = static_cast<int>(u_lo / S);
    const bool has_head =
        HEADS && (u_lo % S) != 0 && u_hi > static_cast<long long>(head_rb + 1) * S;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(full + s), 1);
            mbar_init(smem_u32(empty + s), CWARPS);
        }
        if constexpr (HEADS) {
            mbar_init(smem_u32(head_done), CWARPS);
            mbar_init(smem_u32(ticket_done), 1);
        }
        *s_abort = 0;
        *s_last = 0;
        *s_head_last = 0;
        for (int t = 0; t < MAXM; ++t) s_best[t] = 0ull;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    // Launch overlap: the next kernel may start once every CTA got here. Weights,
    // scales and biases are read before griddepcontrol.wait; x, the workspace and
    // every global write come after it.
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

    if (warp == CWARPS) {
        // ------------------------------ producer ------------------------------------
        if (lane == 0) {
            tma_prefetch_map(&tw);
            tma_prefetch_map(&ts);
            tma_prefetch_map(&tb);
            uint32_t it = 0;
            int slot = 0;
            uint32_t phase = 0;  // parity of the empty-barrier phase to wait for
            int rb = static_cast<int>(u_lo / S), st = static_cast<int>(u_lo % S);
            for (long long u = u_lo; u < u_hi; ++u, ++it) {
                if (it >= static_cast<uint32_t>(stages)) {
                    if (*s_abort) break;
                    if (!mbar_wait_bounded(smem_u32(empty + slot), phase, kSpinLimit)) {
                        atomicCAS(p.err, 0, kErrTimeout);
                        *s_abort = 1;
                        break;
                    }
                }
                const uint32_t dst = smem_u32(ring + slot * STAGE);
                const uint32_t bar = smem_u32(full + slot);
                mbar_arrive_expect_tx(bar, GEO::STAGE_TX);
#pragma unroll
                for (int b = 0; b < GEO::BOXES; ++b)
                    tma_load_2d(dst + b * (BR * 128), &tw, bar, (st * SG * WPG) + b * 32, rb * BR);
                tma_load_2d(dst + W_BYTES, &ts, bar, st * SG, rb * BR);
                tma_load_2d(dst + W_BYTES + SB_BYTES, &tb, bar, st * SG, rb * BR);
                if (++slot == stages) {
                    slot = 0;
                    if (it >= static_cast<uint32_t>(stages)) phase ^= 1u;  // not after the first pass
                }
                if (++st == S) {
                    st = 0;
                    ++rb;
                }
            }
            if (*s_abort) {
                // let the copies already issued land before the CTA can exit
                const uint32_t n = it < static_cast<uint32_t>(stages) ? it : stages;
                for (uint32_t j = it - n; j < it; ++j)
                    mbar_wait_bounded(smem_u32(full + j % stages), (j / stages) & 1, kSpinLimit);
            }
        }
        return;
    }
    if (HEADS && warp == CWARPS + 1) {
        // ---------------------------- ticket warp ------------------------------------
        // Takes the head row block's ticket once every consumer warp has stored its
        // partials (head_done), so the consumers never wait for the atomic's round trip.
        if (lane == 0 && has_head) {
            asm volatile("griddepcontrol.wait;\n" ::: "memory");
            int last = 0;
            if (!mbar_wait_park(smem_u32(head_done), 0, kTicketParkLimit, kTicketParkNs)) {
                atomicCAS(p.err, 0, kErrTimeout);
                *s_abort = 1;
            } else if (!*s_abort) {
                const long long ub = static_cast<long long>(head_rb) * S;
                const int nc = owner(ub + S - 1, U, P) - owner(ub, U, P) + 1;
                // acq_rel: releases the partials the consumers stored (observed through
                // head_done) and acquires the other contributors' for the reduction
                last = atom_add_acq_rel_gpu(p.counter + head_rb, 1u) ==
                       static_cast<unsigned>(nc - 1);
            }
            *s_head_last = last;
            mbar_arrive(smem_u32(ticket_done));
        }
        return;
    }

    // -------------------------------- consumers ------------------------------------
    const int rt = warp % RT, kq = warp / RT;
    const int r = lane >> 2, c = lane & 3;
    const int ctid = threadIdx.x;  // 0 .. CTHREADS-1
    // The K groups this CTA's units use: stages u % S of its share, at most two
    // ranges [ga0, ga1) and [gb0, gb1) of groups (whole stages of 8 groups).
    int ga0 = 0, ga1 = G, gb0 = 0, gb1 = 0;
    if (u_hi - u_lo < S) {
        const int s0 = static_cast<int>(u_lo % S);
        const int s1 = s0 + static_cast<int>(u_hi - u_lo);
        ga0 = s0 * SG;
        ga1 = min(s1, S) * SG;
        gb1 = s1 > S ? (s1 - S) * SG : 0;
    }
    const int na = ga1 - ga0;
    // x may still be being written by the kernel before this one, so it is read only
    // after griddepcontrol.wait; an L2 prefetch of its lines is safe before (L2 is
    // where global memory is coherent: the writes land in the lines prefetched), and
    // the reads after the wait then find them there instead of in HBM.
    {
        const char* xb = static_cast<const char*>(p.x);
        const int items = (na + gb1 - gb0) * M;
        for (int i = ctid; i < items; i += CTHREADS) {
            const int t = i % M, j = i / M;
            const int g = j < na ? ga0 + j : gb0 + (j - na);
            const char* a = xb + (static_cast<long long>(t) * p.K + g * GS) * sizeof(T);
            asm volatile("prefetch.global.L2 [%0];\n" ::"l"(a));
        }
    }
    asm volatile("griddepcontrol.wait;\n" ::: "memory");

    // x[M, K] -> f16 B fragments and records, for the groups this CTA's units use
    // ([ga0, ga1) and [gb0, gb1) above), stored by the group's position in those ranges
    // (at most p.GL of them), not by its index in K.
    {
        const T* xg = static_cast<const T*>(p.x);
        qt_stage_activations<T, BITS, GS, TM>(
            xf, rec, na + gb1 - gb0,
            [&](int t) -> const T* { return t < M ? xg + static_cast<long long>(t) * p.K : nullptr; },
            [&](int j) -> int { return j < na ? ga0 + j : gb0 + (j - na); }, ctid);
    }
    named_bar_sync(1, CTHREADS);

    const QtConsumer<T, BITS, GS, TM, BR> cons(warp, lane, xf, rec);
    const T* biasg = static_cast<const T*>(p.bias);
    T* og = static_cast<T*>(p.out);

    // Last contributor to row block rb_: adds the contributors' fp32 partials in CTA
    // order, writes the outputs and re-arms the ticket.
    auto reduce_row_block = [&](int rb_) {
        const long long ub = static_cast<long long>(rb_) * S;
        const int nc = owner(ub + S - 1, U, P) - owner(ub, U, P) + 1;
        const float* part = p.partial + static_cast<long long>(rb_) * p.maxc * M * BR;
        const int row0 = rb_ * BR;
        const int rows_here = min(BR, N - row0);
        if constexpr (EPI == 2) {
            for (int idx = ctid; idx < M * rows_here; idx += CTHREADS) {
                const int t = idx / rows_here, rw = idx % rows_here;
                float v = 0.f;
                for (int k = 0; k < nc; ++k) v += __ldcg(part + (k * M + t) * BR + rw);
                T y = ET::from_f(v);
                if (biasg) y = ET::from_f(ET::to_f(y) + ET::to_f(biasg[row0 + rw]));
                atomicMax(s_best + t, argmax_key(ET::to_f(y), row0 + rw));
            }
        } else if constexpr (EPI == 1) {
            // pairs (gate row 16i + j, up row 16i + j + 8) -> out column row0/2 + 8i + j
            const int pairs = rows_here / 2;
            for (int idx = ctid; idx < M * pairs; idx += CTHREADS) {
                const int t = idx / pairs, pr = idx % pairs;
                const int rw = 16 * (pr >> 3) + (pr & 7);
                float g = 0.f, u = 0.f;
                for (int k = 0; k < nc; ++k) {
                    g += __ldcg(part + (k * M + t) * BR + rw);
                    u += __ldcg(part + (k * M + t) * BR + rw + 8);
                }
                og[static_cast<long long>(t) * (N / 2) + row0 / 2 + pr] = swiglu_out<T>(g, u);
            }
        } else {
            for (int idx = ctid; idx < M * rows_here; idx += CTHREADS) {
                const int t = idx / rows_here, rw = idx % rows_here;
                float v = 0.f;
                for (int k = 0; k < nc; ++k) v += __ldcg(part + (k * M + t) * BR + rw);
                T y = ET::from_f(v);
                if (biasg) y = ET::from_f(ET::to_f(y) + ET::to_f(biasg[row0 + rw]));
                og[static_cast<long long>(t) * N + row0 + rw] = y;
            }
        }
        if (ctid == 0) p.counter[rb_] = 0u;
    };

    uint32_t it = 0;
    int slot = 0;
    uint32_t phase = 0;  // parity of the full-barrier phase to wait for
    long long u = u_lo;
    while (u < u_hi) {
        const int rb = static_cast<int>(u / S);
        const int st0 = static_cast<int>(u % S);
        const int st_end = static_cast<int>(st0 + (u_hi - u) < S ? st0 + (u_hi - u) : S);
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
        // local position of stage st0 in the staged ranges: range a holds stages
        // ga0/SG.., range b (a share that wraps into the next row block) stages 0..
        const int lst = st0 >= ga0 / SG ? st0 - ga0 / SG : na / SG + st0;
        const uint8_t* xs = cons.x_at(lst);
        const float4* rs = cons.rec_at(lst);

        for (int st = st0; st < st_end; ++st, ++it) {
            if (!*s_abort) {
                const uint32_t fb = smem_u32(full + slot);
                if (!mbar_try_wait(fb, phase) && !wait_slow(fb, phase)) {
                    atomicCAS(p.err, 0, kErrTimeout);
                    *s_abort = 1;
                }
            }
            cons.stage(ring + slot * STAGE, xs, rs, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(empty + slot));
            xs += SG * TM * XG;
            rs += SG * TM;
            if (++slot == stages) {
                slot = 0;
                phase ^= 1u;
            }
        }

        // ---- combine the group-interleaved warps of each row tile (fixed order)
        cons.combine(red, lane, acc);
        const bool abort = *s_abort != 0;
        const int row0 = rb * BR;
        if (st0 == 0 && st_end == S) {
            // the whole row block is this CTA's: write the outputs
            if (kq == 0 && !abort) {
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                if constexpr (EPI == 2) {
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const int n = row0 + 16 * rt + r + 8 * hh;
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const int t = 8 * nt + 2 * c + q;
                            if (t < M && n < N) {
                                T y = ET::from_f(acc[nt][2 * hh + q]);
                                if (biasg) y = ET::from_f(ET::to_f(y) + ET::to_f(biasg[n]));
                                atomicMax(s_best + t, argmax_key(ET::to_f(y), n));
                            }
                        }
                    }
                } else if constexpr (EPI == 1) {
                    // this lane holds gate row r and up row r + 8 of its tile
                    const int n = (row0 + 16 * rt) / 2 + r;
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int t = 8 * nt + 2 * c + q;
                        if (t < M && 2 * n < N)
                            og[static_cast<long long>(t) * (N / 2) + n] =
                                swiglu_out<T>(acc[nt][q], acc[nt][2 + q]);
                    }
                } else {
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const int n = row0 + 16 * rt + r + 8 * hh;
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const int t = 8 * nt + 2 * c + q;
                            if (t < M && n < N) {
                                T y = ET::from_f(acc[nt][2 * hh + q]);
                                if (biasg) y = ET::from_f(ET::to_f(y) + ET::to_f(biasg[n]));
                                og[static_cast<long long>(t) * N + n] = y;
                            }
                        }
                    }
                }
              }
            }
        } else {
            // part of a row block: fp32 partial, then the last contributor reduces
            const int first = owner(static_cast<long long>(rb) * S, U, P);
            const int ci = blockIdx.x - first;
            float* part = p.partial + static_cast<long long>(rb) * p.maxc * M * BR;
            if (kq == 0 && !abort) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int rw = 16 * rt + r + 8 * hh;
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int t = 8 * nt + 2 * c + q;
                        if (t < M && row0 + rw < N)
                            part[(ci * M + t) * BR + rw] = acc[nt][2 * hh + q];
                    }
                }
            }
            if (HEADS && has_head && u == u_lo) {
                // head row block, more units follow: hand the ticket to the ticket warp
                // (mbarrier arrive: release of this warp's partials at CTA scope)
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(head_done));
            } else {
                // The barrier orders every thread's partial before thread 0's acq_rel
                // ticket; its release makes them visible GPU-wide (cumulatively) and its
                // acquire, with the second barrier, the other CTAs' partials to this one.
                named_bar_sync(1, CTHREADS);
                if (ctid == 0) {
                    const int nc = owner(static_cast<long long>(rb) * S + S - 1, U, P) - first + 1;
                    *s_last = (!abort && atom_add_acq_rel_gpu(p.counter + rb, 1u) ==
                                             static_cast<unsigned>(nc - 1));
                }
                named_bar_sync(1, CTHREADS);
                if (*s_last) reduce_row_block(rb);
            }
        }
        u += st_end - st0;
    }
    if constexpr (HEADS) {
        if (has_head) {
            // the head row block's ticket (taken by the ticket warp)
            const uint32_t tb_bar = smem_u32(ticket_done);
            if (!mbar_try_wait(tb_bar, 0) && !wait_slow(tb_bar, 0)) {
                atomicCAS(p.err, 0, kErrTimeout);
                *s_abort = 1;
            } else if (*s_head_last) {
                reduce_row_block(head_rb);
            }
        }
    }
    if constexpr (EPI == 2) {
        // this CTA's best key per token -> the global keys; the last CTA to get here
        // (acq_rel done counter, as for the row-block tickets) turns them into token
        // ids and re-arms keys and counter for the next call
        named_bar_sync(1, CTHREADS);
        if (ctid < M && s_best[ctid] != 0ull) atomicMax(p.am_keys + ctid, s_best[ctid]);
        named_bar_sync(1, CTHREADS);
        if (ctid == 0)
            *s_last = atom_add_acq_rel_gpu(p.am_done, 1u) == static_cast<unsigned>(P - 1);
        named_bar_sync(1, CTHREADS);
        if (*s_last) {
            if (ctid < M) {
                const unsigned long long k = atomicExch(p.am_keys + ctid, 0ull);
                static_cast<int*>(p.out)[ctid] =
                    static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
            }
            if (ctid == 0) *p.am_done = 0u;
        }
    }
}

}  // namespace mlxq
