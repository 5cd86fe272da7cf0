// Skinny (decode-shaped) group-wise affine quantized matmul on sm_100a tensor cores.
//
//   out[t, n] = sum_k x[t, k] * (scale[n, k/g] * q[n, k] + bias[n, k/g])
//
// for up to 32 tokens t per pass (MLX's quantized_matmul with transpose=True,
// as QuantizedLinear calls it at qwen2.py:58-61,123-134 of the reference, and
// gather_qmm's per-expert products, lfm2.py:176-187).
//
// Work decomposition
//   * A CTA owns 128 weight rows (8 row tiles of 16) and a contiguous range of
//     quantization groups (a K split). Weight rows are the M side of an
//     m16n8k16 MMA, tokens the N side (8 per n-tile).
//   * Each row tile is served by KSW warps that take alternate 128-byte chunks
//     of K (KSW = 2 for up to 16 tokens: 16 warps per SM hide the MMA and
//     shared-memory latencies); their partial sums meet in shared memory at
//     the end, in a fixed order.
//   * Weights stream HBM -> shared memory with 16-byte cp.async copies into a
//     STAGES-deep ring private to each warp: one stage is 16 rows x 128 bytes
//     (CG groups) plus the matching scales/biases. No block-wide barrier in
//     the steady state; the hardware wait_group retires copies.
//   * Activations of the CTA's K window are loaded once and stored in shared
//     memory already permuted into MMA B fragments (lane-interleaved so the
//     128-bit fragment loads are conflict free), with two per-group sums per
//     token: S = sum x and T = sum x * (field offset of its code position).
//   * Codes become MMA A operands with one LOP3 per pair (plus one shift per
//     32-bit word): see Elem<T>. The K order inside an MMA is permuted to match
//     the extraction; the B fragments carry the same permutation.
//   * Each group gets a fresh fp32 accumulator D = sum x*(offset + q); the
//     group epilogue folds acc += scale*(D - T) + bias*S in fp32, so no rounded
//     dequantized weight ever exists.
//   * K splits across CTAs (small N) write fp32 partials to the workspace; the
//     last CTA of a row block (atomic ticket, no waiting) sums them in split
//     order, so results are deterministic, and resets its ticket to zero.
#pragma once

#include "common.cuh"
#include "launch.h"

namespace mlxq {

constexpr int kRowTiles = 8;  // 16-row warp tiles per CTA: 128 rows

// Geometry shared by the kernel (as constants) and the host planner.
struct QmvGeom {
    int wpg;         // packed words per group per row
    int wpt;         // words per thread per group
    int cg;          // groups per 128-byte stage row
    int rw;          // stage row stride in words (padded: conflict-free fragment loads)
    int fr;          // B-fragment words per (group, n-tile, lane)
    int sw;          // words per stage
    int ksw;         // warps per row tile (K interleave)
    int stages;      // cp.async ring depth
    int nwarp;       // warps per CTA
    int stage_bytes; // all warps' rings
    int per_group;   // shared bytes per group of the activation window
    int red_bytes;   // cross-warp reduction buffer
};

// two_sums: per-group activation sums carry (S, T) instead of S alone (f16 4-bit,
// whose even and odd code positions have different operand offsets).
__host__ __device__ constexpr QmvGeom qmv_geom(int bits, int gs, int nt, bool sbv,
                                               bool two_sums) {
    const int wpg = gs * bits / 32;
    const int wpt = wpg / 4;
    const int cg = 32 / wpg;
    const int padw = (wpt == 1) ? 4 : (wpt == 2) ? 8 : (wpt == 4) ? 16 : 4;
    const int rw = 32 + padw;
    const int sw = 16 * rw + (sbv ? 16 * cg : 0);
    const int ksw = nt <= 2 ? 2 : 1;
    const int stages = ksw == 2 ? 3 : 4;
    const int nwarp = kRowTiles * ksw;
    return QmvGeom{wpg, wpt, cg, rw, gs / 8, sw, ksw, stages, nwarp,
                   nwarp * stages * sw * 4,
                   nt * 32 * (gs / 8) * 4 + nt * 8 * (two_sums ? 8 : 4),
                   (ksw - 1) * kRowTiles * nt * 4 * 32 * 4};
}

template <typename T, int BITS>
__host__ __device__ constexpr bool qmv_two_sums() {
    return !Elem<T>::template Off<BITS>::kUniform;
}

// ODD = false: every pass has one token, so the fold of odd token columns is
// skipped (decode at batch 1).
template <typename T, int BITS, int GS, int NT, bool SBV, bool ODD>
__global__ void __launch_bounds__(qmv_geom(BITS, GS, NT, SBV, qmv_two_sums<T, BITS>()).nwarp * 32, 1)
    qmv_kernel(const QmvParams p) {
    using E = Elem<T>;
    using OFF = typename Elem<T>::template Off<BITS>;
    constexpr bool TWO = !OFF::kUniform;
    constexpr QmvGeom GEO = qmv_geom(BITS, GS, NT, SBV, TWO);
    constexpr int WPG = GEO.wpg, WPT = GEO.wpt, CG = GEO.cg, RW = GEO.rw, FR = GEO.fr;
    constexpr int SW = GEO.sw, KSW = GEO.ksw, STAGES = GEO.stages, NTHR = GEO.nwarp * 32;
    constexpr int TOK = NT * 8;
    static_assert(WPT >= 1 && FR % 4 == 0, "unsupported group geometry");

    extern __shared__ __align__(16) uint32_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rt = warp % kRowTiles, kh = warp / kRowTiles;
    const int r = lane >> 2, c = lane & 3;
    const int N = p.N, K = p.K;
    const int G = K / GS;
    const long long kw = static_cast<long long>(K) * BITS / 32;
    const int split = blockIdx.y;
    const int g_begin = split * p.gps;
    const int g_end = min(G, g_begin + p.gps);
    const int row_block0 = blockIdx.x * (kRowTiles * 16);
    const int row0 = row_block0 + rt * 16;

    // shared memory: [win][NT][FR/4][32] uint4 fragments | [win][TOK] sums (float or
    // float2) | cross-warp reduction | per-warp cp.async rings
    uint4* xfrag = reinterpret_cast<uint4*>(smem);
    float* sums = reinterpret_cast<float*>(xfrag + static_cast<size_t>(p.win) * NT * (FR / 4) * 32);
    float* red = sums + static_cast<size_t>(p.win) * TOK * (TWO ? 2 : 1);
    uint32_t* stage0 = reinterpret_cast<uint32_t*>(red + (KSW - 1) * kRowTiles * NT * 4 * 32) +
                       warp * STAGES * SW;

    const T* xg = static_cast<const T*>(p.x);
    T* og = static_cast<T*>(p.out);
    __shared__ int s_last;
    const uint32_t magic_a = opaque(E::template Magic<BITS>::kA);
    const uint32_t magic_b = opaque(E::template Magic<BITS>::kB);

    // Launch-overlap protocol (griddepcontrol is a no-op when the launch did not opt
    // in): the next kernel on the stream may start as soon as SMs free up; this
    // kernel reads only weights, scales and biases before griddepcontrol.wait, and
    // activations, index arrays and every global write come after it.
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    bool waited = false;
    auto wait_prior = [&]() {
        if (!waited) {
            asm volatile("griddepcontrol.wait;\n" ::: "memory");
            waited = true;
        }
    };
    if (p.mode != 0) wait_prior();  // gather modes read index arrays first

    for (int z = blockIdx.z; z < p.ztotal; z += gridDim.z) {
        // ---- resolve the work item: expert, token rows ------------------------------
        int expert = 0, tok_total = 0, seg_lo = 0, zb = 0;
        if (p.mode == 0) {
            tok_total = min(TOK, p.M - z * TOK);
        } else if (p.mode == 1) {
            zb = z;
            expert = p.rhs[z];
            const long long xi = p.lhs ? p.lhs[z] : z / p.lhs_div;
            // Out-of-range indices leave the item's rows unwritten (no access).
            tok_total = (expert >= 0 && expert < p.num_experts && xi >= 0 && xi < p.x_batches)
                            ? p.M : 0;
        } else {
            expert = z;
            seg_lo = p.seg[z];
            const int seg_hi = p.seg[z + 1];
            // A table that is not a valid partition (indices not sorted) skips the item.
            tok_total = (seg_lo >= 0 && seg_hi <= p.batch && seg_hi >= seg_lo)
                            ? (seg_hi - seg_lo) * p.M : 0;
        }
        if (tok_total <= 0) continue;
        const uint32_t* wbase = p.w + static_cast<long long>(expert) * p.w_estride;
        const T* sbase = static_cast<const T*>(p.s) + static_cast<long long>(expert) * p.sb_estride;
        const T* bbase = static_cast<const T*>(p.b) + static_cast<long long>(expert) * p.sb_estride;

        // token t of this item -> (x row, out row)
        auto rows_of = [&](int t, long long& xrow, long long& orow) {
            if (p.mode == 0) {
                xrow = orow = static_cast<long long>(z) * TOK + t;
            } else {
                const int b = (p.mode == 1) ? zb : seg_lo + t / p.M;
                const int mm = (p.mode == 1) ? t : t % p.M;
                const long long xi = p.lhs ? p.lhs[b] : b / p.lhs_div;
                xrow = xi * p.M + mm;
                orow = static_cast<long long>(b) * p.M + mm;
            }
        };

        for (int tc = 0; tc < tok_total; tc += TOK) {
            const int ntok = min(TOK, tok_total - tc);
            float acc[NT][4];
#pragma unroll
            for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

            for (int w0 = g_begin; w0 < g_end; w0 += p.win) {
                const int wn = min(p.win, g_end - w0);
                const int nchunks = (wn + CG - 1) / CG;
                const int my_n = (nchunks - kh + KSW - 1) / KSW;  // chunks kh, kh+KSW, ...

                // Per-lane copy descriptors: lane copies 16-byte column `col` of rows
                // lane/8 + 4*it of every chunk, and one row of scales or biases. Rows past
                // N copy zero bytes from a valid address and never advance.
                const int col = lane & 7;
                const int grp_in_chunk = (col * 4) / WPG;
                const uint32_t* wptr[4];
                int wbytes[4];
                long long wstep[4];
#pragma unroll
                for (int it = 0; it < 4; ++it) {
                    const int n = row0 + (lane >> 3) + 4 * it;
                    const bool ok = n < N;
                    wbytes[it] = ok ? 16 : 0;
                    wstep[it] = ok ? static_cast<long long>(KSW) * 32 : 0;
                    wptr[it] = ok ? wbase + static_cast<long long>(n) * kw +
                                        static_cast<long long>(w0 + kh * CG) * WPG + col * 4
                                  : wbase;
                }
                const int srow = row0 + (lane & 15);
                const int sbytes = srow < N ? CG * 2 : 0;
                const T* sb0 = (lane < 16) ? sbase : bbase;
                const T* sbptr = sbytes ? sb0 + static_cast<long long>(srow) * G + w0 + kh * CG : sb0;
                const int sbstep = sbytes ? KSW * CG : 0;
                uint32_t* sdst0 = stage0 + 16 * RW + (lane < 16 ? 0 : 8 * CG) + (lane & 15) * (CG / 2);
                int issue_i = 0;

                auto issue = [&](int slot) {
                    uint32_t* dst = stage0 + slot * SW;
                    const int gch = w0 + (kh + issue_i * KSW) * CG;
#pragma unroll
                    for (int it = 0; it < 4; ++it) {
                        if constexpr (SBV) {
                            // invalid rows keep a valid source address and copy 0 bytes
                            cp_async16(dst + ((lane >> 3) + 4 * it) * RW + col * 4, wptr[it],
                                       wbytes[it]);
                        } else {
                            const int nb = (gch + grp_in_chunk < w0 + wn) ? wbytes[it] : 0;
                            cp_async16(dst + ((lane >> 3) + 4 * it) * RW + col * 4,
                                       nb ? wptr[it] : wbase, nb);
                        }
                        wptr[it] += wstep[it];
                    }
                    if constexpr (SBV) {
                        uint32_t* sdst = sdst0 + slot * SW;
                        if constexpr (CG == 8) cp_async16(sdst, sbptr, sbytes);
                        else if constexpr (CG == 4) cp_async8(sdst, sbptr, sbytes);
                        else cp_async4(sdst, sbptr, sbytes);
                        sbptr += sbstep;
                    }
                    cp_async_commit();
                    ++issue_i;
                };

                // Start streaming weights before building the activation fragments.
#pragma unroll
                for (int i = 0; i < STAGES - 1; ++i) {
                    if (i < my_n) issue(i);
                    else cp_async_commit();
                }
                wait_prior();

                // ---- activation window -> B fragments + per-group sums ---------------------
                __syncthreads();  // previous window / item finished reading the window
                {
                    // Loads of PB entries are issued before any is used, so a thread
                    // pays one memory round trip per PB entries.
                    constexpr int PB = (WPT <= 2) ? 4 : 2;
                    constexpr int XW = (BITS == 4) ? 4 : 2;  // activation words per packed word
                    const int total = wn * NT * 32;
                    for (int base = threadIdx.x; base < total; base += PB * NTHR) {
                        uint32_t raw[PB][WPT][XW];
#pragma unroll
                        for (int b = 0; b < PB; ++b) {
                            const int idx = base + b * NTHR;
                            const int ln = idx & 31;
                            const int jj = (idx >> 5) % NT;
                            const int gi = (idx >> 5) / NT;
                            const int tt = jj * 8 + (ln >> 2);
                            const int cc = ln & 3;
                            long long xrow = -1, orow = 0;
                            if (idx < total && tt < ntok) rows_of(tc + tt, xrow, orow);
                            const bool live =
                                xrow >= 0 && xrow < static_cast<long long>(p.x_batches) * p.M;
#pragma unroll
                            for (int w = 0; w < WPT; ++w) {
                                const long long gw =
                                    static_cast<long long>(w0 + gi) * WPG + cc * WPT + w;
                                if constexpr (BITS == 4) {
                                    uint4 u = make_uint4(0u, 0u, 0u, 0u);
                                    if (live) u = *reinterpret_cast<const uint4*>(xg + xrow * K + gw * 8);
                                    raw[b][w][0] = u.x; raw[b][w][1] = u.y;
                                    raw[b][w][2] = u.z; raw[b][w][3] = u.w;
                                } else {
                                    uint2 u = make_uint2(0u, 0u);
                                    if (live) u = *reinterpret_cast<const uint2*>(xg + xrow * K + gw * 4);
                                    raw[b][w][0] = u.x; raw[b][w][1] = u.y;
                                }
                            }
                        }
#pragma unroll
                        for (int b = 0; b < PB; ++b) {
                            const int idx = base + b * NTHR;
                            if (idx >= total) break;  // warp-uniform: total is a multiple of 32
                            const int ln = idx & 31;
                            const int jj = (idx >> 5) % NT;
                            const int gi = (idx >> 5) / NT;
                            const int tt = jj * 8 + (ln >> 2);
                            const int cc = ln & 3;
                            uint32_t fr[FR];
                            float se = 0.f, so = 0.f;
#pragma unroll
                            for (int w = 0; w < WPT; ++w) {
                                const uint32_t* u = raw[b][w];
                                if constexpr (BITS == 4) {
                                    fr[4 * w + 0] = prmt(u[0], u[2], 0x5410);  // x0, x4
                                    fr[4 * w + 1] = prmt(u[0], u[2], 0x7632);  // x1, x5
                                    fr[4 * w + 2] = prmt(u[1], u[3], 0x5410);  // x2, x6
                                    fr[4 * w + 3] = prmt(u[1], u[3], 0x7632);  // x3, x7
                                    se += (E::lo(u[0]) + E::lo(u[1])) + (E::lo(u[2]) + E::lo(u[3]));
                                    so += (E::hi(u[0]) + E::hi(u[1])) + (E::hi(u[2]) + E::hi(u[3]));
                                } else {
                                    fr[2 * w + 0] = prmt(u[0], u[1], 0x5410);  // x0, x2
                                    fr[2 * w + 1] = prmt(u[0], u[1], 0x7632);  // x1, x3
                                    se += (E::lo(u[0]) + E::hi(u[0])) + (E::lo(u[1]) + E::hi(u[1]));
                                }
                            }
                            se += __shfl_xor_sync(0xffffffffu, se, 1);
                            se += __shfl_xor_sync(0xffffffffu, se, 2);
                            so += __shfl_xor_sync(0xffffffffu, so, 1);
                            so += __shfl_xor_sync(0xffffffffu, so, 2);
                            uint4* dst = xfrag + static_cast<size_t>(gi * NT + jj) * (FR / 4) * 32 + ln;
#pragma unroll
                            for (int f = 0; f < FR / 4; ++f)
                                dst[f * 32] = make_uint4(fr[4 * f], fr[4 * f + 1], fr[4 * f + 2], fr[4 * f + 3]);
                            if (cc == 0) {
                                if constexpr (TWO) {
                                    reinterpret_cast<float2*>(sums)[gi * TOK + tt] =
                                        make_float2(se + so, OFF::kOffE * se + OFF::kOffO * so);
                                } else {
                                    sums[gi * TOK + tt] = se + so;
                                }
                            }
                        }
                    }
                }
                __syncthreads();

                // ---- main loop over this warp's 128-byte chunks ----------------------------
                // Unrolled by the ring depth so every stage slot is a constant.
                auto chunk = [&](const int i, const uint32_t* sw) {
                    const int ch = kh + i * KSW;
                    // packed scales / biases of this chunk for rows r and r+8
                    uint32_t sp0[CG / 2 > 0 ? CG / 2 : 1], sp1[CG / 2 > 0 ? CG / 2 : 1];
                    uint32_t bp0[CG / 2 > 0 ? CG / 2 : 1], bp1[CG / 2 > 0 ? CG / 2 : 1];
                    if constexpr (SBV) {
                        const uint32_t* sp = sw + 16 * RW;
                        const uint32_t* bp = sp + 8 * CG;
                        auto ld = [](const uint32_t* a, uint32_t* dst) {
                            if constexpr (CG == 8) {
                                const uint4 v = *reinterpret_cast<const uint4*>(a);
                                dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
                            } else if constexpr (CG == 4) {
                                const uint2 v = *reinterpret_cast<const uint2*>(a);
                                dst[0] = v.x; dst[1] = v.y;
                            } else {
                                dst[0] = a[0];
                            }
                        };
                        ld(sp + r * (CG / 2), sp0);
                        ld(sp + (r + 8) * (CG / 2), sp1);
                        ld(bp + r * (CG / 2), bp0);
                        ld(bp + (r + 8) * (CG / 2), bp1);
                    }
#pragma unroll
                    for (int gi = 0; gi < CG; ++gi) {
                        const int gl = ch * CG + gi;  // group index within the window
                        if (!SBV && gl >= wn) continue;
                        float s0, s1, b0, b1;
                        if constexpr (SBV) {
                            const int q = gi >> 1;
                            s0 = (gi & 1) ? E::hi(sp0[q]) : E::lo(sp0[q]);
                            s1 = (gi & 1) ? E::hi(sp1[q]) : E::lo(sp1[q]);
                            b0 = (gi & 1) ? E::hi(bp0[q]) : E::lo(bp0[q]);
                            b1 = (gi & 1) ? E::hi(bp1[q]) : E::lo(bp1[q]);
                        } else {
                            const int g = w0 + gl;
                            const int n0 = row0 + r, n1 = row0 + r + 8;
                            s0 = n0 < N ? E::to_f(sbase[static_cast<long long>(n0) * G + g]) : 0.f;
                            b0 = n0 < N ? E::to_f(bbase[static_cast<long long>(n0) * G + g]) : 0.f;
                            s1 = n1 < N ? E::to_f(sbase[static_cast<long long>(n1) * G + g]) : 0.f;
                            b1 = n1 < N ? E::to_f(bbase[static_cast<long long>(n1) * G + g]) : 0.f;
                        }
                        uint32_t wa[WPT], wb[WPT];
                        {
                            const uint32_t* pa = sw + r * RW + gi * WPG + c * WPT;
                            const uint32_t* pb = pa + 8 * RW;
                            if constexpr (WPT == 1) {
                                wa[0] = pa[0];
                                wb[0] = pb[0];
                            } else if constexpr (WPT == 2) {
                                const uint2 a = *reinterpret_cast<const uint2*>(pa);
                                const uint2 b = *reinterpret_cast<const uint2*>(pb);
                                wa[0] = a.x; wa[1] = a.y;
                                wb[0] = b.x; wb[1] = b.y;
                            } else {
#pragma unroll
                                for (int q = 0; q < WPT / 4; ++q) {
                                    const uint4 a = reinterpret_cast<const uint4*>(pa)[q];
                                    const uint4 b = reinterpret_cast<const uint4*>(pb)[q];
                                    wa[4 * q + 0] = a.x; wa[4 * q + 1] = a.y;
                                    wa[4 * q + 2] = a.z; wa[4 * q + 3] = a.w;
                                    wb[4 * q + 0] = b.x; wb[4 * q + 1] = b.y;
                                    wb[4 * q + 2] = b.z; wb[4 * q + 3] = b.w;
                                }
                            }
                        }
                        uint32_t ta[WPT][4], tb[WPT][4];
#pragma unroll
                        for (int w = 0; w < WPT; ++w) {
                            E::template extract<BITS>(wa[w], ta[w], magic_a, magic_b);
                            E::template extract<BITS>(wb[w], tb[w], magic_a, magic_b);
                        }
                        float cr0 = 0.f, cr1 = 0.f;
                        if constexpr (!TWO) {
                            cr0 = fmaf(-OFF::kOff, s0, b0);
                            cr1 = fmaf(-OFF::kOff, s1, b1);
                        }
#pragma unroll
                        for (int j = 0; j < NT; ++j) {
                            uint32_t X[FR];
                            const uint4* xf = xfrag + static_cast<size_t>(gl * NT + j) * (FR / 4) * 32 + lane;
#pragma unroll
                            for (int f = 0; f < FR / 4; ++f) {
                                const uint4 v = xf[f * 32];
                                X[4 * f + 0] = v.x; X[4 * f + 1] = v.y;
                                X[4 * f + 2] = v.z; X[4 * f + 3] = v.w;
                            }
                            float d[4];
#pragma unroll
                            for (int w = 0; w < WPT; ++w) {
                                if constexpr (BITS == 4) {
                                    if (w == 0)
                                        mma16816z<T>(d, ta[w][0], tb[w][0], ta[w][1], tb[w][1],
                                                     X[4 * w + 0], X[4 * w + 1]);
                                    else
                                        mma16816<T>(d, ta[w][0], tb[w][0], ta[w][1], tb[w][1],
                                                    X[4 * w + 0], X[4 * w + 1]);
                                    mma16816<T>(d, ta[w][2], tb[w][2], ta[w][3], tb[w][3],
                                                X[4 * w + 2], X[4 * w + 3]);
                                } else {
                                    if (w == 0)
                                        mma16816z<T>(d, ta[w][0], tb[w][0], ta[w][1], tb[w][1],
                                                     X[2 * w + 0], X[2 * w + 0]);
                                    else
                                        mma16816<T>(d, ta[w][0], tb[w][0], ta[w][1], tb[w][1],
                                                    X[2 * w + 0], X[2 * w + 0]);
                                    mma16816<T>(d, ta[w][2], tb[w][2], ta[w][3], tb[w][3],
                                                X[2 * w + 1], X[2 * w + 1]);
                                }
                            }
                            // fold this group into the accumulators of tokens 2c and 2c+1
                            if constexpr (TWO) {
                                const float4 st = *reinterpret_cast<const float4*>(
                                    reinterpret_cast<const float2*>(sums) + gl * TOK + j * 8 + 2 * c);
                                acc[j][0] = fmaf(s0, d[0] - st.y, fmaf(b0, st.x, acc[j][0]));
                                acc[j][2] = fmaf(s1, d[2] - st.y, fmaf(b1, st.x, acc[j][2]));
                                if constexpr (ODD) {
                                    acc[j][1] = fmaf(s0, d[1] - st.w, fmaf(b0, st.z, acc[j][1]));
                                    acc[j][3] = fmaf(s1, d[3] - st.w, fmaf(b1, st.z, acc[j][3]));
                                }
                            } else {
                                const float2 sx = *reinterpret_cast<const float2*>(sums + gl * TOK + j * 8 + 2 * c);
                                acc[j][0] = fmaf(s0, d[0], fmaf(cr0, sx.x, acc[j][0]));
                                acc[j][2] = fmaf(s1, d[2], fmaf(cr1, sx.x, acc[j][2]));
                                if constexpr (ODD) {
                                    acc[j][1] = fmaf(s0, d[1], fmaf(cr0, sx.y, acc[j][1]));
                                    acc[j][3] = fmaf(s1, d[3], fmaf(cr1, sx.y, acc[j][3]));
                                }
                            }
                        }
                    }
                };
                for (int i0 = 0; i0 < my_n; i0 += STAGES) {
#pragma unroll
                    for (int u = 0; u < STAGES; ++u) {
                        const int i = i0 + u;
                        if (i < my_n) {
                            cp_async_wait<STAGES - 2>();
                            __syncwarp();
                            if (i + STAGES - 1 < my_n) issue((u + STAGES - 1) % STAGES);
                            else cp_async_commit();
                            chunk(i, stage0 + u * SW);
                        }
                    }
                }
                cp_async_wait<0>();
                __syncwarp();
            }

            // ---- combine the K-interleaved warps of each row tile (fixed order) ----------
            if constexpr (KSW > 1) {
                __syncthreads();
                if (kh > 0) {
                    float* dst = red + ((kh - 1) * kRowTiles + rt) * NT * 4 * 32 + lane;
#pragma unroll
                    for (int j = 0; j < NT; ++j)
#pragma unroll
                        for (int e = 0; e < 4; ++e) dst[(j * 4 + e) * 32] = acc[j][e];
                }
                __syncthreads();
                if (kh == 0) {
#pragma unroll
                    for (int h = 1; h < KSW; ++h) {
                        const float* src = red + ((h - 1) * kRowTiles + rt) * NT * 4 * 32 + lane;
#pragma unroll
                        for (int j = 0; j < NT; ++j)
#pragma unroll
                            for (int e = 0; e < 4; ++e) acc[j][e] += src[(j * 4 + e) * 32];
                    }
                }
            }

            // ---- epilogue ---------------------------------------------------------------
            const T* biasg = static_cast<const T*>(p.bias);
            if (p.splits == 1) {
                if (kh == 0) {
#pragma unroll
                    for (int j = 0; j < NT; ++j) {
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int n = row0 + r + 8 * h;
#pragma unroll
                            for (int q = 0; q < 2; ++q) {
                                const int t = j * 8 + 2 * c + q;
                                if (t < ntok && n < N) {
                                    long long xrow, orow;
                                    rows_of(tc + t, xrow, orow);
                                    T y = E::from_f(acc[j][2 * h + q]);
                                    if (biasg) y = E::from_f(E::to_f(y) + E::to_f(biasg[n]));
                                    og[orow * N + n] = y;
                                }
                            }
                        }
                    }
                }
            } else {
                // K split across CTAs: fp32 partial of this split, then the last CTA reduces.
                if (kh == 0) {
#pragma unroll
                    for (int j = 0; j < NT; ++j) {
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int n = row0 + r + 8 * h;
#pragma unroll
                            for (int q = 0; q < 2; ++q) {
                                const int t = j * 8 + 2 * c + q;
                                if (t < ntok && n < N) {
                                    const long long m = static_cast<long long>(z) * TOK + t;
                                    p.partial[(static_cast<long long>(split) * p.M + m) * N + n] =
                                        acc[j][2 * h + q];
                                }
                            }
                        }
                    }
                }
                __threadfence();
                __syncthreads();
                unsigned* ticket = p.counter + static_cast<long long>(z) * gridDim.x + blockIdx.x;
                if (threadIdx.x == 0)
                    s_last = (atomicAdd(ticket, 1u) == static_cast<unsigned>(p.splits - 1));
                __syncthreads();
                if (s_last) {
                    __threadfence();
                    const int rows_here = min(kRowTiles * 16, N - row_block0);
                    for (int idx = threadIdx.x; idx < ntok * rows_here; idx += NTHR) {
                        const int t = idx / rows_here;
                        const int n = row_block0 + idx % rows_here;
                        const long long m = static_cast<long long>(z) * TOK + t;
                        float v = 0.f;
                        for (int sp = 0; sp < p.splits; ++sp)
                            v += __ldcg(p.partial + (static_cast<long long>(sp) * p.M + m) * N + n);
                        T y = E::from_f(v);
                        if (biasg) y = E::from_f(E::to_f(y) + E::to_f(biasg[n]));
                        og[m * N + n] = y;
                    }
                    if (threadIdx.x == 0) *ticket = 0u;
                }
            }
        }
    }
}

}  // namespace mlxq
