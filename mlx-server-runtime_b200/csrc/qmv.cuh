// Skinny (decode-shaped) group-wise affine quantized matmul on sm_100a tensor cores.
//
//   out[t, n] = sum_k x[t, k] * (scale[n, k/g] * q[n, k] + bias[n, k/g])
//
// for up to 32 tokens t per pass (MLX's quantized_matmul with transpose=True,
// as QuantizedLinear calls it at qwen2.py:58-61,123-134 of the reference, and
// gather_qmm's per-expert products, lfm2.py:176-187).
//
// Work decomposition
//   * A warp owns 16 weight rows; a CTA of NW warps owns 16*NW rows and a
//     contiguous range of quantization groups (a K split). Weight rows are
//     the M side of a m16n8k16 MMA, tokens the N side (8 per n-tile).
//   * Weights stream HBM -> shared memory with 16-byte cp.async copies into a
//     STAGES-deep ring private to each warp: one stage is 16 rows x 128 bytes
//     (CG groups), plus the matching scales/biases. No block-wide barrier in
//     the steady state; the hardware wait_group retires copies.
//   * Activations of the CTA's K window are loaded once and stored in shared
//     memory already permuted into MMA B fragments, with the per-group sums
//     sum_k x[t,k] that the affine bias needs.
//   * A 32-bit word of codes becomes MMA A operands with one shift and one
//     LOP3 per pair of codes: (word >> s) & 0x000F000F | magic gives two
//     16-bit floats equal to OFF + q exactly (see Elem<T>). 8-bit codes are
//     split into nibbles, the high nibble carrying a x16 exponent, so the same
//     MMA sums both. The K order inside an MMA is permuted to match this
//     extraction; the B fragments carry the same permutation.
//   * Each group gets a fresh fp32 accumulator D = sum x*(OFF+q); the
//     epilogue of the group folds acc += scale*D + (bias - OFF*scale)*sum(x)
//     in fp32, so no rounded dequantized weight ever exists.
//   * K splits (small N) write fp32 partials to the workspace; the last CTA of
//     a row block (atomic ticket, no waiting) sums them in split order, so
//     results are deterministic, and resets its ticket to zero.
#pragma once

#include "common.cuh"
#include "launch.h"

namespace mlxq {

template <int BITS, int GS>
struct QmvShape {
    static constexpr int WPG = GS * BITS / 32;  // packed words per group per row
    static constexpr int WPT = WPG / 4;         // words per thread per group
    static constexpr int CG = 32 / WPG;         // groups per 128-byte stage row
    // Row padding (words) that keeps the fragment loads bank-conflict free.
    static constexpr int PADW = (WPT == 1) ? 4 : (WPT == 2) ? 8 : (WPT == 4) ? 16 : 4;
    static constexpr int RW = 32 + PADW;        // stage row stride in words
    static constexpr int FR = GS / 8;           // B-fragment words per (group, n-tile, lane)
    static_assert(WPT >= 1, "group too small for the 4-lane split");
};

template <int BITS, int GS, bool SBV>
__host__ __device__ constexpr int qmv_stage_words() {
    return 16 * QmvShape<BITS, GS>::RW + (SBV ? 16 * QmvShape<BITS, GS>::CG : 0);
}

template <int NW, int STAGES, int BITS, int GS, bool SBV>
__host__ __device__ constexpr int qmv_stage_bytes() {
    return NW * STAGES * qmv_stage_words<BITS, GS, SBV>() * 4;
}

// Shared memory per group of the activation window for NT n-tiles.
template <int GS>
__host__ __device__ constexpr int qmv_win_bytes_per_group(int nt) {
    return nt * 32 * (GS / 8) * 4 + nt * 8 * 4;
}

template <typename T, int BITS, int GS, int NT, int NW, int STAGES, bool SBV>
__global__ void __launch_bounds__(NW * 32, 1) qmv_kernel(const QmvParams p) {
    using E = Elem<T>;
    using S = QmvShape<BITS, GS>;
    constexpr int WPG = S::WPG, WPT = S::WPT, CG = S::CG, RW = S::RW, FR = S::FR;
    constexpr int STAGE_WORDS = qmv_stage_words<BITS, GS, SBV>();
    constexpr int TOK = NT * 8;
    constexpr float OFF = (BITS == 4) ? E::kOff4 : E::kOff8;
    constexpr uint32_t MLO = E::kMagicLo, MHI = E::kMagicHi, NIB = 0x000F000Fu;

    extern __shared__ __align__(16) uint32_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = lane >> 2, c = lane & 3;
    const int N = p.N, K = p.K;
    const int G = K / GS;
    const long long kw = static_cast<long long>(K) * BITS / 32;
    const int split = blockIdx.y;
    const int g_begin = split * p.gps;
    const int g_end = min(G, g_begin + p.gps);
    const int row_block0 = blockIdx.x * (NW * 16);
    const int row0 = row_block0 + warp * 16;

    uint32_t* xfrag = smem;
    float* sumx = reinterpret_cast<float*>(smem + static_cast<size_t>(p.win) * NT * 32 * FR);
    uint32_t* stage =
        reinterpret_cast<uint32_t*>(sumx + static_cast<size_t>(p.win) * TOK) +
        warp * STAGES * STAGE_WORDS;

    const T* xg = static_cast<const T*>(p.x);
    T* og = static_cast<T*>(p.out);
    __shared__ int s_last;

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

                auto issue = [&](int ch) {
                    uint32_t* dst = stage + (ch % STAGES) * STAGE_WORDS;
                    const int gch = w0 + ch * CG;
#pragma unroll
                    for (int it = 0; it < 4; ++it) {
                        const int i = lane + 32 * it;
                        const int rr = i >> 3, col = i & 7;
                        const int grp = gch + (col * 4) / WPG;
                        const int n = row0 + rr;
                        const bool ok = (n < N) && (grp < w0 + wn);
                        const uint32_t* src =
                            ok ? wbase + static_cast<long long>(n) * kw +
                                     static_cast<long long>(gch) * WPG + col * 4
                               : wbase;
                        cp_async16(dst + rr * RW + col * 4, src, ok ? 16 : 0);
                    }
                    if constexpr (SBV) {
                        const int rr = lane & 15;
                        const int n = row0 + rr;
                        const bool ok = n < N;
                        const T* base = (lane < 16) ? sbase : bbase;
                        const T* src = ok ? base + static_cast<long long>(n) * G + gch : base;
                        uint32_t* sdst = dst + 16 * RW + (lane < 16 ? 0 : 8 * CG) + rr * (CG / 2);
                        if constexpr (CG == 8) cp_async16(sdst, src, ok ? 16 : 0);
                        else if constexpr (CG == 4) cp_async8(sdst, src, ok ? 8 : 0);
                        else cp_async4(sdst, src, ok ? 4 : 0);
                    }
                    cp_async_commit();
                };

                // Start streaming weights before building the activation fragments.
#pragma unroll
                for (int i = 0; i < STAGES - 1; ++i) {
                    if (i < nchunks) issue(i);
                    else cp_async_commit();
                }

                // ---- activation window -> B fragments + per-group sums ---------------------
                __syncthreads();  // previous window / item finished reading xfrag
                for (int idx = threadIdx.x; idx < wn * NT * 32; idx += NW * 32) {
                    const int ln = idx & 31;
                    const int jj = (idx >> 5) % NT;
                    const int gi = (idx >> 5) / NT;
                    const int tt = jj * 8 + (ln >> 2);
                    const int cc = ln & 3;
                    uint32_t fr[FR];
                    float sum = 0.f;
                    long long xrow = 0, orow = 0;
                    if (tt < ntok) rows_of(tc + tt, xrow, orow);
                    if (tt < ntok && xrow >= 0 && xrow < static_cast<long long>(p.x_batches) * p.M) {
                        const T* xr = xg + xrow * K;
#pragma unroll
                        for (int w = 0; w < WPT; ++w) {
                            const long long gw =
                                static_cast<long long>(w0 + gi) * WPG + cc * WPT + w;
                            if constexpr (BITS == 4) {
                                const uint4 u = *reinterpret_cast<const uint4*>(xr + gw * 8);
                                fr[4 * w + 0] = prmt(u.x, u.z, 0x5410);
                                fr[4 * w + 1] = prmt(u.x, u.z, 0x7632);
                                fr[4 * w + 2] = prmt(u.y, u.w, 0x5410);
                                fr[4 * w + 3] = prmt(u.y, u.w, 0x7632);
                                const T* v = reinterpret_cast<const T*>(&u);
#pragma unroll
                                for (int e = 0; e < 8; ++e) sum += E::to_f(v[e]);
                            } else {
                                const uint2 u = *reinterpret_cast<const uint2*>(xr + gw * 4);
                                fr[2 * w + 0] = prmt(u.x, u.y, 0x5410);
                                fr[2 * w + 1] = prmt(u.x, u.y, 0x7632);
                                const T* v = reinterpret_cast<const T*>(&u);
#pragma unroll
                                for (int e = 0; e < 4; ++e) sum += E::to_f(v[e]);
                            }
                        }
                    } else {
#pragma unroll
                        for (int f = 0; f < FR; ++f) fr[f] = 0u;
                    }
                    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                    uint4* dst = reinterpret_cast<uint4*>(
                        xfrag + (static_cast<size_t>(gi * NT + jj) * 32 + ln) * FR);
#pragma unroll
                    for (int f = 0; f < FR / 4; ++f)
                        dst[f] = make_uint4(fr[4 * f], fr[4 * f + 1], fr[4 * f + 2], fr[4 * f + 3]);
                    if (cc == 0) sumx[gi * TOK + tt] = sum;
                }
                __syncthreads();

                // ---- main loop over 128-byte chunks of the warp's 16 rows ------------------
                for (int ch = 0; ch < nchunks; ++ch) {
                    cp_async_wait<STAGES - 2>();
                    __syncwarp();
                    if (ch + STAGES - 1 < nchunks) issue(ch + STAGES - 1);
                    else cp_async_commit();

                    const uint32_t* sw = stage + (ch % STAGES) * STAGE_WORDS;
#pragma unroll
                    for (int gi = 0; gi < CG; ++gi) {
                        const int gl = ch * CG + gi;  // group index within the window
                        if (gl >= wn) break;
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
                        float s0, s1, b0, b1;
                        if constexpr (SBV) {
                            const T* sh = reinterpret_cast<const T*>(sw + 16 * RW);
                            const T* bh = sh + 16 * CG;
                            s0 = E::to_f(sh[r * CG + gi]);
                            s1 = E::to_f(sh[(r + 8) * CG + gi]);
                            b0 = E::to_f(bh[r * CG + gi]);
                            b1 = E::to_f(bh[(r + 8) * CG + gi]);
                        } else {
                            const int g = w0 + gl;
                            const int n0 = row0 + r, n1 = row0 + r + 8;
                            s0 = n0 < N ? E::to_f(sbase[static_cast<long long>(n0) * G + g]) : 0.f;
                            b0 = n0 < N ? E::to_f(bbase[static_cast<long long>(n0) * G + g]) : 0.f;
                            s1 = n1 < N ? E::to_f(sbase[static_cast<long long>(n1) * G + g]) : 0.f;
                            b1 = n1 < N ? E::to_f(bbase[static_cast<long long>(n1) * G + g]) : 0.f;
                        }
                        const float cr0 = fmaf(-OFF, s0, b0);
                        const float cr1 = fmaf(-OFF, s1, b1);
#pragma unroll
                        for (int j = 0; j < NT; ++j) {
                            uint32_t X[FR];
                            const uint4* xf = reinterpret_cast<const uint4*>(
                                xfrag + (static_cast<size_t>(gl * NT + j) * 32 + lane) * FR);
#pragma unroll
                            for (int f = 0; f < FR / 4; ++f) {
                                const uint4 v = xf[f];
                                X[4 * f + 0] = v.x; X[4 * f + 1] = v.y;
                                X[4 * f + 2] = v.z; X[4 * f + 3] = v.w;
                            }
                            float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                            for (int w = 0; w < WPT; ++w) {
                                if constexpr (BITS == 4) {
                                    const uint32_t a0 = (wa[w] & NIB) | MLO;
                                    const uint32_t a1 = ((wa[w] >> 4) & NIB) | MLO;
                                    const uint32_t a2 = ((wa[w] >> 8) & NIB) | MLO;
                                    const uint32_t a3 = ((wa[w] >> 12) & NIB) | MLO;
                                    const uint32_t b0_ = (wb[w] & NIB) | MLO;
                                    const uint32_t b1_ = ((wb[w] >> 4) & NIB) | MLO;
                                    const uint32_t b2_ = ((wb[w] >> 8) & NIB) | MLO;
                                    const uint32_t b3_ = ((wb[w] >> 12) & NIB) | MLO;
                                    mma16816<T>(d, a0, b0_, a1, b1_, X[4 * w + 0], X[4 * w + 1]);
                                    mma16816<T>(d, a2, b2_, a3, b3_, X[4 * w + 2], X[4 * w + 3]);
                                } else {
                                    const uint32_t l0 = (wa[w] & NIB) | MLO;
                                    const uint32_t h0 = ((wa[w] >> 4) & NIB) | MHI;
                                    const uint32_t l1 = ((wa[w] >> 8) & NIB) | MLO;
                                    const uint32_t h1 = ((wa[w] >> 12) & NIB) | MHI;
                                    const uint32_t m0 = (wb[w] & NIB) | MLO;
                                    const uint32_t k0 = ((wb[w] >> 4) & NIB) | MHI;
                                    const uint32_t m1 = ((wb[w] >> 8) & NIB) | MLO;
                                    const uint32_t k1 = ((wb[w] >> 12) & NIB) | MHI;
                                    mma16816<T>(d, l0, m0, h0, k0, X[2 * w + 0], X[2 * w + 0]);
                                    mma16816<T>(d, l1, m1, h1, k1, X[2 * w + 1], X[2 * w + 1]);
                                }
                            }
                            const float2 sx =
                                *reinterpret_cast<const float2*>(sumx + gl * TOK + j * 8 + 2 * c);
                            acc[j][0] = fmaf(s0, d[0], fmaf(cr0, sx.x, acc[j][0]));
                            acc[j][1] = fmaf(s0, d[1], fmaf(cr0, sx.y, acc[j][1]));
                            acc[j][2] = fmaf(s1, d[2], fmaf(cr1, sx.x, acc[j][2]));
                            acc[j][3] = fmaf(s1, d[3], fmaf(cr1, sx.y, acc[j][3]));
                        }
                    }
                }
                cp_async_wait<0>();
                __syncwarp();
            }

            // ---- epilogue ---------------------------------------------------------------
            const T* biasg = static_cast<const T*>(p.bias);
            if (p.splits == 1) {
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
            } else {
                // K-split: fp32 partial of this split, then the last CTA reduces.
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
                __threadfence();
                __syncthreads();
                unsigned* ticket = p.counter + static_cast<long long>(z) * gridDim.x + blockIdx.x;
                if (threadIdx.x == 0) s_last = (atomicAdd(ticket, 1u) == static_cast<unsigned>(p.splits - 1));
                __syncthreads();
                if (s_last) {
                    __threadfence();
                    const int rows_here = min(NW * 16, N - row_block0);
                    for (int idx = threadIdx.x; idx < ntok * rows_here; idx += NW * 32) {
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
