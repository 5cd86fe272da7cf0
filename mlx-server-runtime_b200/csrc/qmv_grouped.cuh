// Decode-shaped gather_qmm fed by TMA (sm_100a): the few token rows routed to each
// expert of an MoE layer, against that expert's weights,
//
//   out[row, n] = sum_k x[row, k] * (scale[e, n, k/g] * q[e, n, k] + bias[e, n, k/g])
//
// MLX's gather_qmm with transpose=True as QuantizedSwitchLinear calls it
// (lfm2.py:169-190 of the reference), at the small token counts of decode.
//
// Work: a chunk is up to TM token rows of one expert. Sorted entries (rhs_indices
// non-decreasing, the SwitchGLU form after _gather_sort) give each expert's rows as
// consecutive chunks; unsorted entries are one chunk each (TM >= rows per entry, or
// several). An item is one chunk times one block of BR weight rows over all of K; the
// items, chunk-major, are split into equal contiguous shares, one per CTA, so a CTA
// stages the activations of one or two chunks and streams the row blocks of their
// experts. Nothing is split along K, so there are no partial sums and no workspace.
// The chunk table is built by every CTA from the index array in shared memory (no
// extra launch and nothing read back to the host).
//
// Per CTA: one producer warp and the 8 consumer warps of the dense decode kernel
// (qmv_tma.cuh, QtConsumer: ldmatrix, LOP3 code extraction, mma.sync m16n8k16 over
// f16 activation fragments with per-slice power-of-two scaling):
//   * lane 0 streams the packed codes of each (item, 8-group stage) with 2-D TMA
//     loads (expert e's rows are rows e*N.. of a [E*N, K*bits/32] map; boxes past K
//     read zeros);
//   * all 32 lanes copy the stage's scales and biases with cp.async (rows of K/g
//     2-byte values need not be 16-byte multiples, which a TMA map would require)
//     and arrive on the stage's full barrier when their copies land (noinc).
// Every wait is bounded: a timeout records an error in *p.err, turns the remaining
// waits and the global writes off, and lets every warp run to the end.
#pragma once

#include "qmv_tma.cuh"

namespace mlxq {

namespace qgd {
constexpr int MAXE = 1024;  // experts whose chunk table fits in shared memory
constexpr int THREADS = qt::CTHREADS + 32;
// Bytes of the scale (or bias) part of a stage copied per cp.async: the largest
// power of two up to 16 that divides a row of scales (2 G bytes, G even), so every
// copy is aligned and none straddles the end of a row.
__host__ __device__ constexpr int sb_copy_bytes(int G) {
    return (2 * G) % 16 == 0 ? 16 : (2 * G) % 8 == 0 ? 8 : 4;
}

struct Layout {
    int ring, xf, rec, red, bars, flags, seg, cs, total;
};
// Shared-memory layout (from a 1024-byte aligned base), in bytes.
__host__ __device__ inline Layout layout(int stage_bytes, int stages, int Gp, int TM, int xg,
                                         int rt, int E, bool sorted) {
    Layout L;
    L.ring = 0;
    L.xf = stages * stage_bytes;                  // [Gp][FR/4][TM][4 lanes] x 16 B
    L.rec = L.xf + Gp * TM * xg;                  // [Gp][TM] float4 records
    L.red = L.rec + Gp * TM * 16;                 // cross-warp reduction
    L.bars = (L.red + (qt::CWARPS - rt) * qt::n_tiles(TM) * 4 * 32 * 4 + 7) & ~7;
    L.flags = (L.bars + 2 * stages * 8 + 15) & ~15;  // full[stages], empty[stages]; abort
    L.seg = L.flags + 16;                         // sorted: first entry of expert e, [E+1]
    L.cs = L.seg + (sorted ? (E + 1) * 4 : 0);    // sorted: first chunk of expert e, [E+1]
    L.total = L.cs + (sorted ? (E + 1) * 4 : 0);
    return L;
}
}  // namespace qgd

struct QgdParams {
    const void* x;        // [x_batches * M, K]
    const void* s;        // scales [E * N, G]
    const void* b;        // biases [E * N, G]
    void* out;            // [batch * M, N]
    const int32_t* rhs;   // expert of each entry
    const int32_t* lhs;   // x entry of each entry (null: entry / lhs_div)
    int lhs_div;
    int batch, x_batches;
    int M;                // rows per entry
    int N, K, G, E;
    int S;                // stages (8 groups each) per item: ceil(G / 8)
    int RB;               // row blocks of N
    int stages;           // ring depth
    int sorted;
    int* err;
};

// EPI 0: the outputs out[row, n]. EPI 1: SwiGLU over gate/up rows interleaved by
// 16-row tiles in every expert (as the dense decode kernel's epilogue 1): out[row, c]
// = silu(gate) * up for the N / 2 columns, each projection rounded to T first.
template <typename T, int BITS, int GS, int TM, int BR, int EPI>
__global__ void __launch_bounds__(qgd::THREADS, 2)
    qmv_grouped_kernel(const __grid_constant__ CUtensorMap tw, const QgdParams p) {
    using namespace qt;
    using ET = Elem<T>;
    using GEO = Geo<BITS, GS, BR>;
    using CONS = QtConsumer<T, BITS, GS, TM, BR>;
    constexpr int WPG = GEO::WPG, XG = GEO::XG;
    constexpr int STAGE = GEO::STAGE, W_BYTES = GEO::W_BYTES, SB_BYTES = GEO::SB_BYTES;
    constexpr int RT = Rows<BR>::RT, NT = n_tiles(TM);

    extern __shared__ __align__(16) uint8_t qg_smem_raw[];
    uint8_t* base = qg_smem_raw + ((1024u - (smem_u32(qg_smem_raw) & 1023u)) & 1023u);
    const int N = p.N, E = p.E, S = p.S, RB = p.RB, stages = p.stages;
    const int Gp = S * SG;
    const bool sorted = p.sorted != 0;
    const qgd::Layout L = qgd::layout(STAGE, stages, Gp, TM, XG, RT, E, sorted);
    uint8_t* ring = base + L.ring;
    uint8_t* xf = base + L.xf;
    float4* rec = reinterpret_cast<float4*>(base + L.rec);
    float* red = reinterpret_cast<float*>(base + L.red);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bars);
    uint64_t* empty = full + stages;
    volatile int* s_abort = reinterpret_cast<volatile int*>(base + L.flags);
    int* seg = reinterpret_cast<int*>(base + L.seg);
    int* cs = reinterpret_cast<int*>(base + L.cs);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(full + s), 1 + 32);  // TMA thread + the warp's cp.async lanes
            mbar_init(smem_u32(empty + s), CWARPS);
        }
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    // Which weights to read depends on the index array, which the kernels before this
    // one write: everything waits for them (a no-op without launch overlap).
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    asm volatile("griddepcontrol.wait;\n" ::: "memory");

    // ---- chunk table (sorted): seg[e] = first entry of expert e, as segments_kernel
    // builds it (indices clamped to [-1, E]; unsorted indices leave gaps, read as
    // empty experts), cs[e] = chunks of the experts before e.
    const int cpe = (p.M + TM - 1) / TM;  // chunks per entry (unsorted)
    if (sorted) {
        for (int e = tid; e <= E; e += qgd::THREADS) seg[e] = -1;
        __syncthreads();
        for (int i = tid; i <= p.batch; i += qgd::THREADS) {
            int prev = i == 0 ? -1 : p.rhs[i - 1];
            int cur = i == p.batch ? E : p.rhs[i];
            prev = max(-1, min(prev, E));
            cur = max(-1, min(cur, E));
            for (int e = prev + 1; e <= cur; ++e) seg[e] = i;
        }
        __syncthreads();
        if (warp == 0) {
            const int per = (E + 31) / 32;
            const int e0 = min(E, lane * per), e1 = min(E, e0 + per);
            auto chunks = [&](int e) -> int {
                const int lo = seg[e], hi = seg[e + 1];
                return (lo >= 0 && hi <= p.batch && hi > lo) ? ((hi - lo) * p.M + TM - 1) / TM : 0;
            };
            int sum = 0;
            for (int e = e0; e < e1; ++e) sum += chunks(e);
            int incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            int run = incl - sum;
            for (int e = e0; e < e1; ++e) {
                cs[e] = run;
                run += chunks(e);
            }
            if (lane == 31) cs[E] = incl;
        }
    }
    __syncthreads();

    const long long C = sorted ? cs[E] : static_cast<long long>(p.batch) * cpe;
    const long long I = C * RB;
    const int P = gridDim.x;
    const long long i_lo = I * blockIdx.x / P, i_hi = I * (blockIdx.x + 1) / P;

    // chunk c -> expert, x row and out row of its first token slot, rows (0: skipped)
    struct Chunk {
        int e, rows;
        long long xrow, orow;
    };
    auto chunk_of = [&](long long c) -> Chunk {
        Chunk k{0, 0, 0, 0};
        if (sorted) {
            int lo = 0, hi = E - 1;  // the last expert whose first chunk is <= c
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (cs[mid] <= c) lo = mid;
                else hi = mid - 1;
            }
            const long long r0 = static_cast<long long>(seg[lo]) * p.M +
                                 (c - cs[lo]) * static_cast<long long>(TM);
            const long long r1 = static_cast<long long>(seg[lo + 1]) * p.M;
            k.e = lo;
            k.xrow = k.orow = r0;
            k.rows = static_cast<int>(min(static_cast<long long>(TM), r1 - r0));
        } else {
            const int b = static_cast<int>(c / cpe), part = static_cast<int>(c % cpe);
            const int e = p.rhs[b];
            const long long xi = p.lhs ? p.lhs[b] : b / p.lhs_div;
            // out-of-range indices leave the entry's rows unwritten (no access)
            if (e >= 0 && e < E && xi >= 0 && xi < p.x_batches) {
                k.e = e;
                k.xrow = xi * p.M + static_cast<long long>(part) * TM;
                k.orow = static_cast<long long>(b) * p.M + static_cast<long long>(part) * TM;
                k.rows = min(TM, p.M - part * TM);
            }
        }
        return k;
    };

    if (warp == CWARPS) {
        // ------------------------------ producer warp -------------------------------
        if (lane == 0) tma_prefetch_map(&tw);
        const int csz = qgd::sb_copy_bytes(p.G);
        const int cpr = 16 / csz;                 // copies per row of a stage's 8 groups
        const int gpc = csz / 2;                  // groups per copy
        const int ncp = 2 * BR * cpr;             // copies per stage (scales, biases)
        const char* sg = static_cast<const char*>(p.s);
        const char* bg = static_cast<const char*>(p.b);
        uint32_t it = 0;
        int slot = 0;
        uint32_t phase = 0;  // parity of the empty-barrier phase to wait for
        long long cprev = -1;
        Chunk ck{0, 0, 0, 0};
        bool abort = false;
        for (long long i = i_lo; i < i_hi && !abort; ++i) {
            const long long c = i / RB;
            const int rb = static_cast<int>(i % RB);
            if (c != cprev) {
                ck = chunk_of(c);
                cprev = c;
            }
            if (ck.rows <= 0) continue;
            const int wrow = ck.e * N + rb * BR;  // first weight row of the item
            for (int st = 0; st < S; ++st, ++it) {
                if (it >= static_cast<uint32_t>(stages)) {
                    int ok = 1;
                    if (lane == 0) {
                        ok = !*s_abort && mbar_wait_bounded(smem_u32(empty + slot), phase, kSpinLimit);
                        if (!ok) {
                            atomicCAS(p.err, 0, kErrTimeout);
                            *s_abort = 1;
                        }
                    }
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) {
                        abort = true;
                        break;
                    }
                }
                uint8_t* dst = ring + slot * STAGE;
                const uint32_t bar = smem_u32(full + slot);
                if (lane == 0) {
                    mbar_arrive_expect_tx(bar, W_BYTES);
#pragma unroll
                    for (int b = 0; b < GEO::BOXES; ++b)
                        tma_load_2d(smem_u32(dst) + b * (BR * 128), &tw, bar,
                                    (st * SG * WPG) + b * 32, wrow);
                }
                // scales and biases [BR rows][8 groups]: rows past N and groups past K
                // are filled with zeros
                for (int q = lane; q < ncp; q += 32) {
                    const int a = q / (BR * cpr), rem = q % (BR * cpr);
                    const int row = rem / cpr, ch = rem % cpr;
                    const int g = st * SG + ch * gpc;
                    const bool ok = rb * BR + row < N && g < p.G;
                    const char* src = (a ? bg : sg) +
                                      (ok ? ((static_cast<long long>(wrow) + row) * p.G + g) * 2 : 0);
                    uint8_t* d = dst + W_BYTES + a * SB_BYTES + row * 16 + ch * csz;
                    const int nb = ok ? csz : 0;
                    if (csz == 16) cp_async16(d, src, nb);
                    else if (csz == 8) cp_async8(d, src, nb);
                    else cp_async4(d, src, nb);
                }
                cp_async_mbar_arrive_noinc(bar);
                if (++slot == stages) {
                    slot = 0;
                    if (it >= static_cast<uint32_t>(stages)) phase ^= 1u;  // not after the first pass
                }
            }
        }
        // copies issued must land before the CTA can exit
        asm volatile("cp.async.wait_all;\n" ::: "memory");
        if (lane == 0 && *s_abort) {
            const uint32_t n = it < static_cast<uint32_t>(stages) ? it : stages;
            for (uint32_t j = it - n; j < it; ++j)
                mbar_wait_bounded(smem_u32(full + j % stages), (j / stages) & 1, kSpinLimit);
        }
        return;
    }

    // -------------------------------- consumers ------------------------------------
    const CONS cons(warp, lane, xf, rec);
    const T* xg = static_cast<const T*>(p.x);
    T* og = static_cast<T*>(p.out);
    const int ctid = tid;
    int slot = 0;
    uint32_t phase = 0;  // parity of the full-barrier phase to wait for
    long long staged = -1;
    Chunk ck{0, 0, 0, 0};
    for (long long i = i_lo; i < i_hi; ++i) {
        const long long c = i / RB;
        const int rb = static_cast<int>(i % RB);
        if (c != staged) {
            ck = chunk_of(c);
            staged = c;
            if (ck.rows <= 0) continue;
            // every consumer warp is past the previous item's stages (the combine's
            // barriers): its fragments can be overwritten
            const T* x0 = xg + ck.xrow * p.K;
            const int rows = ck.rows, G = p.G;
            qt_stage_activations<T, BITS, GS, TM>(
                xf, rec, Gp,
                [&](int t) -> const T* { return t < rows ? x0 + static_cast<long long>(t) * p.K : nullptr; },
                [&](int j) -> int { return j < G ? j : -1; }, ctid);
            named_bar_sync(1, CTHREADS);
        }
        if (ck.rows <= 0) continue;
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
        for (int st = 0; st < S; ++st) {
            if (!*s_abort) {
                const uint32_t fb = smem_u32(full + slot);
                if (!mbar_try_wait(fb, phase) && !wait_slow(fb, phase)) {
                    atomicCAS(p.err, 0, kErrTimeout);
                    *s_abort = 1;
                }
            }
            cons.stage(ring + slot * STAGE, cons.x_at(st), cons.rec_at(st), acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(empty + slot));
            if (++slot == stages) {
                slot = 0;
                phase ^= 1u;
            }
        }
        cons.combine(red, lane, acc);
        if (cons.kq == 0 && !*s_abort) {
            if constexpr (EPI == 1) {
                // this lane holds gate row r and up row r + 8 of its 16-row tile
                const int n = (rb * BR + 16 * cons.rt) / 2 + cons.r;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int t = 8 * nt + 2 * cons.c + q;
                        if (t < ck.rows && 2 * n < N)
                            og[(ck.orow + t) * (N / 2) + n] =
                                swiglu_out<T>(acc[nt][q], acc[nt][2 + q]);
                    }
            } else {
                const int row0 = rb * BR + 16 * cons.rt + cons.r;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const int n = row0 + 8 * hh;
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const int t = 8 * nt + 2 * cons.c + q;
                            if (t < ck.rows && n < N)
                                og[(ck.orow + t) * N + n] = ET::from_f(acc[nt][2 * hh + q]);
                        }
                    }
            }
        }
    }
}

}  // namespace mlxq
