// Planning and dispatch for the skinny kernel family, and the expert segment
// table used by sorted gather_qmm.
#include <algorithm>

#include "qmv_inst.cuh"

namespace mlxq {

template <typename T, int BITS, int GS, int NT, bool SBV, bool ODD>
cudaError_t qmv_launch_t(const QmvPlan& plan, const QmvParams& p, cudaStream_t st);

static int nt_for(long long tokens) { return tokens <= 8 ? 1 : tokens <= 16 ? 2 : 4; }

bool qmv_plan(int dtype, int bits, int gs, int M, int N, int K, int mode, int z_items,
              int num_sms, int max_smem, QmvPlan* plan) {
    const int G = K / gs;
    const int cg = 32 / (gs * bits / 32);
    QmvPlan pl{};
    if (mode == 0) {
        pl.nt = nt_for(M);
    } else if (mode == 1) {
        pl.nt = nt_for(M);
    } else {
        // z_items = batch*M / E: the average rows per expert decides the n-tile count
        pl.nt = nt_for(z_items < 1 ? 1 : z_items);
    }
    pl.sbvec = (cg >= 2) && (G % cg == 0);
    // every pass holds exactly one token: dense or per-entry gather with M == 1
    pl.single = (mode != 2) && M == 1;
    pl.rowblocks = (N + kRowTiles * 16 - 1) / (kRowTiles * 16);
    const QmvGeom geo = qmv_geom(bits, gs, pl.nt, pl.sbvec, dtype == kF16 && bits == 4);
    const size_t sb = static_cast<size_t>(geo.stage_bytes) + geo.red_bytes;
    const size_t per_group = geo.per_group;
    if (static_cast<size_t>(max_smem) <= sb + per_group * cg) return false;
    int win_max = static_cast<int>((max_smem - sb) / per_group);
    win_max = (win_max / cg) * cg;
    if (win_max < cg) return false;

    if (mode == 0) {
        const int tok = pl.nt * 8;
        pl.ztotal = (M + tok - 1) / tok;
        const long long items = static_cast<long long>(pl.rowblocks) * pl.ztotal;
        int S = 1;
        if (items < num_sms) S = static_cast<int>(num_sms / items);
        const int max_splits = (G + cg - 1) / cg;
        S = std::max(1, std::min(S, max_splits));
        int gps = ((G + S - 1) / S + cg - 1) / cg * cg;
        S = (G + gps - 1) / gps;
        pl.splits = S;
        pl.gps = gps;
    } else {
        pl.ztotal = mode == 1 ? z_items : 0;  // caller fills ztotal for mode 2
        pl.splits = 1;
        pl.gps = ((G + cg - 1) / cg) * cg;
    }
    pl.win = std::min(pl.gps, win_max);
    pl.smem = sb + per_group * pl.win;
    pl.gridz = std::min(std::max(pl.ztotal, 1), 65535);
    pl.ws_bytes = 0;
    if (pl.splits > 1) {
        const size_t counters = static_cast<size_t>(pl.ztotal) * pl.rowblocks * 4;
        if (counters > kArgmaxOffset) return false;
        pl.ws_bytes = kTicketBytes +
                      static_cast<size_t>(pl.splits) * M * static_cast<size_t>(N) * 4;
    }
    *plan = pl;
    return true;
}

#define QMV_CASE_NT(T, BITS, GS, SBV)                                                    \
    switch (plan.nt) {                                                                   \
        case 1:                                                                          \
            if (plan.single) return qmv_launch_t<T, BITS, GS, 1, SBV, false>(plan, p, st); \
            return qmv_launch_t<T, BITS, GS, 1, SBV, true>(plan, p, st);                 \
        case 2: return qmv_launch_t<T, BITS, GS, 2, SBV, true>(plan, p, st);             \
        default: return qmv_launch_t<T, BITS, GS, 4, SBV, true>(plan, p, st);            \
    }

#define QMV_CASE_GS(T, BITS)                                                             \
    switch (gs) {                                                                        \
        case 32:                                                                         \
            if (plan.sbvec) { QMV_CASE_NT(T, BITS, 32, true) } else { QMV_CASE_NT(T, BITS, 32, false) } \
        case 64:                                                                         \
            if (plan.sbvec) { QMV_CASE_NT(T, BITS, 64, true) } else { QMV_CASE_NT(T, BITS, 64, false) } \
        case 128:                                                                        \
            if (plan.sbvec) { QMV_CASE_NT(T, BITS, 128, true) } else { QMV_CASE_NT(T, BITS, 128, false) } \
        default: return cudaErrorInvalidValue;                                           \
    }

template <typename T>
static cudaError_t qmv_launch_dtype(int bits, int gs, const QmvPlan& plan, const QmvParams& p,
                                    cudaStream_t st) {
    if (bits == 4) { QMV_CASE_GS(T, 4) }
    if (bits == 8) { QMV_CASE_GS(T, 8) }
    return cudaErrorInvalidValue;
}

cudaError_t qmv_launch(int dtype, int bits, int gs, const QmvPlan& plan, const QmvParams& p,
                       cudaStream_t st) {
    if (dtype == kBF16) return qmv_launch_dtype<__nv_bfloat16>(bits, gs, plan, p, st);
    if (dtype == kF16) return qmv_launch_dtype<__half>(bits, gs, plan, p, st);
    return cudaErrorInvalidValue;
}

// seg[e] = first batch index whose (sorted) expert is >= e, seg[E] = batch.
// Thread i looks at the boundary between entries i-1 and i and writes the
// offsets of every expert id in (rhs[i-1], rhs[i]]; ids are clamped to
// [-1, E] so out-of-range entries cannot write outside seg.
__global__ void segments_kernel(const int32_t* __restrict__ rhs, int batch, int E,
                                int32_t* __restrict__ seg) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i > batch) return;
    int prev = (i == 0) ? -1 : rhs[i - 1];
    int cur = (i == batch) ? E : rhs[i];
    prev = max(-1, min(prev, E));
    cur = max(-1, min(cur, E));
    for (int e = prev + 1; e <= cur; ++e) seg[e] = i;
}

cudaError_t launch_segments(const int32_t* rhs, int batch, int num_experts, int32_t* seg,
                            cudaStream_t st) {
    const int threads = 256;
    const int blocks = (batch + 1 + threads - 1) / threads;
    segments_kernel<<<blocks, threads, 0, st>>>(rhs, batch, num_experts, seg);
    return cudaGetLastError();
}

}  // namespace mlxq
