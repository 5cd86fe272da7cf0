// Planning and dispatch for the TMA-fed grouped decode kernel (qmv_grouped.cuh).
#include <algorithm>

#include "qmv_grouped.cuh"

namespace mlxq {

template <typename T, int BITS, int GS, int TM, int BR, int EPI>
cudaError_t qgd_launch_t(const CUtensorMap& tw, const QgdParams& p, int grid, size_t smem,
                         bool overlap, cudaStream_t st);

// CTAs meant to share an SM: each streams its own items, so two per SM keep more
// TMA copies in flight while the other stages activations.
constexpr int kQgdCtasPerSm = 2;
constexpr int kQgdRows = 64;  // weight rows per item

bool qmv_grouped_plan(int bits, int gs, long long batch, int M, int N, int K, int E, bool sorted,
                      int num_sms, int max_smem, int sm_smem, QgdPlan* plan) {
    if (batch < 1 || M < 1 || N < 1 || K < 1 || E < 1 || num_sms < 1) return false;
    if (bits != 4 && bits != 8) return false;
    if (gs != 32 && gs != 64 && gs != 128) return false;
    if (bits == 8 && gs == 128) return false;
    if (K % gs) return false;
    const int G = K / gs;
    if (G % 2) return false;  // scale rows of 2G bytes: cp.async needs 4-byte pieces
    if (sorted && E > qgd::MAXE) return false;
    if (static_cast<long long>(E) * N > (1LL << 31) - 1) return false;  // TMA row coordinate
    if (!qt_maps_available()) return false;
    QgdPlan pl{};
    pl.sorted = sorted;
    // Token slots: unsorted entries are their own chunks (M rows); sorted, about
    // twice the mean rows per expert, so most experts take one chunk.
    const long long rows = batch * M;
    const int want = sorted ? static_cast<int>(2 * ((rows + E - 1) / E)) : M;
    pl.TM = want <= 1 ? 1 : want <= 4 ? 4 : 8;
    pl.BR = kQgdRows;
    pl.S = (G + qt::SG - 1) / qt::SG;
    pl.RB = (N + pl.BR - 1) / pl.BR;
    const long long chunks =
        sorted ? (rows + pl.TM - 1) / pl.TM + std::min<long long>(E, batch)
               : batch * ((M + pl.TM - 1) / pl.TM);
    const long long items = chunks * pl.RB;
    const int stage = qt::stage_stride(bits, gs, pl.BR);
    const int fixed = qgd::layout(stage, 0, pl.S * qt::SG, pl.TM, gs * 2, pl.BR / 16, E, sorted)
                          .total + 1024;  // + alignment
    int cap = std::min(max_smem, sm_smem / kQgdCtasPerSm - 1024);
    int per_sm = kQgdCtasPerSm;
    if (fixed + 2 * stage > cap) {
        cap = max_smem;
        per_sm = 1;
    }
    if (fixed + 2 * stage > cap) return false;
    pl.P = static_cast<int>(std::max<long long>(1, std::min<long long>(items, static_cast<long long>(num_sms) * per_sm)));
    const long long per_cta = (items + pl.P - 1) / pl.P * pl.S;  // stages per CTA (bound)
    int stages = std::min((cap - fixed) / stage, qt::MAX_STAGES);
    stages = static_cast<int>(std::min<long long>(stages, std::max<long long>(2, per_cta)));
    pl.stages = std::max(2, stages);
    pl.smem = static_cast<size_t>(qgd::layout(stage, pl.stages, pl.S * qt::SG, pl.TM, gs * 2,
                                              pl.BR / 16, E, sorted).total) + 1024;
    *plan = pl;
    return true;
}

#define QGD_CASE_TM(T, BITS, GS, EPI)                                                        \
    switch (plan.TM) {                                                                       \
        case 1: return qgd_launch_t<T, BITS, GS, 1, 64, EPI>(tw, p, plan.P, plan.smem, overlap, st); \
        case 4: return qgd_launch_t<T, BITS, GS, 4, 64, EPI>(tw, p, plan.P, plan.smem, overlap, st); \
        default: return qgd_launch_t<T, BITS, GS, 8, 64, EPI>(tw, p, plan.P, plan.smem, overlap, st); \
    }
#define QGD_CASE(T, BITS, GS)                     \
    if (epi == 1) { QGD_CASE_TM(T, BITS, GS, 1) } \
    QGD_CASE_TM(T, BITS, GS, 0)

template <typename T>
static cudaError_t qgd_dispatch(int bits, int gs, int epi, const CUtensorMap& tw,
                                const QgdParams& p, const QgdPlan& plan, bool overlap,
                                cudaStream_t st) {
    if (bits == 4) {
        if (gs == 32) { QGD_CASE(T, 4, 32) }
        if (gs == 64) { QGD_CASE(T, 4, 64) }
        if (gs == 128) { QGD_CASE(T, 4, 128) }
    } else if (bits == 8) {
        if (gs == 32) { QGD_CASE(T, 8, 32) }
        if (gs == 64) { QGD_CASE(T, 8, 64) }
    }
    return cudaErrorInvalidValue;
}

cudaError_t qmv_grouped_launch(int dtype, int bits, int gs, const QgdPlan& plan, const void* x,
                               const uint32_t* w, const void* s, const void* b, void* out,
                               const int32_t* rhs, const int32_t* lhs, int lhs_div, int batch,
                               int x_batches, int M, int N, int K, int E, bool overlap,
                               cudaStream_t st, int epi) {
    if (epi == 1 && N % 16) return cudaErrorInvalidValue;
    const unsigned long long kw = static_cast<unsigned long long>(K) * bits / 32;
    CUtensorMap tw;
    if (plan.BR != kQgdRows ||
        !qt_make_map(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, kw,
                     static_cast<unsigned long long>(E) * N, 32, plan.BR,
                     CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    QgdParams p{};
    p.err = qmv_tma_error_flag();
    if (!p.err) return cudaErrorInvalidSymbol;
    p.x = x; p.s = s; p.b = b; p.out = out;
    p.rhs = rhs; p.lhs = lhs; p.lhs_div = lhs_div < 1 ? 1 : lhs_div;
    p.batch = batch; p.x_batches = x_batches; p.M = M;
    p.N = N; p.K = K; p.G = K / gs; p.E = E;
    p.S = plan.S; p.RB = plan.RB; p.stages = plan.stages; p.sorted = plan.sorted ? 1 : 0;
    if (dtype == kBF16)
        return qgd_dispatch<__nv_bfloat16>(bits, gs, epi, tw, p, plan, overlap, st);
    if (dtype == kF16) return qgd_dispatch<__half>(bits, gs, epi, tw, p, plan, overlap, st);
    return cudaErrorInvalidValue;
}

}  // namespace mlxq
