// Planning, tensor maps and dispatch for the TMA-fed decode kernel (qmv_tma.cuh).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "qmv_tma.cuh"

namespace mlxq {

__device__ int g_qmv_tma_error;

template <typename T, int BITS, int GS, int TM, int BR, bool HEADS, int EPI>
cudaError_t qt_launch_t(const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& tb,
                        const QtParams& p, int grid, size_t smem, bool overlap, cudaStream_t st);

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D map over a row-major [rows, cols] array of `esize`-byte elements, box
// [box_rows, box_cols].
bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize,
              unsigned long long cols, unsigned long long rows, unsigned box_cols,
              unsigned box_rows, CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
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

bool qt_make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize,
                 unsigned long long cols, unsigned long long rows, unsigned box_cols,
                 unsigned box_rows, CUtensorMapSwizzle swz) {
    return make_map(m, base, dt, esize, cols, rows, box_cols, box_rows, swz);
}
bool qt_maps_available() { return encode_fn() != nullptr; }

// CTAs of this kernel meant to fit on one SM together: with 2, the shared memory
// of a CTA is capped at half the SM's, so under launch overlap the next matmul's
// CTAs can start streaming their weights while this one finishes.
constexpr int kCtasPerSm = 2;
// CTAs launched per SM (stream-K shares = kGridPerSm x SMs).
constexpr int kGridPerSm = 1;
// 64-row blocks of at most this many units go whole to one CTA when they fit on the SMs.
constexpr int kWholeRowBlockStages = 8;
// Shares of at most this many units hand their head row block's ticket to a ticket
// warp: the consumers' wait for the atomic is then a large part of a short share.
constexpr int kHeadTicketUnits = 32;

// Unit rows forced by the MLXQ_DECODE_ROWS environment variable (16 or 64; read
// once), else 0: the plan chooses.
static int rows_override() {
    static int v = [] {
        const char* e = std::getenv("MLXQ_DECODE_ROWS");
        const int r = e ? std::atoi(e) : 0;
        return (r == 16 || r == 64) ? r : 0;
    }();
    return v;
}

bool qmv_tma_plan(int dtype, int bits, int gs, int M, int N, int K, int num_sms, int max_smem,
                  int sm_smem, QtPlan* plan) {
    if (M < 1 || M > qt::MAXM || N < 1 || K < 1 || K % gs) return false;
    if (bits != 4 && bits != 8) return false;
    if (gs != 32 && gs != 64 && gs != 128) return false;
    if (bits == 8 && gs == 128) return false;  // 64 KB stages: too shallow a ring
    const int G = K / gs;
    if (G % qt::SG) return false;  // scale/bias rows must be whole 16-byte TMA boxes
    if (!encode_fn()) return false;
    // the driver reserves 1 KB of shared memory per CTA
    const int full_smem = max_smem;
    const int half_smem = std::min(max_smem, sm_smem / kCtasPerSm - 1024);
    const int TM = qt::token_slots(M);
    // Unit rows: a matrix with short rows (at most kWholeRowBlockStages stages) whose
    // 16-row blocks all fit on the SMs at kCtasPerSm CTAs per SM takes one CTA per
    // 16-row block: no split row block, hence no ticket reduction, and a short chain
    // of stages per CTA. Everything else streams 64-row units.
    int br = rows_override();
    if (!br)
        br = ((N + 15) / 16 <= kCtasPerSm * num_sms && G / qt::SG <= kWholeRowBlockStages)
                 ? 16 : 64;
    // 16 token slots stage twice the activations of 8: a 16-row plan (one CTA per row
    // block) then fits one CTA per SM, so it is taken only when its row blocks fit on
    // the SMs at that (else the cp.async kernel is faster for these shapes).
    if (TM > 8 && br == 16 && (N + 15) / 16 > num_sms) return false;
    const int rt = br / 16;
    const int stage = qt::stage_stride(bits, gs, br);
    QtPlan pl{};
    pl.BR = br;
    pl.RB = (N + br - 1) / br;
    if (static_cast<size_t>(pl.RB) * 4 > kArgmaxOffset) return false;
    pl.S = G / qt::SG;
    pl.U = static_cast<long long>(pl.RB) * pl.S;
    pl.P = static_cast<int>(std::min<long long>(pl.U, static_cast<long long>(num_sms) * kGridPerSm));
    // Row blocks that fit on the SMs are not split at all: one CTA per row block needs
    // no ticket reduction, which costs more than the extra units per CTA. (64-row
    // blocks only when short: one CTA per SM, the chain of stages grows with K.)
    if (br < 64 ? pl.RB <= kCtasPerSm * num_sms
                : (pl.RB <= num_sms && pl.S <= kWholeRowBlockStages))
        pl.P = pl.RB;
    const long long per_cta = (pl.U + pl.P - 1) / pl.P;
    // activation fragments are staged for the K groups of a CTA's own units only
    pl.GL = static_cast<int>(std::min<long long>(G, per_cta * qt::SG));
    const int fixed = qt::layout(stage, 0, pl.GL, TM, gs * 2, rt).total + 1024;  // + alignment
    // Half an SM's shared memory lets the next matmul's CTAs co-reside where their warps
    // fit; a plan whose staged activations leave that too shallow a ring (many tokens,
    // long shares) takes the whole SM instead.
    int cap = half_smem;
    const int want = static_cast<int>(std::min<long long>(4, std::max<long long>(2, per_cta)));
    if ((cap - fixed) / stage < want) cap = full_smem;
    if (fixed + 2 * stage > cap) return false;
    int stages = std::min((cap - fixed) / stage, qt::MAX_STAGES);
    stages = static_cast<int>(std::min<long long>(stages, std::max<long long>(2, per_cta)));
    pl.stages = std::max(2, stages);
    pl.smem = static_cast<size_t>(qt::layout(stage, pl.stages, pl.GL, TM, gs * 2, rt).total) +
              1024;
    int maxc = 1;
    for (int rb = 0; rb < pl.RB; ++rb) {
        const long long ub = static_cast<long long>(rb) * pl.S;
        const int nc = qt::owner(ub + pl.S - 1, pl.U, pl.P) - qt::owner(ub, pl.U, pl.P) + 1;
        maxc = std::max(maxc, nc);
    }
    pl.maxc = maxc;
    pl.heads = false;
    if (br == 64 && maxc > 1 && per_cta <= kHeadTicketUnits) {
        for (int b = 0; b < pl.P && !pl.heads; ++b) {
            const long long lo = pl.U * b / pl.P, hi = pl.U * (b + 1) / pl.P;
            pl.heads = (lo % pl.S) != 0 && hi > (lo / pl.S + 1) * pl.S;
        }
    }
    pl.ws_bytes = 0;
    if (maxc > 1)
        pl.ws_bytes = kTicketBytes +
                      static_cast<size_t>(pl.RB) * maxc * M * br * 4;
    *plan = pl;
    return true;
}

#define QT_CASE_TM(T, BITS, GS, BR, H, EPI)                                                      \
    switch (qt::token_slots(M)) {                                                                \
        case 1: return qt_launch_t<T, BITS, GS, 1, BR, H, EPI>(tw, ts, tb, p, plan.P, plan.smem, overlap, st); \
        case 2: return qt_launch_t<T, BITS, GS, 2, BR, H, EPI>(tw, ts, tb, p, plan.P, plan.smem, overlap, st); \
        case 4: return qt_launch_t<T, BITS, GS, 4, BR, H, EPI>(tw, ts, tb, p, plan.P, plan.smem, overlap, st); \
        case 8: return qt_launch_t<T, BITS, GS, 8, BR, H, EPI>(tw, ts, tb, p, plan.P, plan.smem, overlap, st); \
        default: return qt_launch_t<T, BITS, GS, 16, BR, H, EPI>(tw, ts, tb, p, plan.P, plan.smem, overlap, st); \
    }
#define QT_CASE_SW(T, BITS, GS, EPI)                                           \
    if (plan.BR == 16) { QT_CASE_TM(T, BITS, GS, 16, false, EPI) }             \
    if (plan.heads) { QT_CASE_TM(T, BITS, GS, 64, true, EPI) }                 \
    QT_CASE_TM(T, BITS, GS, 64, false, EPI)
#define QT_CASE(T, BITS, GS)                                                  \
    if (epi == 1) { QT_CASE_SW(T, BITS, GS, 1) }                              \
    if (epi == 2) { QT_CASE_SW(T, BITS, GS, 2) }                              \
    QT_CASE_SW(T, BITS, GS, 0)

template <typename T>
static cudaError_t qt_dispatch(int bits, int gs, int M, int epi, const CUtensorMap& tw,
                               const CUtensorMap& ts, const CUtensorMap& tb, const QtParams& p,
                               const QtPlan& plan, bool overlap, cudaStream_t st) {
    if (bits == 4) {
        if (gs == 32) { QT_CASE(T, 4, 32) }
        if (gs == 64) { QT_CASE(T, 4, 64) }
        if (gs == 128) { QT_CASE(T, 4, 128) }
    } else if (bits == 8) {
        if (gs == 32) { QT_CASE(T, 8, 32) }
        if (gs == 64) { QT_CASE(T, 8, 64) }
    }
    return cudaErrorInvalidValue;
}

// Device address of g_qmv_tma_error, looked up once per device (kernels in other
// translation units reach the flag through this pointer).
int* qmv_tma_error_flag() {
    static std::atomic<int*> addr[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    int* a = addr[dev].load(std::memory_order_acquire);
    if (!a) {
        void* sym = nullptr;
        if (cudaGetSymbolAddress(&sym, g_qmv_tma_error) != cudaSuccess) return nullptr;
        a = static_cast<int*>(sym);
        addr[dev].store(a, std::memory_order_release);  // the same value from every thread
    }
    return a;
}

cudaError_t qmv_tma_launch(int dtype, int bits, int gs, const QtPlan& plan, const void* x,
                           const uint32_t* w, const void* s, const void* b, const void* bias,
                           void* out, int M, int N, int K, void* workspace, bool overlap,
                           cudaStream_t st, int epi) {
    const int G = K / gs;
    const unsigned long long kw = static_cast<unsigned long long>(K) * bits / 32;
    CUtensorMap tw, ts, tb;
    const unsigned br = static_cast<unsigned>(plan.BR);
    if (!make_map(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, kw, N, 32, br,
                  CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&ts, s, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, G, N, qt::SG, br,
                  CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map(&tb, b, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, G, N, qt::SG, br,
                  CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    QtParams p{};
    p.err = qmv_tma_error_flag();
    if (!p.err) return cudaErrorInvalidSymbol;
    p.x = x; p.bias = bias; p.out = out;
    p.M = M; p.N = N; p.K = K; p.G = G; p.GL = plan.GL;
    p.S = plan.S; p.RB = plan.RB; p.U = plan.U; p.stages = plan.stages; p.maxc = plan.maxc;
    if (plan.ws_bytes) {
        p.counter = static_cast<unsigned*>(workspace);
        p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kTicketBytes);
    }
    if (epi == 1 && (N % 16 || bias)) return cudaErrorInvalidValue;
    if (epi == 2) {
        // greedy argmax: per-token keys and a done counter at the end of the ticket region
        if (!workspace) return cudaErrorInvalidValue;
        p.am_done = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + kArgmaxOffset);
        p.am_keys = reinterpret_cast<unsigned long long*>(static_cast<char*>(workspace) +
                                                          kArgmaxOffset + 64);
    }
    if (dtype == kBF16)
        return qt_dispatch<__nv_bfloat16>(bits, gs, M, epi, tw, ts, tb, p, plan, overlap, st);
    if (dtype == kF16)
        return qt_dispatch<__half>(bits, gs, M, epi, tw, ts, tb, p, plan, overlap, st);
    return cudaErrorInvalidValue;
}

// One bounded mbarrier wait that nothing completes: thread 0 initialises a barrier
// that expects one arrival, never arrives, and polls it `polls` times with the same
// bounded wait the decode kernels use; when the wait gives up it records
// kErrTimeout in the error word, exactly as a kernel whose copies never landed
// would. No copy or tensor-core operation is in flight, so nothing is left pending.
__global__ void bounded_wait_check_kernel(int* err, uint32_t polls) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    const uint32_t b = smem_u32(&bar);
    mbar_init(b, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    if (!mbar_wait_bounded(b, 0, polls)) atomicCAS(err, 0, qt::kErrTimeout);
}

cudaError_t launch_bounded_wait_check(uint32_t polls, cudaStream_t st) {
    int* err = qmv_tma_error_flag();
    if (!err) return cudaErrorInvalidSymbol;
    bounded_wait_check_kernel<<<1, 32, 0, st>>>(err, polls);
    return cudaGetLastError();
}

cudaError_t qmv_tma_read_error(int* code) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_qmv_tma_error, sizeof(int));
    if (e != cudaSuccess) return e;
    if (v) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_qmv_tma_error, &zero, sizeof(int));
    }
    *code = v;
    return e;
}

}  // namespace mlxq
