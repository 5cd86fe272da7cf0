// Launch wrapper for one instantiation of the TMA-fed decode kernel; the
// qmv_tma_<dtype>.cu translation units instantiate them per activation type.
#pragma once

#include "qmv_tma.cuh"

namespace mlxq {

template <typename T, int BITS, int GS, int TM, int BR, bool HEADS, int EPI>
cudaError_t qt_launch_t(const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& tb,
                        const QtParams& p, int grid, size_t smem, bool overlap, cudaStream_t st) {
    auto kern = qmv_tma_kernel<T, BITS, GS, TM, BR, HEADS, EPI>;
    static PerDevice configured;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    e = ensure_smem_attr(kern, configured, dev, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(qt::threads(HEADS));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = overlap ? attr : nullptr;
    cfg.numAttrs = overlap ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, tw, ts, tb, p);
}

#define MLXQ_QT_INST0(T, BITS, GS, TM, BR, H, EPI)                                               \
    template cudaError_t qt_launch_t<T, BITS, GS, TM, BR, H, EPI>(                                \
        const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const QtParams&, int, size_t, \
        bool, cudaStream_t);
#define MLXQ_QT_INST1(T, BITS, GS, BR, H, EPI) \
    MLXQ_QT_INST0(T, BITS, GS, 1, BR, H, EPI)  \
    MLXQ_QT_INST0(T, BITS, GS, 2, BR, H, EPI)  \
    MLXQ_QT_INST0(T, BITS, GS, 4, BR, H, EPI)  \
    MLXQ_QT_INST0(T, BITS, GS, 8, BR, H, EPI)  \
    MLXQ_QT_INST0(T, BITS, GS, 16, BR, H, EPI)

// Every (bits, group size) the plan accepts, for activation type T, BR-row units,
// ticket warp or not, and plain or SwiGLU epilogue.
#define MLXQ_INSTANTIATE_QT(T, BR, H, EPI)  \
    MLXQ_QT_INST1(T, 4, 32, BR, H, EPI)     \
    MLXQ_QT_INST1(T, 4, 64, BR, H, EPI)     \
    MLXQ_QT_INST1(T, 4, 128, BR, H, EPI)    \
    MLXQ_QT_INST1(T, 8, 32, BR, H, EPI)     \
    MLXQ_QT_INST1(T, 8, 64, BR, H, EPI)

}  // namespace mlxq
