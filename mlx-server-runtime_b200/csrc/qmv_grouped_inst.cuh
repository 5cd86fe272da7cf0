// Launch wrapper for one instantiation of the TMA-fed grouped decode kernel; the
// qmv_grouped_<dtype>.cu translation units instantiate them per activation type.
#pragma once

#include "qmv_grouped.cuh"

namespace mlxq {

template <typename T, int BITS, int GS, int TM, int BR, int EPI>
cudaError_t qgd_launch_t(const CUtensorMap& tw, const QgdParams& p, int grid, size_t smem,
                         bool overlap, cudaStream_t st) {
    auto kern = qmv_grouped_kernel<T, BITS, GS, TM, BR, EPI>;
    static PerDevice configured;
    int dev = 0;
    cudaError_t e = current_device(&dev);
    if (e != cudaSuccess) return e;
    e = ensure_smem_attr(kern, configured, dev, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(qgd::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = overlap ? attr : nullptr;
    cfg.numAttrs = overlap ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, tw, p);
}

#define MLXQ_QGD_INST0(T, BITS, GS, TM, BR, EPI)                                              \
    template cudaError_t qgd_launch_t<T, BITS, GS, TM, BR, EPI>(                              \
        const CUtensorMap&, const QgdParams&, int, size_t, bool, cudaStream_t);
#define MLXQ_QGD_INST1(T, BITS, GS, EPI)      \
    MLXQ_QGD_INST0(T, BITS, GS, 1, 64, EPI)   \
    MLXQ_QGD_INST0(T, BITS, GS, 4, 64, EPI)   \
    MLXQ_QGD_INST0(T, BITS, GS, 8, 64, EPI)

// Every (bits, group size) the plan accepts, for activation type T and epilogue EPI.
#define MLXQ_INSTANTIATE_QGD(T, EPI)   \
    MLXQ_QGD_INST1(T, 4, 32, EPI)      \
    MLXQ_QGD_INST1(T, 4, 64, EPI)      \
    MLXQ_QGD_INST1(T, 4, 128, EPI)     \
    MLXQ_QGD_INST1(T, 8, 32, EPI)      \
    MLXQ_QGD_INST1(T, 8, 64, EPI)

}  // namespace mlxq
