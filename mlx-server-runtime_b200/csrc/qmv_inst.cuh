// Launch wrapper for one instantiation of the skinny kernel. Each
// qmv_<dtype>_<bits>.cu translation unit instantiates the wrappers for its
// (dtype, bits) pair so the kernel family compiles in parallel.
#pragma once

#include "qmv.cuh"

namespace mlxq {

template <typename T, int BITS, int GS, int NT, bool SBV, bool ODD>
cudaError_t qmv_launch_t(const QmvPlan& plan, const QmvParams& p, cudaStream_t st) {
    auto kern = qmv_kernel<T, BITS, GS, NT, SBV, ODD>;
    constexpr QmvGeom geo = qmv_geom(BITS, GS, NT, SBV, qmv_two_sums<T, BITS>());
    static PerDevice configured;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    e = ensure_smem_attr(kern, configured, dev, static_cast<int>(plan.smem));
    if (e != cudaSuccess) return e;
    dim3 grid(plan.rowblocks, plan.splits, plan.gridz);
    if (!plan.overlap) {
        kern<<<grid, geo.nwarp * 32, plan.smem, st>>>(p);
        return cudaGetLastError();
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(geo.nwarp * 32);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

#define MLXQ_INSTANTIATE_QMV(T, BITS)  \
    template cudaError_t qmv_launch_t<T, BITS, 32, 1, true, false>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 32, 1, true, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 32, 2, true, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 32, 4, true, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 32, 1, false, false>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 32, 1, false, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 32, 2, false, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 32, 4, false, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 64, 1, true, false>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 64, 1, true, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 64, 2, true, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 64, 4, true, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 64, 1, false, false>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 64, 1, false, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 64, 2, false, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 64, 4, false, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 128, 1, true, false>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 128, 1, true, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 128, 2, true, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 128, 4, true, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 128, 1, false, false>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 128, 1, false, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 128, 2, false, true>(const QmvPlan&, const QmvParams&, cudaStream_t);  \
    template cudaError_t qmv_launch_t<T, BITS, 128, 4, false, true>(const QmvPlan&, const QmvParams&, cudaStream_t);

}  // namespace mlxq
