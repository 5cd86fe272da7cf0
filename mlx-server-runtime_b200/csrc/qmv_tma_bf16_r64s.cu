#include "qmv_tma_inst.cuh"
namespace mlxq {
// SwiGLU epilogue
MLXQ_INSTANTIATE_QT(__nv_bfloat16, 64, false, 1)
MLXQ_INSTANTIATE_QT(__nv_bfloat16, 64, true, 1)
}
