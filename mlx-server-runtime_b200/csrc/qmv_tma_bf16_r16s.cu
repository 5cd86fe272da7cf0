#include "qmv_tma_inst.cuh"
namespace mlxq {
// SwiGLU epilogue
MLXQ_INSTANTIATE_QT(__nv_bfloat16, 16, false, 1)
}
