#include "qmv_tma_inst.cuh"
namespace mlxq {
// SwiGLU epilogue
MLXQ_INSTANTIATE_QT(__half, 64, false, 1)
MLXQ_INSTANTIATE_QT(__half, 64, true, 1)
}
