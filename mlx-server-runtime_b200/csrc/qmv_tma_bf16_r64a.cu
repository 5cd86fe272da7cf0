#include "qmv_tma_inst.cuh"
namespace mlxq {
// greedy argmax epilogue
MLXQ_INSTANTIATE_QT(__nv_bfloat16, 64, false, 2)
MLXQ_INSTANTIATE_QT(__nv_bfloat16, 64, true, 2)
}
