#include "qmv_tma_inst.cuh"
namespace mlxq {
// greedy argmax epilogue
MLXQ_INSTANTIATE_QT(__half, 16, false, 2)
}
