#include "qmv_tma_inst.cuh"
namespace mlxq {
MLXQ_INSTANTIATE_QT(__half, 64, true, 0)
}
