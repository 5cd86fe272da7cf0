#include "qmv_tma_inst.cuh"
namespace mlxq {
MLXQ_INSTANTIATE_QT(__half, 16, false, 0)
}
