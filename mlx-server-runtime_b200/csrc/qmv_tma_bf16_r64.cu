#include "qmv_tma_inst.cuh"
namespace mlxq {
MLXQ_INSTANTIATE_QT(__nv_bfloat16, 64, false, 0)
}
