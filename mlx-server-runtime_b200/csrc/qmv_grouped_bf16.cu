#include "qmv_grouped_inst.cuh"
namespace mlxq {
MLXQ_INSTANTIATE_QGD(__nv_bfloat16, 0)
}
