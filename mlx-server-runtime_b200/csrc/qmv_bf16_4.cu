// Instantiations of the skinny kernel for __nv_bfloat16 activations, 4-bit codes.
#include "qmv_inst.cuh"

namespace mlxq {
MLXQ_INSTANTIATE_QMV(__nv_bfloat16, 4)
}  // namespace mlxq
