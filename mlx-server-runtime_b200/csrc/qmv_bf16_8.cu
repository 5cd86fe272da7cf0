// Instantiations of the skinny kernel for __nv_bfloat16 activations, 8-bit codes.
#include "qmv_inst.cuh"

namespace mlxq {
MLXQ_INSTANTIATE_QMV(__nv_bfloat16, 8)
}  // namespace mlxq
