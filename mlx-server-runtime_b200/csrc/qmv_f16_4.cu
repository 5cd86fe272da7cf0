// Instantiations of the skinny kernel for __half activations, 4-bit codes.
#include "qmv_inst.cuh"

namespace mlxq {
MLXQ_INSTANTIATE_QMV(__half, 4)
}  // namespace mlxq
