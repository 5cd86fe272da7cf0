// Instantiations of the skinny kernel for __half activations, 8-bit codes.
#include "qmv_inst.cuh"

namespace mlxq {
MLXQ_INSTANTIATE_QMV(__half, 8)
}  // namespace mlxq
