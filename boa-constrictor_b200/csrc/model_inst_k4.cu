// Kernel instantiations of k_boa_step for the 2xFP16 scaled-residual operand
// kind (one translation unit per kind, so the kinds compile in parallel).
#include "model_kernel.cuh"

namespace boa {
BOA_DEFINE_LAUNCH(64, 4)
BOA_DEFINE_LAUNCH(256, 4)
}  // namespace boa
