// Kernel instantiations of k_boa_step for the tf32 operand kind (one translation
// unit per kind, so the kinds compile in parallel).
#include "model_kernel.cuh"

namespace boa {
BOA_DEFINE_LAUNCH(64, 0)
BOA_DEFINE_LAUNCH(256, 0)
}  // namespace boa
