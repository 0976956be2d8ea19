// Kernel instantiations of k_boa_step for the bf16 operand kind (one translation
// unit per kind, so the kinds compile in parallel).
#include "model_kernel.cuh"

namespace boa {
BOA_DEFINE_LAUNCH(64, 1)
BOA_DEFINE_LAUNCH(256, 1)
BOA_DEFINE_LAUNCH(512, 1)
}  // namespace boa
