// Kernel instantiations of k_boa_step for the 3xTF32 split operand kind (one translation
// unit per kind, so the kinds compile in parallel).
#include "model_kernel.cuh"

namespace boa {
BOA_DEFINE_LAUNCH(64, 3)
BOA_DEFINE_LAUNCH(256, 3)
}  // namespace boa
