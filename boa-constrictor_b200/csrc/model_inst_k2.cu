// Kernel instantiations of k_boa_step for the fp16 operand kind (one translation
// unit per kind, so the kinds compile in parallel).
#include "model_kernel.cuh"

namespace boa {
BOA_DEFINE_LAUNCH(64, 2)
BOA_DEFINE_LAUNCH(256, 2)
BOA_DEFINE_LAUNCH(512, 2)
}  // namespace boa
