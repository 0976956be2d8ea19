// Model entry points (placeholder until the fused step kernel lands).
#include "boa_b200.h"
#include "capi_util.h"

extern "C" {
BOA_API int boa_model_create(boa_model** out, int, int, int, const float*, size_t, int, int) {
  if (out) *out = nullptr;
  return boa_fail(BOA_ERR_UNSUPPORTED, "boa_model_create: not built yet");
}
BOA_API int boa_model_destroy(boa_model*) { return BOA_OK; }
BOA_API size_t boa_model_workspace_bytes(const boa_model*, int) { return 0; }
BOA_API int boa_model_step(boa_model*, int, const int32_t*, float*, void*, size_t, void*) {
  return boa_fail(BOA_ERR_UNSUPPORTED, "boa_model_step: not built yet");
}
BOA_API int boa_model_logits(boa_model*, int, int, const int32_t*, float*, void*, size_t, void*) {
  return boa_fail(BOA_ERR_UNSUPPORTED, "boa_model_logits: not built yet");
}
BOA_API int boa_codec_encode(boa_model*, int, const uint8_t*, int64_t, const int32_t*, uint32_t*, int, int32_t*,
                             int, void*, size_t, void*) {
  return boa_fail(BOA_ERR_UNSUPPORTED, "boa_codec_encode: not built yet");
}
BOA_API int boa_codec_decode(boa_model*, int, const uint32_t*, int, const int32_t*, const int32_t*, const uint8_t*,
                             uint8_t*, int64_t, int, void*, size_t, void*) {
  return boa_fail(BOA_ERR_UNSUPPORTED, "boa_codec_decode: not built yet");
}
}
