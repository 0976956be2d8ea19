// Thread-local last-error string for the C-ABI (boa_last_error).
#include "boa_b200.h"
#include "capi_util.h"

static thread_local std::string g_last_error;

int boa_fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

extern "C" BOA_API const char* boa_last_error(void) { return g_last_error.c_str(); }

extern "C" BOA_API int boa_abi_version(void) { return BOA_ABI_VERSION; }
