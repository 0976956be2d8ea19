// Error plumbing shared by the C-ABI translation units: a thread-local last
// error string plus helpers that turn CUDA errors into BOA_ERR_CUDA returns.
#pragma once
#include <cuda_runtime.h>
#include <string>

int boa_fail(int code, const std::string& msg);

#define BOA_CUDA(expr)                                                          \
  do {                                                                          \
    cudaError_t _e = (expr);                                                    \
    if (_e != cudaSuccess)                                                      \
      return boa_fail(BOA_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)
