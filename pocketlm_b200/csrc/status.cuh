// Error reporting shared by the C entry points: the message of the last
// failing call on the calling thread (moe_b200_last_error).
#pragma once
#include <cstdio>

#include "common.cuh"

namespace moe {

inline thread_local char g_last_error[512] = "";

inline int fail(int code, const char* what) {
  std::snprintf(g_last_error, sizeof g_last_error, "%s", what);
  return code;
}

inline int cuda_fail(cudaError_t err, const char* where) {
  std::snprintf(g_last_error, sizeof g_last_error, "%s: %s", where, cudaGetErrorString(err));
  return kCudaError - static_cast<int>(err);
}

}  // namespace moe

#define MOE_CUDA(expr, where)                               \
  do {                                                      \
    cudaError_t _e = (expr);                                \
    if (_e != cudaSuccess) return ::moe::cuda_fail(_e, where); \
  } while (0)
