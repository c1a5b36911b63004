// Status codes and the thread-local error message behind every extern "C" entry point.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "../../include/b200ep.h"

namespace b200ep {

// Records `msg` as this thread's last error (read by b200ep_last_error) and returns `code`.
int set_error(int code, const std::string& msg);
void clear_error();

inline int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return B200EP_OK;
  return set_error(B200EP_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace b200ep

#define B200EP_CHECK_ARG(cond, msg)                          \
  do {                                                       \
    if (!(cond)) return ::b200ep::set_error(B200EP_EINVAL, msg); \
  } while (0)

#define B200EP_CUDA_RET(expr)                                      \
  do {                                                             \
    cudaError_t _e = (expr);                                       \
    if (_e != cudaSuccess) return ::b200ep::cuda_status(_e, #expr); \
  } while (0)
