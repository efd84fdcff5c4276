// Host-side status plumbing shared by every C-ABI entry point.
#pragma once
#include <cuda_runtime.h>
#include <string>

#include "../../include/rnet_capi.h"

namespace rnet_status {

// Record a message for rnet_last_error() and return `code`.
int fail(int code, const std::string& msg);
int fail_cuda(cudaError_t e, const char* what);

// Device error word (bounded-wait timeouts, bad indices) shared by all kernels
// of this library on the current device.
unsigned* device_error_word();

// Count of kernels launched by this library (process-wide).
void count_launch(unsigned n = 1);
unsigned long long launches();

}  // namespace rnet_status

#define RNET_TRY_CUDA(expr)                                            \
  do {                                                                 \
    cudaError_t _e = (expr);                                           \
    if (_e != cudaSuccess) return rnet_status::fail_cuda(_e, #expr);   \
  } while (0)
