// Status / error plumbing of the C ABI.
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>

#include "status.h"

namespace rnet_status {

static thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int fail_cuda(cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                  cudaGetErrorString(e) + ")";
  g_last_error = m;
  return RNET_ERR_CUDA;
}

// One error word per device, allocated lazily and never freed (it lives as
// long as the library's context on that device).
unsigned* device_error_word() {
  static std::mutex mu;
  static unsigned* words[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!words[dev]) {
    unsigned* p = nullptr;
    if (cudaMalloc(&p, sizeof(unsigned)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(unsigned)) != cudaSuccess) return nullptr;
    words[dev] = p;
  }
  return words[dev];
}

static std::atomic<unsigned long long> g_launches{0};
void count_launch(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
unsigned long long launches() { return g_launches.load(std::memory_order_relaxed); }

}  // namespace rnet_status

namespace rnet_k {
cudaError_t launched(unsigned n) {
  rnet_status::count_launch(n);
  return cudaGetLastError();
}
}  // namespace rnet_k

extern "C" const char* rnet_last_error(void) { return rnet_status::g_last_error.c_str(); }

extern "C" int rnet_kernel_launches(unsigned long long* n) {
  if (!n) return rnet_status::fail(RNET_ERR_ARG, "null output");
  *n = rnet_status::launches();
  return RNET_OK;
}

extern "C" int rnet_abi_version(void) { return 100; }

extern "C" int rnet_device_error(unsigned* word, int clear) {
  if (!word) return rnet_status::fail(RNET_ERR_ARG, "rnet_device_error: null output");
  unsigned* d = rnet_status::device_error_word();
  if (!d) return rnet_status::fail(RNET_ERR_CUDA, "rnet_device_error: no device error word");
  RNET_TRY_CUDA(cudaDeviceSynchronize());
  RNET_TRY_CUDA(cudaMemcpy(word, d, sizeof(unsigned), cudaMemcpyDeviceToHost));
  if (clear) RNET_TRY_CUDA(cudaMemset(d, 0, sizeof(unsigned)));
  return RNET_OK;
}
