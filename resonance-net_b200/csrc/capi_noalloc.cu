// Allocation-free variant of the cross-entropy op for callers that cannot
// allocate device memory while they run: a host framework that owns all
// device memory through its own pool or arena (and forbids other allocators
// from taking memory behind its back), or code that calls into this library
// from a context where cudaMalloc / cudaMallocAsync would be an implicit
// synchronisation or is simply not allowed. The regular
// rnet_cross_entropy_forward takes its per-block loss partials from a
// stream-ordered cudaMallocAsync; this variant uses a fixed scratch array
// that lives in the library's own device image instead.
//
// The scratch array holds at most RNET_NOALLOC_CE_MAX_PARTIALS floats (one
// partial per 8 tokens), i.e. 256 KiB on every GPU that loads the library,
// kept until the process exits. That bounds batch_seq to
// 8 * RNET_NOALLOC_CE_MAX_PARTIALS - 8 = 524,280 tokens per call.
#include <mutex>
#include <string>

#include "kernels.cuh"
#include "status.h"

namespace {

constexpr size_t RNET_NOALLOC_CE_MAX_PARTIALS = 65536;

// Device scratch shared by every call on a device. In host code this name is
// only a stand-in for the symbol; the device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) float g_ce_scratch[RNET_NOALLOC_CE_MAX_PARTIALS];

// Per-device address of g_ce_scratch, looked up once per device with that
// device current and cached for the life of the process. A cudaDeviceReset
// unloads the module and may move the array, so this entry point must not be
// used on a device after cudaDeviceReset has been called on it.
float* scratch_address(int dev, cudaError_t* err) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_ce_scratch);
    if (*err != cudaSuccess) return nullptr;
    addr[dev] = static_cast<float*>(p);
  }
  *err = cudaSuccess;
  return addr[dev];
}

}  // namespace

extern "C" int rnet_cross_entropy_forward_noalloc(const float* logits, const int* targets,
                                                  float* loss, float* dlogits, int batch_seq,
                                                  int vocab, void* stream) {
  if (!logits || !targets || !loss || !dlogits)
    return rnet_status::fail(RNET_ERR_ARG, "cross_entropy_forward_noalloc: null pointer");
  if (batch_seq < 0 || vocab <= 0)
    return rnet_status::fail(RNET_ERR_ARG, "cross_entropy_forward_noalloc: bad size");
  const size_t need = rnet_k::ce_partials_floats(batch_seq);
  if (need > RNET_NOALLOC_CE_MAX_PARTIALS)
    return rnet_status::fail(
        RNET_ERR_ARG, "cross_entropy_forward_noalloc: batch_seq " + std::to_string(batch_seq) +
                          " exceeds the fixed scratch limit of " +
                          std::to_string(8 * (RNET_NOALLOC_CE_MAX_PARTIALS - 1)) + " tokens");
  int dev = 0;
  RNET_TRY_CUDA(cudaGetDevice(&dev));
  cudaError_t e = cudaSuccess;
  float* scratch = scratch_address(dev, &e);
  if (!scratch) return rnet_status::fail_cuda(e, "cudaGetSymbolAddress(g_ce_scratch)");
  // Every partial the loss reduction reads is written by the same call first,
  // so stale contents from an earlier call need no clearing. No error word is
  // passed (that word is allocated on first use): out-of-range targets are
  // clamped to class 0 without being reported.
  RNET_TRY_CUDA(rnet_k::cross_entropy(logits, targets, loss, dlogits, 1.0f, scratch, batch_seq,
                                      vocab, nullptr, (cudaStream_t)stream));
  return RNET_OK;
}
