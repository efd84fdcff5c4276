// Self-test of the bounded-wait failure path shared by the pipelined kernels
// (GEMM, conv backward, RMSNorm backward).
//
// Every spin on an mbarrier in this library goes through mbar_wait_for():
// after a time limit the waiting role sets ERR_WAIT_TIMEOUT in the device
// error word, raises the CTA's shared abort flag so the other roles stop
// waiting too, and the CTA unwinds: the TMEM-owning warp still deallocates
// its columns and every thread returns. This kernel reproduces that exact
// role structure (one TMEM-owning warp, waiters on a "full" barrier) around
// a barrier that nothing arrives on, so the path can be exercised on a GPU
// without a fault, a trap or a hang: the wait runs out after `timeout_ns`
// (a few milliseconds in the tests) and the kernel returns normally.
//
// With arrive != 0 one thread arrives on the barrier, the control case: the
// waits succeed and no error bit is set.
#include "common.cuh"
#include "kernels.cuh"
#include "status.h"

namespace {

using namespace rnet_dev;

__global__ void __launch_bounds__(128) bounded_wait_selftest_kernel(int arrive, uint64_t timeout_ns,
                                                                    unsigned* err,
                                                                    unsigned* result) {
  __shared__ __align__(8) uint64_t full_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ int timed_out;
  const int warp = threadIdx.x / 32;
  if (threadIdx.x == 0) {
    mbar_init(&full_bar, 1);
    abort_flag = 0;
    timed_out = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc<1>(&tmem_base, 32);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (arrive && threadIdx.x == 32) mbar_arrive(&full_bar);
  // every role waits on the phase, as producer/consumer roles do
  const bool ok = mbar_wait_for(&full_bar, 0, err, &abort_flag, timeout_ns);
  if (!ok) atomicExch(&timed_out, 1);
  tc_fence_before();
  __syncthreads();
  // teardown runs on both paths: the TMEM owner frees its columns
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc<1>(tmem_base, 32);
  }
  if (threadIdx.x == 0)
    atomicAdd(result, timed_out ? 1u : 0u);
}

}  // namespace

extern "C" int rnet_selftest_bounded_wait(int arrive, unsigned timeout_us, int n_ctas,
                                          unsigned* h_timed_out_ctas) {
  if (!h_timed_out_ctas || n_ctas <= 0 || n_ctas > 1024 || timeout_us == 0 ||
      timeout_us > 1000000)
    return rnet_status::fail(RNET_ERR_ARG,
                             "rnet_selftest_bounded_wait: need 1..1024 CTAs, 1 us..1 s limit");
  unsigned* err = rnet_status::device_error_word();
  if (!err) return rnet_status::fail(RNET_ERR_CUDA, "no device error word");
  unsigned* d_res = nullptr;
  RNET_TRY_CUDA(cudaMalloc(&d_res, sizeof(unsigned)));
  cudaError_t e = cudaMemset(d_res, 0, sizeof(unsigned));
  if (e == cudaSuccess) {
    bounded_wait_selftest_kernel<<<n_ctas, 128>>>(arrive, (uint64_t)timeout_us * 1000ull, err,
                                                  d_res);
    e = rnet_k::launched();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(h_timed_out_ctas, d_res, sizeof(unsigned),
                                       cudaMemcpyDeviceToHost);
  cudaFree(d_res);
  if (e != cudaSuccess) return rnet_status::fail_cuda(e, "rnet_selftest_bounded_wait");
  return RNET_OK;
}
