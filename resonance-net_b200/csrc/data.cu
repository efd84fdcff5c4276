// Training batches on the device (the reference's DataLoader, restated).
//
// Reference: src/data_loader.cpp:31-52 (get_batch) driven by
// src/main.cpp:117-133 — per step the host draws B window starts with
// std::uniform_int_distribution<size_t>(0, size - seq_len - 2) from a
// std::mt19937, copies B*T input and target bytes into host arrays and
// uploads both with synchronous cudaMemcpy (2 * B * T * 4 bytes per step).
//
// Here the byte corpus is uploaded once and stays resident in HBM. Per step
// the host makes the same B draws from the same generator (so the batches are
// the reference's, byte for byte, for the same seed), puts the B starts in
// a pinned slot, copies them asynchronously (8 bytes per sequence) and one
// kernel gathers the windows into int32 inputs / targets on the caller's
// stream. A ring of pinned slots, each guarded by an event, lets the host
// draw step k+1 while step k's copy is in flight: no host synchronisation.
//
// Without a corpus (n = 0) the reference draws synthetic tokens
// (input = rng() % 256, target = rng() % 256, interleaved per position);
// that path is restated on the host and uploaded from pinned memory.
#include <cstdint>
#include <cstring>
#include <random>
#include <vector>

#include "kernels.cuh"
#include "status.h"

namespace {

constexpr int SLOTS = 4;

__global__ void gather_windows_kernel(const unsigned char* __restrict__ bytes,
                                      const unsigned long long* __restrict__ starts, int T,
                                      int* __restrict__ inputs, int* __restrict__ targets) {
  const int b = blockIdx.y;
  const unsigned long long p = starts[b];
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
    inputs[(size_t)b * T + t] = (int)bytes[p + t];
    targets[(size_t)b * T + t] = (int)bytes[p + t + 1];
  }
}

}  // namespace

struct rnet_data {
  int device = 0;
  unsigned char* d_bytes = nullptr;
  size_t n = 0;
  std::mt19937 rng;
  // pinned ring: starts (corpus) or synthetic inputs|targets
  void* h_slot[SLOTS] = {nullptr};
  size_t slot_bytes = 0;
  unsigned long long* d_starts[SLOTS] = {nullptr};
  cudaEvent_t done[SLOTS] = {nullptr};
  int next = 0;
};

extern "C" {

int rnet_data_create(const unsigned char* host_bytes, size_t n, int device, unsigned seed,
                     rnet_data** out) {
  if (!out) return rnet_status::fail(RNET_ERR_ARG, "rnet_data_create: null output");
  if (n > 0 && !host_bytes) return rnet_status::fail(RNET_ERR_ARG, "rnet_data_create: null bytes");
  RNET_TRY_CUDA(cudaSetDevice(device));
  rnet_data* d = new rnet_data();
  d->device = device;
  d->n = n;
  d->rng.seed(seed);
  cudaError_t e = cudaSuccess;
  if (n > 0) {
    e = cudaMalloc(&d->d_bytes, n);
    if (e == cudaSuccess) e = cudaMemcpy(d->d_bytes, host_bytes, n, cudaMemcpyHostToDevice);
  }
  for (int i = 0; i < SLOTS && e == cudaSuccess; ++i)
    e = cudaEventCreateWithFlags(&d->done[i], cudaEventDisableTiming);
  if (e != cudaSuccess) {
    rnet_data_destroy(d);
    return rnet_status::fail_cuda(e, "rnet_data_create");
  }
  *out = d;
  return RNET_OK;
}

int rnet_data_destroy(rnet_data* d) {
  if (!d) return RNET_OK;
  cudaSetDevice(d->device);
  for (int i = 0; i < SLOTS; ++i) {
    if (d->done[i]) {
      cudaEventSynchronize(d->done[i]);
      cudaEventDestroy(d->done[i]);
    }
    if (d->h_slot[i]) cudaFreeHost(d->h_slot[i]);
    if (d->d_starts[i]) cudaFree(d->d_starts[i]);
  }
  if (d->d_bytes) cudaFree(d->d_bytes);
  delete d;
  return RNET_OK;
}

int rnet_data_batch(rnet_data* d, int batch, int seq_len, int* d_inputs, int* d_targets,
                    void* stream) {
  if (!d || !d_inputs || !d_targets)
    return rnet_status::fail(RNET_ERR_ARG, "rnet_data_batch: null argument");
  if (batch <= 0 || seq_len <= 0) return rnet_status::fail(RNET_ERR_ARG, "rnet_data_batch: empty");
  if (d->n > 0 && d->n < (size_t)seq_len + 2)
    return rnet_status::fail(RNET_ERR_ARG, "rnet_data_batch: corpus shorter than seq_len + 2");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t BT = (size_t)batch * seq_len;
  const size_t need = d->n > 0 ? batch * sizeof(unsigned long long) : 2 * BT * sizeof(int);
  if (need > d->slot_bytes) {
    for (int i = 0; i < SLOTS; ++i) {
      RNET_TRY_CUDA(cudaEventSynchronize(d->done[i]));
      if (d->h_slot[i]) cudaFreeHost(d->h_slot[i]);
      if (d->d_starts[i]) cudaFree(d->d_starts[i]);
      d->h_slot[i] = nullptr;
      d->d_starts[i] = nullptr;
      RNET_TRY_CUDA(cudaMallocHost(&d->h_slot[i], need));
      if (d->n > 0) RNET_TRY_CUDA(cudaMalloc(&d->d_starts[i], need));
    }
    d->slot_bytes = need;
  }
  const int k = d->next;
  d->next = (k + 1) % SLOTS;
  // the slot's previous copy has left the pinned buffer
  RNET_TRY_CUDA(cudaEventSynchronize(d->done[k]));
  if (d->n == 0) {
    // src/data_loader.cpp:33-41: interleaved input / target draws
    int* hi = static_cast<int*>(d->h_slot[k]);
    int* ht = hi + BT;
    for (size_t i = 0; i < BT; ++i) {
      hi[i] = (int)(d->rng() % 256);
      ht[i] = (int)(d->rng() % 256);
    }
    RNET_TRY_CUDA(cudaMemcpyAsync(d_inputs, hi, BT * sizeof(int), cudaMemcpyHostToDevice, s));
    RNET_TRY_CUDA(cudaMemcpyAsync(d_targets, ht, BT * sizeof(int), cudaMemcpyHostToDevice, s));
  } else {
    // src/data_loader.cpp:43-51: one window start per sequence
    unsigned long long* hs = static_cast<unsigned long long*>(d->h_slot[k]);
    std::uniform_int_distribution<size_t> dist(0, d->n - seq_len - 2);
    for (int b = 0; b < batch; ++b) hs[b] = (unsigned long long)dist(d->rng);
    RNET_TRY_CUDA(cudaMemcpyAsync(d->d_starts[k], hs, batch * sizeof(unsigned long long),
                                  cudaMemcpyHostToDevice, s));
    dim3 grid((seq_len + 255) / 256 < 8 ? (seq_len + 255) / 256 : 8, batch);
    gather_windows_kernel<<<grid, 256, 0, s>>>(d->d_bytes, d->d_starts[k], seq_len, d_inputs,
                                               d_targets);
    RNET_TRY_CUDA(rnet_k::launched());
  }
  RNET_TRY_CUDA(cudaEventRecord(d->done[k], s));
  return RNET_OK;
}

}  // extern "C"
