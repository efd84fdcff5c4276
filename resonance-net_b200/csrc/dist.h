// Data-parallel gradient exchange over NCCL (NVLink / NVSwitch).
//
// NCCL is resolved at run time (dlopen "libnccl.so.2", reusing a copy that is
// already loaded in the process, e.g. PyTorch's), so the library has no hard
// link dependency and a missing NCCL is a clean RNET_ERR_NCCL.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstddef>

namespace rnet_engine {

class DistComm;

int dist_unique_id(unsigned char uid[128]);
// Non-blocking communicator init polled against a host deadline; on timeout
// the communicator is aborted and RNET_ERR_TIMEOUT returned.
int dist_create(int rank, int world, int local_rank, const unsigned char uid[128],
                int timeout_ms, DistComm** out);
void dist_destroy(DistComm* d);
int dist_world(const DistComm* d);
int dist_rank(const DistComm* d);
// Enqueue an in-place sum all-reduce of buf[0:count] on the comm stream,
// ordered after all work already queued on `compute`: fp32 on the wire, or
// bf16 when scratch16 (count bf16 elements) is given.
int dist_reduce_range(DistComm* d, float* buf, size_t count, cudaStream_t compute,
                      __nv_bfloat16* scratch16 = nullptr);
// Make `compute` wait for every reduction enqueued so far.
int dist_wait(DistComm* d, cudaStream_t compute);
// Synchronous-order all-reduce on `stream` itself (drop-in dist_allreduce_sum).
int dist_allreduce_on(DistComm* d, float* buf, size_t count, cudaStream_t stream);
int dist_group_start(DistComm* d);
int dist_group_end(DistComm* d);

}  // namespace rnet_engine
