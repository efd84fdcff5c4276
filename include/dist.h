// Drop-in replacement for the reference's include/dist.h:12-36.
//
// Environment: RANK, WORLD_SIZE, LOCAL_RANK, NCCL_UID_PATH (file rendezvous of
// the ncclUniqueId, rank 0 writes it atomically). NCCL is loaded at run time
// by librnet_b200.so, so no RNET_NCCL build switch is needed.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdio>
#include <string>

struct rnet_dist;

namespace rnet {

struct DistState {
  int world_size = 1;
  int rank = 0;
  int local_rank = 0;
  rnet_dist* comm = nullptr;  // library communicator (null when single-process)
  bool active() const { return world_size > 1; }
  bool is_master() const { return rank == 0; }
};

// Reads the environment, calls cudaSetDevice(local_rank) and, when
// WORLD_SIZE > 1, creates the NCCL communicator. Failures print and abort(),
// as in the reference (rendezvous deadline 120 s).
DistState dist_init_from_env();

void dist_destroy(DistState& st);

// In-place sum all-reduce on `stream`; no-op when inactive.
void dist_allreduce_sum(DistState& st, float* buf, size_t count, cudaStream_t stream);

void dist_group_start(DistState& st);
void dist_group_end(DistState& st);

}  // namespace rnet
