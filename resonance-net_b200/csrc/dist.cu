// NCCL data-parallel plumbing (see dist.h).
//
// Reference: src/dist.cpp:31-127 — blocking ncclCommInitRank, one grouped
// ncclAllReduce per parameter tensor issued after the whole backward on the
// compute stream, errors abort(). Here: a non-blocking communicator polled
// against a deadline, and contiguous gradient buckets (one per layer of the
// flat gradient buffer) all-reduced on a separate stream as soon as backward
// has produced them, overlapping the remaining backward.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "dist.h"
#include "kernels.cuh"
#include "status.h"

namespace rnet_engine {

namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
  const char* (*GetErrorString)(ncclResult_t);
};

NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.why = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
#define SYM(field, name)                                                   \
  a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name));           \
  if (!a.field) {                                                          \
    a.why = std::string("NCCL symbol missing: ") + name;                   \
    return;                                                                \
  }
    SYM(GetUniqueId, "ncclGetUniqueId");
    SYM(CommInitRankConfig, "ncclCommInitRankConfig");
    SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    SYM(CommAbort, "ncclCommAbort");
    SYM(CommDestroy, "ncclCommDestroy");
    SYM(AllReduce, "ncclAllReduce");
    SYM(GroupStart, "ncclGroupStart");
    SYM(GroupEnd, "ncclGroupEnd");
    SYM(GetErrorString, "ncclGetErrorString");
#undef SYM
    a.ok = true;
  });
  return a;
}

int nccl_fail(ncclResult_t r, const char* what) {
  NcclApi& a = api();
  return rnet_status::fail(RNET_ERR_NCCL, std::string(what) + ": " +
                                              (a.ok ? a.GetErrorString(r) : "nccl unavailable"));
}

}  // namespace

class DistComm {
 public:
  int world = 1, rank = 0, local_rank = 0;
  ncclComm_t comm = nullptr;
  cudaStream_t comm_stream = nullptr;
  // cudaStreamWaitEvent captures the event's state when it is called, so one
  // event per direction can be re-recorded for every bucket.
  cudaEvent_t to_comm = nullptr, to_compute = nullptr;
  int timeout_ms = 120000;

  // Non-blocking communicator: wait until the last call left ncclInProgress.
  int settle(const char* what) {
    NcclApi& a = api();
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
      ncclResult_t st = ncclSuccess;
      ncclResult_t r = a.CommGetAsyncError(comm, &st);
      if (r != ncclSuccess) return nccl_fail(r, what);
      if (st == ncclSuccess) return RNET_OK;
      if (st != ncclInProgress) return nccl_fail(st, what);
      if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
        a.CommAbort(comm);
        comm = nullptr;
        return rnet_status::fail(RNET_ERR_TIMEOUT, std::string(what) + ": NCCL deadline exceeded");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  }
};

int dist_unique_id(unsigned char uid[128]) {
  NcclApi& a = api();
  if (!a.ok) return rnet_status::fail(RNET_ERR_NCCL, a.why);
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  ncclUniqueId id;
  ncclResult_t r = a.GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(uid, &id, 128);
  return RNET_OK;
}

int dist_create(int rank, int world, int local_rank, const unsigned char uid[128],
                int timeout_ms, DistComm** out) {
  if (!out || world < 1 || rank < 0 || rank >= world)
    return rnet_status::fail(RNET_ERR_ARG, "dist_create: bad rank/world");
  NcclApi& a = api();
  if (!a.ok) return rnet_status::fail(RNET_ERR_NCCL, a.why);
  RNET_TRY_CUDA(cudaSetDevice(local_rank));
  DistComm* d = new DistComm();
  d->world = world;
  d->rank = rank;
  d->local_rank = local_rank;
  d->timeout_ms = timeout_ms > 0 ? timeout_ms : 120000;
  ncclUniqueId id;
  std::memcpy(&id, uid, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  // Cap on the SMs NCCL's kernels occupy while backward runs beside them
  // (the GEMM and conv-backward grids are persistent, one CTA per SM):
  // RNET_NCCL_MAX_CTAS, default NCCL's own choice.
  if (const char* e = getenv("RNET_NCCL_MAX_CTAS")) {
    const int v = atoi(e);
    if (v > 0) {
      cfg.maxCTAs = v;
      if (cfg.minCTAs > v || cfg.minCTAs == NCCL_CONFIG_UNDEF_INT) cfg.minCTAs = 1;
    }
  }
  ncclResult_t r = a.CommInitRankConfig(&d->comm, world, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete d;
    return nccl_fail(r, "ncclCommInitRankConfig");
  }
  int rc = d->settle("ncclCommInitRankConfig");
  if (rc) {
    delete d;
    return rc;
  }
  cudaError_t e = cudaStreamCreateWithFlags(&d->comm_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&d->to_comm, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&d->to_compute, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    dist_destroy(d);
    return rnet_status::fail_cuda(e, "dist comm stream");
  }
  *out = d;
  return RNET_OK;
}

void dist_destroy(DistComm* d) {
  if (!d) return;
  NcclApi& a = api();
  if (d->comm_stream) cudaStreamSynchronize(d->comm_stream);
  if (d->comm && a.ok) a.CommDestroy(d->comm);
  if (d->to_comm) cudaEventDestroy(d->to_comm);
  if (d->to_compute) cudaEventDestroy(d->to_compute);
  if (d->comm_stream) cudaStreamDestroy(d->comm_stream);
  delete d;
}

int dist_world(const DistComm* d) { return d ? d->world : 1; }
int dist_rank(const DistComm* d) { return d ? d->rank : 0; }

int dist_reduce_range(DistComm* d, float* buf, size_t count, cudaStream_t compute,
                      __nv_bfloat16* scratch16) {
  if (!d || d->world <= 1 || count == 0) return RNET_OK;
  NcclApi& a = api();
  RNET_TRY_CUDA(cudaEventRecord(d->to_comm, compute));
  RNET_TRY_CUDA(cudaStreamWaitEvent(d->comm_stream, d->to_comm, 0));
  if (scratch16) {
    // bf16 on the wire: half the bytes; the summed bf16 values come back
    // into the fp32 gradient (the comm stream orders the shared scratch)
    RNET_TRY_CUDA(rnet_k::to_bf16(buf, scratch16, count, d->comm_stream));
    ncclResult_t r = a.AllReduce(scratch16, scratch16, count, ncclBfloat16, ncclSum, d->comm,
                                 d->comm_stream);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclAllReduce(bf16)");
    int rc = d->settle("ncclAllReduce(bf16)");
    if (rc) return rc;
    RNET_TRY_CUDA(rnet_k::from_bf16(scratch16, buf, count, d->comm_stream));
    return RNET_OK;
  }
  ncclResult_t r = a.AllReduce(buf, buf, count, ncclFloat32, ncclSum, d->comm, d->comm_stream);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclAllReduce");
  return d->settle("ncclAllReduce");
}

int dist_wait(DistComm* d, cudaStream_t compute) {
  if (!d || d->world <= 1) return RNET_OK;
  RNET_TRY_CUDA(cudaEventRecord(d->to_compute, d->comm_stream));
  RNET_TRY_CUDA(cudaStreamWaitEvent(compute, d->to_compute, 0));
  return RNET_OK;
}

int dist_allreduce_on(DistComm* d, float* buf, size_t count, cudaStream_t stream) {
  if (!d || d->world <= 1 || count == 0) return RNET_OK;
  NcclApi& a = api();
  ncclResult_t r = a.AllReduce(buf, buf, count, ncclFloat32, ncclSum, d->comm, stream);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclAllReduce");
  return d->settle("ncclAllReduce");
}

int dist_group_start(DistComm* d) {
  if (!d || d->world <= 1) return RNET_OK;
  ncclResult_t r = api().GroupStart();
  return r == ncclSuccess ? RNET_OK : nccl_fail(r, "ncclGroupStart");
}

int dist_group_end(DistComm* d) {
  if (!d || d->world <= 1) return RNET_OK;
  ncclResult_t r = api().GroupEnd();
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclGroupEnd");
  return d->settle("ncclGroupEnd");
}

}  // namespace rnet_engine
