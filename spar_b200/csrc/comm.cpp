// Data-parallel gradient reduction over NCCL (NVLink / NVSwitch inside one box).
//
// Spar itself has no collectives (cross-device copies bounce through the host,
// src/backend/cuda_runtime.cppm:212-237); this is the new data-parallel exchange: one sum
// all-reduce per gradient bucket, issued on a communication stream. NCCL is resolved at run time
// with dlopen("libnccl.so.2"), so the library binds to whichever NCCL the process already loaded
// (torch's) and needs no link-time dependency.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <thread>

#include "spar_b200.h"

namespace spar_b200 {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                                 ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.init_rank = reinterpret_cast<decltype(a.init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.reduce_scatter = reinterpret_cast<decltype(a.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(h, "ncclCommDestroy"));
    a.abort = reinterpret_cast<decltype(a.abort)>(dlsym(h, "ncclCommAbort"));
    a.async_error = reinterpret_cast<decltype(a.async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    a.ok = a.get_unique_id && a.init_rank && a.all_reduce && a.reduce_scatter && a.all_gather &&
           a.destroy && a.abort;
  });
  return a;
}

// Seconds a bounded wait on a step's collectives may take before the communicator is aborted:
// $SPAR_B200_COMM_TIMEOUT_S, default 600 (well above any step; a peer that left or hung is the
// only way to reach it).
double default_timeout() {
  const char* e = getenv("SPAR_B200_COMM_TIMEOUT_S");
  const double v = e ? atof(e) : 0.0;
  return v > 0.0 ? v : 600.0;
}

struct Comm {
  ncclComm_t nccl = nullptr;
  int rank = 0, world = 1, device = 0;
  double timeout_s = default_timeout();
  bool aborted = false;
  // The abort runs on its own thread (see comm_wait); set when ncclCommAbort has returned.
  // While it has not, the handle is never freed (the thread still uses it).
  std::shared_ptr<std::atomic<bool>> abort_done;
};

// Seconds comm_wait waits for ncclCommAbort to return before reporting the failure anyway.
constexpr double kAbortWaitS = 20.0;

// Status for a failed NCCL call: code 3, the ncclResult_t in cuda_error.
SparCudaStatus nccl_status(ncclResult_t r) { return {r == ncclSuccess ? 0 : 3, static_cast<int>(r)}; }

}  // namespace

cudaError_t comm_allreduce_sum(void* comm, float* data, uint64_t count, cudaStream_t stream) {
  const Comm* c = static_cast<const Comm*>(comm);
  if (!c || !api().ok || c->aborted) return cudaErrorInvalidValue;
  const ncclResult_t r = api().all_reduce(data, data, count, ncclFloat32, ncclSum, c->nccl, stream);
  return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

cudaError_t comm_allreduce_sum_f64(void* comm, double* data, uint64_t count, cudaStream_t stream) {
  const Comm* c = static_cast<const Comm*>(comm);
  if (!c || !api().ok || c->aborted) return cudaErrorInvalidValue;
  const ncclResult_t r = api().all_reduce(data, data, count, ncclFloat64, ncclSum, c->nccl, stream);
  return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

// In place: data[world * shard] in, the sum of every rank's data[rank * shard, + shard) lands
// there (the rest of data is left unspecified).
cudaError_t comm_reduce_scatter_sum(void* comm, float* data, uint64_t shard, cudaStream_t stream) {
  const Comm* c = static_cast<const Comm*>(comm);
  if (!c || !api().ok || c->aborted) return cudaErrorInvalidValue;
  const ncclResult_t r = api().reduce_scatter(data, data + static_cast<uint64_t>(c->rank) * shard,
                                              shard, ncclFloat32, ncclSum, c->nccl, stream);
  return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

// In place: every rank's data[rank * shard, + shard) is copied to the same place on all ranks.
cudaError_t comm_all_gather(void* comm, float* data, uint64_t shard, cudaStream_t stream) {
  const Comm* c = static_cast<const Comm*>(comm);
  if (!c || !api().ok || c->aborted) return cudaErrorInvalidValue;
  const ncclResult_t r = api().all_gather(data + static_cast<uint64_t>(c->rank) * shard, data,
                                          shard, ncclFloat32, c->nccl, stream);
  return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

// Waits for `stream` (whose work includes this communicator's collectives) with a deadline,
// polling the stream and NCCL's asynchronous error state. A collective whose peer left or failed
// never completes: on an asynchronous error or at the deadline the communicator is aborted
// (ncclCommAbort stops its kernels, so the stream drains) and {3, ncclResult} is returned; the
// communicator is unusable afterwards. The communicator stays blocking (collective enqueues never
// return ncclInProgress), which keeps the step's collectives capturable in a CUDA graph on the
// calling thread; this wait is where a hang would otherwise show.
// SPAR_B200_COMM_TRACE=1: the failure path reports its stages on stderr.
bool comm_trace() {
  static const bool on = getenv("SPAR_B200_COMM_TRACE") && getenv("SPAR_B200_COMM_TRACE")[0] == '1';
  return on;
}

SparCudaStatus comm_wait(void* comm, cudaStream_t stream) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return {1, static_cast<int>(cudaErrorInvalidValue)};
  if (c->aborted) return {3, static_cast<int>(ncclInvalidUsage)};
  const auto start = std::chrono::steady_clock::now();
  auto sleep_us = std::chrono::microseconds(20);
  for (;;) {
    const cudaError_t q = cudaStreamQuery(stream);
    if (q == cudaSuccess) return {0, 0};
    if (q != cudaErrorNotReady) return {2, static_cast<int>(q)};
    ncclResult_t async = ncclSuccess;
    if (api().async_error) {
      const ncclResult_t r = api().async_error(c->nccl, &async);
      if (r != ncclSuccess) async = r;
    }
    const double waited =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
    if ((async != ncclSuccess && async != ncclInProgress) || waited > c->timeout_s) {
      if (comm_trace())
        fprintf(stderr, "spar_b200 comm_wait: rank %d gives up after %.1f s (async %d), aborting\n",
                c->rank, waited, static_cast<int>(async));
      // ncclCommAbort stops the communicator's kernels (they see its abort flag and return), but
      // it has been seen to block the calling thread while the step's captured collectives were
      // in flight. It runs on a detached thread, waited for at most kAbortWaitS, so the step
      // reports the failure within its bound either way.
      c->aborted = true;
      c->abort_done = std::make_shared<std::atomic<bool>>(false);
      {
        ncclComm_t nc = c->nccl;
        auto done = c->abort_done;
        std::thread([nc, done] {
          api().abort(nc);
          done->store(true);
        }).detach();
      }
      c->nccl = nullptr;
      const auto stop = std::chrono::steady_clock::now();
      while (!c->abort_done->load() &&
             std::chrono::steady_clock::now() - stop < std::chrono::duration<double>(kAbortWaitS))
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
      const bool returned = c->abort_done->load();
      if (comm_trace())
        fprintf(stderr, "spar_b200 comm_wait: rank %d abort %s\n", c->rank,
                returned ? "returned" : "still running (the step's streams may not drain)");
      cudaError_t q2 = cudaErrorNotReady;
      if (returned) {
        const auto drain = std::chrono::steady_clock::now();
        while ((q2 = cudaStreamQuery(stream)) == cudaErrorNotReady &&
               std::chrono::steady_clock::now() - drain < std::chrono::seconds(30))
          std::this_thread::sleep_for(std::chrono::milliseconds(1));
        if (comm_trace())
          fprintf(stderr, "spar_b200 comm_wait: rank %d stream after abort: %s\n", c->rank,
                  q2 == cudaSuccess ? "drained" : cudaGetErrorString(q2));
      }
      cudaGetLastError();
      // ncclInProgress: the abort (or the drain) had not finished when the wait gave up.
      if (!returned || q2 != cudaSuccess) return {3, static_cast<int>(ncclInProgress)};
      return {3, static_cast<int>(async != ncclSuccess ? async : ncclRemoteError)};
    }
    std::this_thread::sleep_for(sleep_us);
    if (sleep_us < std::chrono::microseconds(1000)) sleep_us *= 2;
  }
}

int comm_rank(void* comm) { return comm ? static_cast<const Comm*>(comm)->rank : 0; }
int comm_size(void* comm) { return comm ? static_cast<const Comm*>(comm)->world : 1; }

}  // namespace spar_b200

using namespace spar_b200;

extern "C" SparCudaStatus spar_b200_comm_unique_id(char* out, uint64_t capacity) {
  if (!out || capacity < sizeof(ncclUniqueId)) return {1, static_cast<int>(cudaErrorInvalidValue)};
  if (!api().ok) return {3, static_cast<int>(ncclSystemError)};
  ncclUniqueId id;
  const ncclResult_t r = api().get_unique_id(&id);
  if (r == ncclSuccess) std::memcpy(out, &id, sizeof(id));
  return nccl_status(r);
}

extern "C" SparCudaStatus spar_b200_comm_init(const char* unique_id, int rank, int world_size,
                                              int device, void** comm) {
  if (!unique_id || !comm || world_size < 1 || rank < 0 || rank >= world_size)
    return {1, static_cast<int>(cudaErrorInvalidValue)};
  *comm = nullptr;
  if (!api().ok) return {3, static_cast<int>(ncclSystemError)};
  int previous = 0;
  cudaGetDevice(&previous);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return {2, static_cast<int>(e)};
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  Comm* c = new Comm();
  c->rank = rank;
  c->world = world_size;
  c->device = device;
  const ncclResult_t r = api().init_rank(&c->nccl, world_size, id, rank);
  cudaSetDevice(previous);
  if (r != ncclSuccess) {
    delete c;
    return nccl_status(r);
  }
  *comm = c;
  return {0, 0};
}

extern "C" SparCudaStatus spar_b200_comm_allreduce_sum(void* comm, float* data, uint64_t count,
                                                       void* stream) {
  if (!comm || (count && !data)) return {1, static_cast<int>(cudaErrorInvalidValue)};
  if (count == 0) return {0, 0};
  const Comm* c = static_cast<const Comm*>(comm);
  if (c->aborted) return {3, static_cast<int>(ncclInvalidUsage)};
  const ncclResult_t r = api().all_reduce(data, data, count, ncclFloat32, ncclSum, c->nccl,
                                          static_cast<cudaStream_t>(stream));
  return nccl_status(r);
}

// Polls the communicator's asynchronous error state (a peer that died, a network failure).
extern "C" SparCudaStatus spar_b200_comm_check(void* comm) {
  if (!comm) return {1, static_cast<int>(cudaErrorInvalidValue)};
  const Comm* c = static_cast<const Comm*>(comm);
  if (c->aborted) return {3, static_cast<int>(ncclRemoteError)};
  if (!api().async_error) return {0, 0};
  ncclResult_t async = ncclSuccess;
  const ncclResult_t r = api().async_error(c->nccl, &async);
  return nccl_status(r != ncclSuccess ? r : async);
}

// Tears the communicator down; abort != 0 cancels outstanding operations (failure path). A
// communicator already aborted by a bounded wait only frees its handle.
extern "C" SparCudaStatus spar_b200_comm_destroy(void* comm, int abort) {
  if (!comm) return {0, 0};
  Comm* c = static_cast<Comm*>(comm);
  const ncclResult_t r = c->aborted ? ncclSuccess
                         : abort    ? api().abort(c->nccl)
                                    : api().destroy(c->nccl);
  delete c;  // the abort thread, if any, holds its own references
  return nccl_status(r);
}

// Deadline of the bounded waits on this communicator's collectives (seconds, > 0).
extern "C" SparCudaStatus spar_b200_comm_set_timeout(void* comm, double seconds) {
  if (!comm || !(seconds > 0.0)) return {1, static_cast<int>(cudaErrorInvalidValue)};
  static_cast<Comm*>(comm)->timeout_s = seconds;
  return {0, 0};
}

// Bounded wait for `stream` (see comm_wait): {0,0} when it finished, {3, ncclResult} after an
// asynchronous NCCL error or the deadline (the communicator is then aborted), {2, cudaError} for
// a CUDA error.
extern "C" SparCudaStatus spar_b200_comm_wait(void* comm, void* stream) {
  return comm_wait(comm, static_cast<cudaStream_t>(stream));
}
