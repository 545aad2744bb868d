// tp.cpp — the head-sharding communicator of b200_tp.h: NCCL, loaded at run time, with
// every wait on the group bounded (non-blocking communicator + polling of its
// asynchronous error, abort on timeout).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "../../include/b200_tp.h"

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclCommFinalize) finalize = nullptr;
  decltype(&ncclCommCount) count = nullptr;
  decltype(&ncclCommUserRank) user_rank = nullptr;
  bool ok = false;
};

// The NCCL already mapped into the process (a host framework's) when there is one, so the
// communicator and the framework share one library; otherwise the system's.
const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    auto sym = [h](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      return fn != nullptr;
    };
    api.ok = sym(api.get_unique_id, "ncclGetUniqueId") &&
             sym(api.init_rank_config, "ncclCommInitRankConfig") &&
             sym(api.async_error, "ncclCommGetAsyncError") &&
             sym(api.all_reduce, "ncclAllReduce") && sym(api.abort, "ncclCommAbort") &&
             sym(api.destroy, "ncclCommDestroy") && sym(api.finalize, "ncclCommFinalize") &&
             sym(api.count, "ncclCommCount") &&
             sym(api.user_rank, "ncclCommUserRank");
  });
  return api;
}

using Clock = std::chrono::steady_clock;

}  // namespace

struct b200_tp_comm {
  ncclComm_t comm = nullptr;
  bool owned = true;    // made by b200_tp_init (destroyed with the handle)
  bool aborted = false;
  uint32_t timeout_ms = 60000;
  int rank = 0, size = 1;
};

namespace {

// A failed wait aborts a communicator this library made (which also releases it); one
// borrowed from the caller is left to its owner.
void fail(b200_tp_comm* c) {
  if (c->owned && !c->aborted) nccl().abort(c->comm);
  c->aborted = true;
}

// Polls the communicator's asynchronous state until it leaves ncclInProgress, the
// deadline passes, or it reports an error.
int settle(b200_tp_comm* c, Clock::time_point deadline) {
  const NcclApi& api = nccl();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    if (api.async_error(c->comm, &st) != ncclSuccess) st = ncclSystemError;
    if (st == ncclSuccess) return B200_OK;
    if (st != ncclInProgress || Clock::now() > deadline) {
      fail(c);
      return st == ncclInProgress ? B200_ERR_DEVICE_TIMEOUT : B200_ERR_CUDA;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

Clock::time_point deadline_of(const b200_tp_comm* c) {
  return Clock::now() + std::chrono::milliseconds(c->timeout_ms);
}

}  // namespace

extern "C" int b200_tp_unique_id(uint8_t id[B200_TP_ID_BYTES]) {
  if (!id) return B200_ERR_INVALID;
  static_assert(sizeof(ncclUniqueId) == B200_TP_ID_BYTES, "ncclUniqueId size");
  const NcclApi& api = nccl();
  if (!api.ok) return B200_ERR_UNSUPPORTED;
  ncclUniqueId uid;
  if (api.get_unique_id(&uid) != ncclSuccess) return B200_ERR_CUDA;
  std::memcpy(id, &uid, sizeof(uid));
  return B200_OK;
}

extern "C" int b200_tp_init(b200_tp_comm** out, const uint8_t id[B200_TP_ID_BYTES],
                            int32_t nranks, int32_t rank, uint32_t timeout_ms) {
  if (!out || !id || nranks < 1 || rank < 0 || rank >= nranks) return B200_ERR_INVALID;
  *out = nullptr;
  const NcclApi& api = nccl();
  if (!api.ok) return B200_ERR_UNSUPPORTED;
  auto* c = new b200_tp_comm;
  c->timeout_ms = timeout_ms ? timeout_ms : 60000;
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // the join returns at once; settle() bounds the wait for the peers
  const auto deadline = deadline_of(c);
  const ncclResult_t r = api.init_rank_config(&c->comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (c->comm) api.abort(c->comm);
    delete c;
    return B200_ERR_CUDA;
  }
  const int rc = settle(c, deadline);
  if (rc != B200_OK) {  // settle() aborted (and so released) the communicator
    delete c;
    return rc;
  }
  c->rank = rank;
  c->size = nranks;
  *out = c;
  return B200_OK;
}

extern "C" int b200_tp_init_from_nccl(b200_tp_comm** out, void* nccl_comm, uint32_t timeout_ms) {
  if (!out || !nccl_comm) return B200_ERR_INVALID;
  *out = nullptr;
  const NcclApi& api = nccl();
  if (!api.ok) return B200_ERR_UNSUPPORTED;
  auto* c = new b200_tp_comm;
  c->comm = static_cast<ncclComm_t>(nccl_comm);
  c->owned = false;
  c->timeout_ms = timeout_ms ? timeout_ms : 60000;
  if (api.count(c->comm, &c->size) != ncclSuccess ||
      api.user_rank(c->comm, &c->rank) != ncclSuccess) {
    delete c;
    return B200_ERR_CUDA;
  }
  *out = c;
  return B200_OK;
}

extern "C" int b200_tp_rank(const b200_tp_comm* c) { return c ? c->rank : B200_ERR_INVALID; }
extern "C" int b200_tp_size(const b200_tp_comm* c) { return c ? c->size : B200_ERR_INVALID; }

extern "C" int b200_tp_out_proj_allreduce(b200_tp_comm* c, void* partial, size_t n,
                                          int32_t dtype, b200_stream_t stream) {
  if (!c || c->aborted) return B200_ERR_INVALID;
  if (dtype != B200_DTYPE_BF16 && dtype != B200_DTYPE_F32) return B200_ERR_INVALID;
  if (n == 0) return B200_OK;
  if (!partial) return B200_ERR_INVALID;
  const NcclApi& api = nccl();
  const ncclDataType_t t = dtype == B200_DTYPE_BF16 ? ncclBfloat16 : ncclFloat32;
  const ncclResult_t r =
      api.all_reduce(partial, partial, n, t, ncclSum, c->comm, static_cast<cudaStream_t>(stream));
  if (r == ncclSuccess) return B200_OK;
  if (r == ncclInProgress) return settle(c, deadline_of(c));  // enqueue finishing
  return B200_ERR_CUDA;
}

extern "C" int b200_tp_wait(b200_tp_comm* c, b200_stream_t stream) {
  if (!c || c->aborted) return B200_ERR_INVALID;
  const NcclApi& api = nccl();
  const auto deadline = deadline_of(c);
  auto s = static_cast<cudaStream_t>(stream);
  for (;;) {
    const cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) return B200_OK;
    if (q != cudaErrorNotReady) {
      fail(c);
      return B200_ERR_CUDA;
    }
    ncclResult_t st = ncclSuccess;
    api.async_error(c->comm, &st);
    if ((st != ncclSuccess && st != ncclInProgress) || Clock::now() > deadline) {
      fail(c);
      return st != ncclSuccess && st != ncclInProgress ? B200_ERR_CUDA : B200_ERR_DEVICE_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

extern "C" int b200_tp_destroy(b200_tp_comm* c) {
  if (!c) return B200_ERR_INVALID;
  const NcclApi& api = nccl();
  int rc = B200_OK;
  // An aborted communicator was released by ncclCommAbort.  A live one is finalised
  // first (flushes its work; non-blocking, so polled with the timeout), then destroyed.
  if (c->owned && c->comm && api.ok && !c->aborted) {
    const ncclResult_t f = api.finalize(c->comm);
    if (f != ncclSuccess && f != ncclInProgress) {
      fail(c);
      rc = B200_ERR_CUDA;
    } else if ((rc = settle(c, deadline_of(c))) == B200_OK) {
      if (api.destroy(c->comm) != ncclSuccess) rc = B200_ERR_CUDA;
    }
  }
  delete c;
  return rc;
}
