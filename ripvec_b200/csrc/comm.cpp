// NCCL communicator of the row-sharded search: one rank per GPU, each holding a contiguous range
// of database rows, exchanges its per-shard top-k lists with one all-gather and merges them on
// the device (the multi-GPU search step; the reference ranks one in-memory matrix,
// crates/ripvec-core/src/index.rs:172-186).
//
// NCCL is opened with dlopen on first use (libnccl.so.2, the library torch and the system ship),
// so the library itself loads on hosts without NCCL; only these entry points need it.  The
// communicator is non-blocking: every wait on it (initialisation, the all-gather) polls with a
// host-side time limit, and a rank that never joins or stops answering ends the call with
// RV_E_COMM after the limit instead of hanging the caller; the communicator is then aborted
// and refuses further work.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "../../include/ripvec_b200.h"
#include "comm_impl.h"

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string why;
  bool ok = false;
};

const NcclApi& nccl() {
  static const NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      a.why = std::string("NCCL could not be loaded: ") + dlerror();
      return a;
    }
    bool all = true;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn) {
        all = false;
        a.why = std::string("NCCL symbol missing: ") + name;
      }
    };
    sym(a.get_unique_id, "ncclGetUniqueId");
    sym(a.init_rank_config, "ncclCommInitRankConfig");
    sym(a.all_gather, "ncclAllGather");
    sym(a.group_start, "ncclGroupStart");
    sym(a.group_end, "ncclGroupEnd");
    sym(a.get_async_error, "ncclCommGetAsyncError");
    sym(a.comm_destroy, "ncclCommDestroy");
    sym(a.comm_abort, "ncclCommAbort");
    sym(a.error_string, "ncclGetErrorString");
    a.ok = all;
    return a;
  }();
  return api;
}

std::string nccl_msg(const char* what, ncclResult_t r) {
  const NcclApi& a = nccl();
  return std::string(what) + ": " + (a.error_string ? a.error_string(r) : "NCCL error") + " (" +
         std::to_string(int(r)) + ")";
}

using Clock = std::chrono::steady_clock;

// Polls until the communicator leaves ncclInProgress (and, with a stream, until the stream's
// work has finished).  Returns RV_OK, or an error after an NCCL failure or timeout_ms.
int settle(rv_comm* c, cudaStream_t st, const char* what) {
  const NcclApi& a = nccl();
  const auto t0 = Clock::now();
  for (int spin = 0;; ++spin) {
    ncclResult_t r = ncclSuccess;
    if (a.get_async_error(c->comm, &r) != ncclSuccess) r = ncclInternalError;
    if (r != ncclSuccess && r != ncclInProgress) {
      c->err = nccl_msg(what, r);
      a.comm_abort(c->comm);
      c->broken = true;
      return RV_E_COMM;
    }
    if (r == ncclSuccess) {
      if (!st) return RV_OK;
      const cudaError_t q = cudaStreamQuery(st);
      if (q == cudaSuccess) return RV_OK;
      if (q != cudaErrorNotReady) {
        c->err = std::string(what) + ": " + cudaGetErrorString(q);
        return RV_E_CUDA;
      }
    }
    const double ms = std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    if (ms > c->timeout_ms) {
      c->err = std::string(what) + ": no completion within " + std::to_string(c->timeout_ms) +
               " ms (a rank did not take part); the communicator is aborted";
      a.comm_abort(c->comm);
      c->broken = true;
      return RV_E_COMM;
    }
    if (spin < 2000)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

struct DeviceScope {
  int prev = -1;
  bool ok = true;
  explicit DeviceScope(int d) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != d) ok = cudaSetDevice(d) == cudaSuccess;
  }
  ~DeviceScope() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

int rv_comm_allgather_lists(rv_comm* c, const int64_t* idx, const double* score, size_t count,
                            int64_t** gathered_idx, double** gathered_score, cudaStream_t st) {
  if (c->broken) {
    c->err = "the communicator was aborted by an earlier failure";
    return RV_E_COMM;
  }
  const size_t total = count * size_t(c->world);
  if (!c->gi.reserve(total) || !c->gs.reserve(total)) {
    c->err = "all-gather buffers could not be allocated";
    return RV_E_NOMEM;
  }
  const NcclApi& a = nccl();
  ncclResult_t r = a.group_start();
  if (r == ncclSuccess || r == ncclInProgress) r = a.all_gather(idx, c->gi.p, count, ncclInt64, c->comm, st);
  if (r == ncclSuccess || r == ncclInProgress) r = a.all_gather(score, c->gs.p, count, ncclFloat64, c->comm, st);
  const ncclResult_t e = a.group_end();
  if (r == ncclSuccess || r == ncclInProgress) r = e;
  if (r != ncclSuccess && r != ncclInProgress) {
    c->err = nccl_msg("ncclAllGather", r);
    return RV_E_COMM;
  }
  const int rc = settle(c, st, "all-gather of the per-shard top-k lists");
  if (rc) return rc;
  *gathered_idx = c->gi.p;
  *gathered_score = c->gs.p;
  return RV_OK;
}

extern "C" {

int rv_comm_get_unique_id(uint8_t* id) {
  if (!id) return RV_E_INVALID;
  const NcclApi& a = nccl();
  if (!a.ok) return RV_E_COMM;
  ncclUniqueId u;
  if (a.get_unique_id(&u) != ncclSuccess) return RV_E_COMM;
  static_assert(sizeof(u) == RV_COMM_ID_BYTES, "NCCL unique id size");
  std::memcpy(id, &u, sizeof(u));
  return RV_OK;
}

int rv_comm_create(int device, const uint8_t* id, int32_t rank, int32_t world, int32_t timeout_ms,
                   rv_comm** out) {
  if (!out) return RV_E_INVALID;
  *out = nullptr;
  if (!id || world < 1 || rank < 0 || rank >= world || timeout_ms <= 0) return RV_E_INVALID;
  const NcclApi& a = nccl();
  if (!a.ok) return RV_E_COMM;
  DeviceScope g(device);
  if (!g.ok) return RV_E_CUDA;
  rv_comm* c = new rv_comm();
  c->device = device;
  c->rank = rank;
  c->world = world;
  c->timeout_ms = timeout_ms;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // every wait is polled with the time limit above
  ncclResult_t r = a.init_rank_config(&c->comm, world, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete c;
    return RV_E_COMM;
  }
  if (settle(c, nullptr, "communicator initialisation") != RV_OK) {
    delete c;  // aborted inside settle
    return RV_E_COMM;
  }
  *out = c;
  return RV_OK;
}

void rv_comm_destroy(rv_comm* c) {
  if (!c) return;
  {
    DeviceScope g(c->device);
    if (!c->broken && c->comm) nccl().comm_destroy(c->comm);
    c->gi.release();
    c->gs.release();
  }
  delete c;
}

const char* rv_comm_last_error(const rv_comm* c) { return c ? c->err.c_str() : "null communicator"; }
int rv_comm_rank(const rv_comm* c) { return c ? c->rank : -1; }
int rv_comm_world(const rv_comm* c) { return c ? c->world : 0; }

}  // extern "C"
