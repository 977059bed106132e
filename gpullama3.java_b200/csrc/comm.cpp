// comm.cpp - NCCL all-gather for KV-sequence-sharded decode (dlopen binding)
// with a host watchdog (non-blocking communicator, polled with deadlines).
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "gpullama_attn.h"
#include "gla_comm.h"

namespace gla {

namespace {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int,
                                        ncclConfig_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_finalize)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string load_error;
};

template <class F>
void bind(void* h, F*& fn, const char* name) {
  fn = reinterpret_cast<F*>(dlsym(h, name));
}

NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    // prefer a copy that is already loaded in the process
    a.handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!a.handle) a.handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!a.handle) a.handle = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!a.handle) {
      const char* e = dlerror();
      a.load_error = std::string("cannot load libnccl: ") + (e ? e : "?");
      return;
    }
    bind(a.handle, a.get_unique_id, "ncclGetUniqueId");
    bind(a.handle, a.comm_init_rank_config, "ncclCommInitRankConfig");
    bind(a.handle, a.all_gather, "ncclAllGather");
    bind(a.handle, a.comm_finalize, "ncclCommFinalize");
    bind(a.handle, a.comm_destroy, "ncclCommDestroy");
    bind(a.handle, a.comm_abort, "ncclCommAbort");
    bind(a.handle, a.get_async_error, "ncclCommGetAsyncError");
    bind(a.handle, a.error_string, "ncclGetErrorString");
    if (!a.get_unique_id || !a.comm_init_rank_config || !a.all_gather || !a.comm_finalize ||
        !a.comm_destroy || !a.comm_abort || !a.get_async_error || !a.error_string) {
      a.load_error = "libnccl lacks a required symbol";
      a.handle = nullptr;
    }
  });
  return a;
}

int nccl_fail(ncclResult_t r, const char* what, std::string* err) {
  NcclApi& a = api();
  *err = std::string(what) + ": " + (a.error_string ? a.error_string(r) : "nccl error");
  return GLA_ERR_COMM;
}

using Clock = std::chrono::steady_clock;

Clock::time_point deadline_after(int ms) { return Clock::now() + std::chrono::milliseconds(ms); }

// Short sleep between polls once the first few polls have failed.
void backoff(int& spins) {
  if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
}

}  // namespace

int Comm::unique_id_size() { return (int)sizeof(ncclUniqueId); }

int Comm::get_unique_id(void* out, std::string* err) {
  NcclApi& a = api();
  if (!a.handle) {
    *err = a.load_error;
    return GLA_ERR_COMM;
  }
  ncclUniqueId id;
  ncclResult_t r = a.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId", err);
  std::memcpy(out, &id, sizeof id);
  return GLA_OK;
}

// Polls the communicator's asynchronous state until the last operation has
// left ncclInProgress; past the deadline the communicator is aborted.
int Comm::poll_async(const char* what, std::string* err) {
  NcclApi& a = api();
  const auto end = deadline_after(timeout_ms);
  int spins = 0;
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = a.get_async_error(static_cast<ncclComm_t>(comm_), &st);
    if (r != ncclSuccess) {
      abort();
      return nccl_fail(r, what, err);
    }
    if (st == ncclSuccess) return GLA_OK;
    if (st != ncclInProgress) {
      abort();
      return nccl_fail(st, what, err);
    }
    if (Clock::now() > end) {
      abort();
      *err = std::string(what) + ": no progress within the communicator timeout "
             "(a rank did not take part); communicator aborted";
      return GLA_ERR_TIMEOUT;
    }
    backoff(spins);
  }
}

int Comm::init(int n, int r, const void* unique_id, std::string* err) {
  NcclApi& a = api();
  if (!a.handle) {
    *err = a.load_error;
    return GLA_ERR_COMM;
  }
  destroy();
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof id);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t c = nullptr;
  ncclResult_t res = a.comm_init_rank_config(&c, n, id, r, &cfg);
  if (res != ncclSuccess && res != ncclInProgress) {
    if (c) a.comm_abort(c);
    return nccl_fail(res, "ncclCommInitRankConfig", err);
  }
  comm_ = c;
  nranks = n;
  rank = r;
  int rc = poll_async("ncclCommInitRankConfig", err);
  if (rc != GLA_OK) return rc;
  if (cudaMalloc(&scratch_, sizeof(float) * (n + 1)) != cudaSuccess) {
    cudaGetLastError();
    scratch_ = nullptr;
    destroy();
    *err = "communicator scratch allocation failed";
    return GLA_ERR_OUT_OF_MEMORY;
  }
  return GLA_OK;
}

int Comm::all_gather(const float* send, float* recv, size_t count, cudaStream_t stream,
                     std::string* err) {
  NcclApi& a = api();
  if (!comm_) {
    *err = "communicator not initialised";
    return GLA_ERR_COMM;
  }
  ncclResult_t r =
      a.all_gather(send, recv, count, ncclFloat32, static_cast<ncclComm_t>(comm_), stream);
  if (r != ncclSuccess && r != ncclInProgress) {
    abort();
    return nccl_fail(r, "ncclAllGather", err);
  }
  return r == ncclInProgress ? poll_async("ncclAllGather", err) : GLA_OK;
}

int Comm::wait(cudaStream_t stream, std::string* err) {
  if (!comm_) {
    cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
      *err = std::string("cudaStreamSynchronize: ") + cudaGetErrorString(e);
      return GLA_ERR_CUDA;
    }
    return GLA_OK;
  }
  NcclApi& a = api();
  const auto end = deadline_after(timeout_ms);
  int spins = 0;
  for (;;) {
    cudaError_t e = cudaStreamQuery(stream);
    if (e == cudaSuccess) return GLA_OK;
    if (e != cudaErrorNotReady) {
      *err = std::string("cudaStreamQuery: ") + cudaGetErrorString(e);
      return GLA_ERR_CUDA;
    }
    ncclResult_t st = ncclSuccess;
    if (a.get_async_error(static_cast<ncclComm_t>(comm_), &st) != ncclSuccess ||
        (st != ncclSuccess && st != ncclInProgress)) {
      abort();
      cudaStreamSynchronize(stream);  // the aborted collective has exited
      cudaGetLastError();
      *err = "a collective on the stream failed; communicator aborted";
      return GLA_ERR_COMM;
    }
    if (Clock::now() > end) {
      abort();
      cudaStreamSynchronize(stream);
      cudaGetLastError();
      *err = "the stream did not drain within the communicator timeout (a collective waits "
             "for a rank that did not take part); communicator aborted";
      return GLA_ERR_TIMEOUT;
    }
    backoff(spins);
  }
}

int Comm::barrier(cudaStream_t stream, std::string* err) {
  if (!comm_) {
    *err = "communicator not initialised";
    return GLA_ERR_COMM;
  }
  int rc = all_gather(scratch_, scratch_ + 1, 1, stream, err);
  if (rc != GLA_OK) return rc;
  return wait(stream, err);
}

void Comm::abort() {
  if (comm_) {
    NcclApi& a = api();
    a.comm_abort(static_cast<ncclComm_t>(comm_));
    comm_ = nullptr;
  }
  if (scratch_) cudaFree(scratch_);
  scratch_ = nullptr;
  cudaGetLastError();
}

void Comm::destroy() {
  if (comm_) {
    NcclApi& a = api();
    std::string err;
    ncclResult_t r = a.comm_finalize(static_cast<ncclComm_t>(comm_));
    if ((r == ncclSuccess || r == ncclInProgress) && poll_async("ncclCommFinalize", &err) == GLA_OK)
      a.comm_destroy(static_cast<ncclComm_t>(comm_));
    else
      abort();
    comm_ = nullptr;
  }
  if (scratch_) cudaFree(scratch_);
  scratch_ = nullptr;
  nranks = 0;
  rank = 0;
}

}  // namespace gla
