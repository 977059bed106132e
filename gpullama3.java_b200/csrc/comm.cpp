// comm.cpp - NCCL all-gather for KV-sequence-sharded decode (dlopen binding).
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "gpullama_attn.h"
#include "gla_comm.h"

namespace gla {

namespace {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string load_error;
};

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
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(a.handle, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(a.handle, "ncclCommInitRank"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(a.handle, "ncclAllGather"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(a.handle, "ncclCommDestroy"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(a.handle, "ncclGetErrorString"));
    if (!a.get_unique_id || !a.comm_init_rank || !a.all_gather || !a.comm_destroy ||
        !a.error_string) {
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

int Comm::init(int n, int r, const void* unique_id, std::string* err) {
  NcclApi& a = api();
  if (!a.handle) {
    *err = a.load_error;
    return GLA_ERR_COMM;
  }
  destroy();
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof id);
  ncclComm_t c = nullptr;
  ncclResult_t res = a.comm_init_rank(&c, n, id, r);
  if (res != ncclSuccess) return nccl_fail(res, "ncclCommInitRank", err);
  comm_ = c;
  nranks = n;
  rank = r;
  return GLA_OK;
}

int Comm::all_gather(const float* send, float* recv, size_t count, cudaStream_t stream,
                     std::string* err) {
  NcclApi& a = api();
  if (!comm_) {
    *err = "communicator not initialised";
    return GLA_ERR_COMM;
  }
  ncclResult_t r = a.all_gather(send, recv, count, ncclFloat32, static_cast<ncclComm_t>(comm_), stream);
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather", err);
  return GLA_OK;
}

void Comm::destroy() {
  if (comm_) {
    NcclApi& a = api();
    if (a.comm_destroy) a.comm_destroy(static_cast<ncclComm_t>(comm_));
    comm_ = nullptr;
  }
  nranks = 0;
  rank = 0;
}

}  // namespace gla
