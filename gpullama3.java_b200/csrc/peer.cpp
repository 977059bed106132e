// peer.cpp - CUDA IPC setup of the sharded-decode peer exchange.
#include <cuda_runtime.h>

#include <cstring>
#include <vector>

#include "gla_comm.h"
#include "gla_peer.h"
#include "gla_xch.h"
#include "gpullama_attn.h"

namespace gla {

namespace {

// All-gathers one float per rank (1.0 = yes) and returns whether every rank
// said yes.  The float buffers live on the device; NCCL is stream ordered.
int agree(Comm& comm, bool mine, cudaStream_t stream, bool* all, std::string* err) {
  float* d = nullptr;
  const int n = comm.nranks;
  if (cudaMalloc(&d, sizeof(float) * (n + 1)) != cudaSuccess) {
    *err = "peer exchange: cudaMalloc failed";
    return GLA_ERR_OUT_OF_MEMORY;
  }
  const float v = mine ? 1.f : 0.f;
  std::vector<float> h(n);
  int rc = GLA_OK;
  if (cudaMemcpyAsync(d, &v, sizeof v, cudaMemcpyHostToDevice, stream) != cudaSuccess) {
    *err = "peer exchange: copy failed";
    rc = GLA_ERR_CUDA;
  }
  if (rc == GLA_OK) rc = comm.all_gather(d, d + 1, 1, stream, err);
  if (rc == GLA_OK &&
      cudaMemcpyAsync(h.data(), d + 1, sizeof(float) * n, cudaMemcpyDeviceToHost, stream) !=
          cudaSuccess) {
    *err = "peer exchange: copy failed";
    rc = GLA_ERR_CUDA;
  }
  if (rc == GLA_OK) rc = comm.wait(stream, err);
  cudaFree(d);
  bool ok = true;
  for (float x : h) ok = ok && x == 1.f;
  *all = ok;
  return rc;
}

}  // namespace

int PeerExchange::setup(Comm& comm, cudaStream_t stream, std::string* err) {
  teardown();
  const int n = comm.nranks, me = comm.rank;
  world = n;
  rank = me;
  // 1. own buffer and its IPC handle
  bool ok = n >= 2 && n <= kXchMaxWorld;
  cudaIpcMemHandle_t handle{};
  if (ok) ok = cudaMalloc(&local_, xch_bytes()) == cudaSuccess;
  if (ok) ok = cudaMemset(local_, 0, xch_bytes()) == cudaSuccess;
  if (ok) ok = cudaIpcGetMemHandle(&handle, local_) == cudaSuccess;
  cudaGetLastError();
  // 2. all-gather (handle bytes, ok) as 17 floats per rank
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle is 64 bytes");
  constexpr int kF = 17;
  std::vector<float> send(kF, 0.f), recv((size_t)kF * (n > 0 ? n : 1));
  std::memcpy(send.data(), &handle, sizeof handle);
  send[16] = ok ? 1.f : 0.f;
  float* d = nullptr;
  if (cudaMalloc(&d, sizeof(float) * kF * (n + 1)) != cudaSuccess) {
    teardown();
    *err = "peer exchange: cudaMalloc failed";
    return GLA_ERR_OUT_OF_MEMORY;
  }
  int rc = GLA_OK;
  if (cudaMemcpyAsync(d, send.data(), sizeof(float) * kF, cudaMemcpyHostToDevice, stream) !=
      cudaSuccess) {
    *err = "peer exchange: copy failed";
    rc = GLA_ERR_CUDA;
  }
  if (rc == GLA_OK) rc = comm.all_gather(d, d + kF, kF, stream, err);
  if (rc == GLA_OK &&
      cudaMemcpyAsync(recv.data(), d + kF, sizeof(float) * kF * n, cudaMemcpyDeviceToHost,
                      stream) != cudaSuccess) {
    *err = "peer exchange: copy failed";
    rc = GLA_ERR_CUDA;
  }
  if (rc == GLA_OK) rc = comm.wait(stream, err);
  cudaFree(d);
  if (rc != GLA_OK) {
    teardown();
    return rc;
  }
  bool all = true;
  for (int r = 0; r < n; ++r) all = all && recv[(size_t)r * kF + 16] == 1.f;
  // 3. map every peer's buffer
  std::vector<uint64_t> bases(n, 0);
  bool mapped = all;
  for (int r = 0; r < n && mapped; ++r) {
    if (r == me) {
      bases[r] = reinterpret_cast<uint64_t>(local_);
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, recv.data() + (size_t)r * kF, sizeof h);
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      mapped = false;
      break;
    }
    opened_.push_back(p);
    bases[r] = reinterpret_cast<uint64_t>(p);
  }
  if (mapped) {
    mapped = cudaMalloc(&d_bases_, sizeof(uint64_t) * n) == cudaSuccess &&
             cudaMemcpy(d_bases_, bases.data(), sizeof(uint64_t) * n, cudaMemcpyHostToDevice) ==
                 cudaSuccess;
    cudaGetLastError();
  }
  // 4. enabled only if every rank mapped every peer
  bool every = false;
  rc = agree(comm, mapped, stream, &every, err);
  if (rc != GLA_OK || !every) {
    teardown();
    world = n;
    rank = me;
    return rc;
  }
  active_ = true;
  return GLA_OK;
}

int PeerExchange::setup_loopback(int n, std::string* err) {
  teardown();
  if (n < 2 || n > kXchMaxWorld) {
    *err = "loopback world must be in [2, 8]";
    return GLA_ERR_INVALID_ARG;
  }
  std::vector<uint64_t> bases(n, 0);
  for (int r = 0; r < n; ++r) {
    void* p = nullptr;
    if (cudaMalloc(&p, xch_bytes()) != cudaSuccess || cudaMemset(p, 0, xch_bytes()) != cudaSuccess) {
      cudaGetLastError();
      if (p) cudaFree(p);
      teardown();
      *err = "loopback exchange allocation failed";
      return GLA_ERR_OUT_OF_MEMORY;
    }
    if (r == 0) local_ = p;
    else owned_.push_back(p);
    bases[r] = reinterpret_cast<uint64_t>(p);
  }
  if (cudaMalloc(&d_bases_, sizeof(uint64_t) * n) != cudaSuccess ||
      cudaMemcpy(d_bases_, bases.data(), sizeof(uint64_t) * n, cudaMemcpyHostToDevice) !=
          cudaSuccess) {
    cudaGetLastError();
    teardown();
    *err = "loopback exchange allocation failed";
    return GLA_ERR_OUT_OF_MEMORY;
  }
  world = n;
  rank = 0;
  active_ = true;
  loopback_ = true;
  return GLA_OK;
}

int PeerExchange::reset(cudaStream_t stream, std::string* err) {
  if (!local_) return GLA_OK;
  if (cudaMemsetAsync(local_, 0, xch_bytes(), stream) != cudaSuccess) {
    cudaGetLastError();
    *err = "peer exchange: reset failed";
    return GLA_ERR_CUDA;
  }
  return GLA_OK;
}

void PeerExchange::teardown() {
  for (void* p : opened_) cudaIpcCloseMemHandle(p);
  opened_.clear();
  for (void* p : owned_) cudaFree(p);
  owned_.clear();
  loopback_ = false;
  if (d_bases_) cudaFree(d_bases_);
  d_bases_ = nullptr;
  if (local_) cudaFree(local_);
  local_ = nullptr;
  active_ = false;
  cudaGetLastError();
}

}  // namespace gla
