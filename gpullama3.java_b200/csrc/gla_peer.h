// gla_peer.h - the peer exchange buffers of KV-sequence-sharded decode.
//
// Set up once per communicator (collectively, after the NCCL communicator):
// every rank allocates one exchange buffer (layout in gla_xch.h), its CUDA
// IPC handle is all-gathered with NCCL, and every rank maps every other
// rank's buffer.  The exchange is used only if every rank succeeded (a
// second all-gather agrees on it), so all ranks take the same path.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace gla {

class Comm;

class PeerExchange {
 public:
  PeerExchange() = default;
  ~PeerExchange() { teardown(); }
  PeerExchange(const PeerExchange&) = delete;
  PeerExchange& operator=(const PeerExchange&) = delete;

  // Collective over `comm`; returns GLA_OK whether or not the exchange could
  // be enabled (active() says which), an error code only when the
  // collective itself failed.
  int setup(Comm& comm, cudaStream_t stream, std::string* err);
  void teardown();
  bool active() const { return active_; }

  const uint64_t* bases() const { return d_bases_; }  // device [world]
  char* local() const { return static_cast<char*>(local_); }
  int world = 0;
  int rank = 0;

 private:
  bool active_ = false;
  void* local_ = nullptr;
  uint64_t* d_bases_ = nullptr;
  std::vector<void*> opened_;  // peers' buffers mapped here (to close)
};

}  // namespace gla
