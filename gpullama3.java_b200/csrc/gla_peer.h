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
  // Test hook: one process plays rank 0 of a `world`-rank exchange whose
  // other ranks' buffers are local allocations nobody else writes, so the
  // kernel's wait for their records runs out (bounded) and latches
  // GLA_ERR_TIMEOUT.
  int setup_loopback(int world, std::string* err);
  bool loopback() const { return loopback_; }
  // Zeroes this rank's buffer (records and epochs), stream ordered.  Only
  // between two barriers of every rank: no peer may be writing into it.
  int reset(cudaStream_t stream, std::string* err);
  // Closes the peers' mappings and frees this rank's buffer.  Only after a
  // barrier of every rank (no peer still stores into it), or after the
  // communicator was aborted.
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
  std::vector<void*> owned_;   // loopback: the stand-in peers' buffers (to free)
  bool loopback_ = false;
};

}  // namespace gla
