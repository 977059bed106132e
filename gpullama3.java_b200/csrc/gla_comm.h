// gla_comm.h - NCCL communicator of a context, bound at run time, with a host
// watchdog on every step that can wait for another rank.
//
// libnccl is opened with dlopen (an already loaded copy first, e.g. the one
// PyTorch ships), so the library has no link-time NCCL dependency and a
// process never mixes two NCCL builds on one communicator.
//
// The communicator is non-blocking (ncclConfig_t.blocking = 0): joining it,
// enqueueing a collective and waiting for the stream are polled on the host
// with a deadline (`timeout_ms`).  When a deadline passes - a rank never
// joined, or a collective waits for a rank that left - the communicator is
// aborted (ncclCommAbort ends its kernels), the call returns GLA_ERR_TIMEOUT
// and the context needs gla_comm_init again.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include <string>

namespace gla {

class Comm {
 public:
  Comm() = default;
  ~Comm() { destroy(); }
  Comm(const Comm&) = delete;
  Comm& operator=(const Comm&) = delete;

  static int unique_id_size();
  static int get_unique_id(void* out, std::string* err);

  int init(int nranks, int rank, const void* unique_id, std::string* err);
  // all-gather of `count` floats per rank, stream ordered
  int all_gather(const float* send, float* recv, size_t count, cudaStream_t stream,
                 std::string* err);
  // Collective: an all-gather of one value, then waits (bounded) until it
  // has completed on `stream`: every rank has reached this point.
  int barrier(cudaStream_t stream, std::string* err);
  // Waits (bounded) until `stream` has drained; a collective still waiting
  // for a rank at the deadline is ended by aborting the communicator.
  int wait(cudaStream_t stream, std::string* err);
  // Ends the communicator at once (its kernels in flight exit).
  void abort();
  void destroy();
  bool active() const { return comm_ != nullptr; }

  int nranks = 0;
  int rank = 0;
  int timeout_ms = 60000;  // host deadline of every bounded step

 private:
  int poll_async(const char* what, std::string* err);
  void* comm_ = nullptr;
  float* scratch_ = nullptr;  // barrier buffer: [1 + nranks] floats
};

}  // namespace gla
