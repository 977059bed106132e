// gla_comm.h - NCCL communicator of a context, bound at run time.
//
// libnccl is opened with dlopen (an already loaded copy first, e.g. the one
// PyTorch ships), so the library has no link-time NCCL dependency and a
// process never mixes two NCCL builds on one communicator.
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
  void destroy();
  bool active() const { return comm_ != nullptr; }

  int nranks = 0;
  int rank = 0;

 private:
  void* comm_ = nullptr;
};

}  // namespace gla
