// debug.cu - test hooks of the C ABI (gla_debug_*): kernels that stand in for
// the caller's own device work around an attention call, so tests can check
// the library's ordering rules without a second program.
#include <cuda_runtime.h>

#include "gla_common.cuh"
#include "gla_internal.h"

namespace gla {

namespace {

// A caller's kernel that advances the position holder on the device (a
// layer plan whose position update is itself a kernel): launched with
// programmatic dependent launch, it releases its dependents at once, waits
// `delay_ns` (so a following decode's pre-wait work runs while the old
// position is still in place), then adds `delta`.
__global__ void advance_position_kernel(int32_t* position_holder, int32_t delta,
                                        unsigned long long delay_ns) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    const unsigned long long t0 = global_timer_ns();
    while (global_timer_ns() - t0 < delay_ns) {
    }
    position_holder[0] += delta;
  }
}

}  // namespace

int launch_advance_position(int32_t* position_holder, int32_t delta, int32_t delay_us,
                            cudaStream_t stream, std::string* err) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // the spin is bounded: at most 1 ms
  const unsigned long long ns = (unsigned long long)(delay_us < 0 ? 0 : delay_us > 1000 ? 1000 : delay_us) * 1000ull;
  cudaError_t e = cudaLaunchKernelEx(&cfg, advance_position_kernel, position_holder, delta, ns);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("advance_position launch failed: ") + cudaGetErrorString(e);
    return GLA_ERR_CUDA;
  }
  return GLA_OK;
}

}  // namespace gla
