// prefill.cu - causal prefill attention (tcgen05 / TMEM); placeholder until
// the tensor-core kernel lands.
#include "gla_common.cuh"
#include "gla_internal.h"

namespace gla {

int launch_prefill_f16(const uint16_t*, const uint16_t*, const uint16_t*, float*, int32_t,
                       int32_t, int32_t, int32_t, float, int32_t*, const DeviceInfo&,
                       cudaStream_t, std::string* err) {
  *err = "prefill kernel not built yet";
  return GLA_ERR_NOT_SUPPORTED;
}

}  // namespace gla
