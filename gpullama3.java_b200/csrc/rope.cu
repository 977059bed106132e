// rope.cu - RoPE rotation of the new token's q/k followed by the KV append:
// the producers of the attention inputs (InferenceCore.java:82-100 on the CPU;
// ropeRotation + copyToCache, TransformerComputeKernelsLayered.java:129-139
// and :179-205, on the GPU).
//
// Frequencies follow RoPE.precomputeFreqsCis (RoPE.java:6-37):
//   freq_i = (float)(1 / theta^(2i/head_dim)),  angle = (float)pos * freq_i,
//   fcr = (float)cos(angle), fci = (float)sin(angle)   (double evaluation)
// with the configured theta (the reference GPU kernels hard-code 50000,
// 10000 or 1e6 instead: TransformerComputeKernelsLayered.java:184, :221,
// Qwen3Kernels.java:171).  The rotation uses explicitly rounded FP32 products
// and sums so no FMA changes the result.
#include "gla_common.cuh"
#include "gla_internal.h"
#include "gla_rope.cuh"

namespace gla {

__device__ __forceinline__ void rotate_pair(float* x, int i0, int i1, float fcr, float fci) {
  rope_rotate(x[i0], x[i1], fcr, fci, &x[i0], &x[i1]);
}

__global__ void rope_append_f32_kernel(float* __restrict__ q, float* __restrict__ k,
                                       const float* __restrict__ v, float* __restrict__ key_cache,
                                       float* __restrict__ value_cache, int32_t n_heads,
                                       int32_t n_kv_heads, int32_t head_dim,
                                       const int32_t* __restrict__ position_holder, double theta,
                                       int32_t style) {
  // programmatic dependent launch: start behind the preceding kernel, touch
  // memory only once it has finished, and let the following decode start
  // (its early reads never cover the row or the q written here)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int pos = position_holder[0];
  const int half = head_dim / 2;
  const int64_t kv_dim = (int64_t)n_kv_heads * head_dim;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int n_pairs = n_heads * half;
  if (idx < n_pairs) {
    const int h = idx / half, ic = idx - h * half;
    float fcr, fci;
    rope_cos_sin(pos, ic, head_dim, theta, &fcr, &fci);
    int i0, i1;
    rope_pair(style, ic, head_dim, &i0, &i1);
    i0 += h * head_dim;
    i1 += h * head_dim;
    rotate_pair(q, i0, i1, fcr, fci);
    if (h < n_kv_heads) {
      rotate_pair(k, i0, i1, fcr, fci);
      key_cache[(int64_t)pos * kv_dim + i0] = k[i0];
      key_cache[(int64_t)pos * kv_dim + i1] = k[i1];
      value_cache[(int64_t)pos * kv_dim + i0] = v[i0];
      value_cache[(int64_t)pos * kv_dim + i1] = v[i1];
    }
  }
}

int launch_rope_append_f32(float* q, float* k, const float* v, float* key_cache,
                           float* value_cache, int32_t n_heads, int32_t n_kv_heads,
                           int32_t head_dim, const int32_t* position_holder, float theta,
                           int32_t rope_style, cudaStream_t stream, std::string* err) {
  const int n_pairs = n_heads * (head_dim / 2);
  const int threads = 128;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((n_pairs + threads - 1) / threads);
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, rope_append_f32_kernel, q, k, v, key_cache,
                                     value_cache, n_heads, n_kv_heads, head_dim, position_holder,
                                     (double)theta, rope_style);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("rope launch failed: ") + cudaGetErrorString(e);
    return GLA_ERR_CUDA;
  }
  return GLA_OK;
}

}  // namespace gla
