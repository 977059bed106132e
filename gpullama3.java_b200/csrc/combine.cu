// combine.cu - log-sum-exp merge of per-shard attention records.
//
// A record set holds, per q head, (o normalised, m, l) of one KV shard
// (layout [n_heads][head_dim + 2]; see gla_decode_partial_*).  Merging the
// shards of one sequence gives exactly the unsharded softmax:
//     M = max_i m_i,  w_i = l_i exp(m_i - M),  xb = sum_i w_i o_i / sum_i w_i.
#include "gla_common.cuh"
#include "gla_internal.h"

namespace gla {

__global__ void lse_combine_kernel(const float* __restrict__ parts, int32_t n_parts,
                                   int32_t n_heads, int32_t head_dim, float* __restrict__ xb) {
  const int h = blockIdx.x;
  const int64_t rec = (int64_t)head_dim + 2;
  const int64_t set = (int64_t)n_heads * rec;
  float M = -INFINITY;
  for (int i = 0; i < n_parts; ++i) {
    const float* r = parts + i * set + h * rec;
    if (r[head_dim + 1] > 0.f) M = fmaxf(M, r[head_dim]);
  }
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float O = 0.f, L = 0.f;
    if (M != -INFINITY) {
      for (int i = 0; i < n_parts; ++i) {
        const float* r = parts + i * set + h * rec;
        const float l = r[head_dim + 1];
        if (l > 0.f) {
          const float w = l * __expf(r[head_dim] - M);
          O += w * r[d];
          L += w;
        }
      }
    }
    xb[(int64_t)h * head_dim + d] = L > 0.f ? O / L : 0.f;
  }
}

int launch_lse_combine(const float* parts, int32_t n_parts, int32_t n_heads, int32_t head_dim,
                       float* xb, cudaStream_t stream, std::string* err) {
  const int threads = head_dim >= 128 ? 128 : (head_dim + 31) / 32 * 32;
  lse_combine_kernel<<<n_heads, threads, 0, stream>>>(parts, n_parts, n_heads, head_dim, xb);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("combine launch failed: ") + cudaGetErrorString(e);
    return GLA_ERR_CUDA;
  }
  return GLA_OK;
}

}  // namespace gla
