// q8.cu - quantisation of K/V rows into the Q8 cache layout.
//
// Q8 cache (an addition: the reference keeps FP32 caches; its quantised
// weight type Q8_0, tensor/GGMLType.java:13, has the same block shape):
//   values  int8 [rows][kv_stride] for K and for V, kv head g at column g*hd;
//   scales  FP16 [rows][n_kv][8]: K block scales at [0, hd/32), V block
//           scales at [4, 4 + hd/32), the other halves 0.
// A block is 32 consecutive values x of one head row, quantised as GGML's
// Q8_0 reference quantiser does: d = amax / 127, id = d ? 1/d : 0,
// q = roundf(x * id) (half away from zero), d stored rounded to FP16; the
// value is read back as q * (float)d16.
//
// One warp per (row, kv head): lane j handles value j of every block, a
// shuffle reduction gives each block's amax.
#include <cuda_fp16.h>

#include "decode_kernel.cuh"
#include "gla_internal.h"
#include "gla_rope.cuh"

namespace gla {

namespace {

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// Quantises the nb blocks of one head row; returns the FP16 scale bits of
// block `lane` (lanes >= nb return 0).
__device__ __forceinline__ uint16_t quantize_head_row(const float* __restrict__ x,
                                                      int8_t* __restrict__ out, int nb, int lane) {
  uint16_t mine = 0;
  for (int b = 0; b < nb; ++b) {
    const float v = x[32 * b + lane];
    const float amax = warp_max(fabsf(v));
    const float d = amax / 127.0f;
    // d below ~1e-38 makes 1/d overflow; such a block's FP16 scale is 0 anyway
    const float r = 1.0f / d;
    const float id = (d != 0.0f && r < INFINITY) ? r : 0.0f;
    out[32 * b + lane] = (int8_t)roundf(__fmul_rn(v, id));
    if (lane == b) mine = __half_as_ushort(__float2half_rn(d));
  }
  return mine;
}

__global__ void quantize_q8_kernel(const float* __restrict__ k, const float* __restrict__ v,
                                   int64_t src_stride, int32_t n_rows, int32_t n_kv, int32_t hd,
                                   int8_t* __restrict__ kq, int8_t* __restrict__ vq,
                                   int64_t kv_stride, uint16_t* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int64_t item = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;  // (row, head)
  if (item >= (int64_t)n_rows * n_kv) return;
  const int64_t row = item / n_kv;
  const int g = (int)(item - row * n_kv);
  const int nb = hd / 32;
  const uint16_t ks = quantize_head_row(k + row * src_stride + (int64_t)g * hd,
                                        kq + row * kv_stride + (int64_t)g * hd, nb, lane);
  const uint16_t vs = quantize_head_row(v + row * src_stride + (int64_t)g * hd,
                                        vq + row * kv_stride + (int64_t)g * hd, nb, lane);
  // the row's 8 scale halves: K blocks from lanes 0..nb-1, V blocks at 4..
  uint16_t* srow = scales + item * kQ8ScaleHalves;
  if (lane < 4) {
    srow[lane] = lane < nb ? ks : (uint16_t)0;
    srow[4 + lane] = lane < nb ? vs : (uint16_t)0;
  }
}

// The new token: RoPE of q and k in place (the same helpers and rounding as
// the FP32 RoPE kernel), then k and v quantised into row `position` of a Q8
// cache.  One warp per head: warps [0, n_kv) rotate kv head g's k (through
// shared memory) and quantise k and v, warps [n_kv, n_kv + n_heads) rotate q.
// A position outside [0, context_length) writes nothing and latches
// GLA_ERR_INVALID_ARG in the status word.
__global__ void __launch_bounds__(128)
    rope_append_q8_kernel(float* __restrict__ q, float* __restrict__ k,
                          const float* __restrict__ v, int8_t* __restrict__ kq,
                          int8_t* __restrict__ vq, uint16_t* __restrict__ scales, int32_t n_heads,
                          int32_t n_kv, int32_t hd, const int32_t* __restrict__ position_holder,
                          int32_t context_length, double theta, int32_t style,
                          int32_t* __restrict__ status) {
  __shared__ float s_row[4][128];
  // programmatic dependent launch, as the FP32 RoPE kernel: memory only after
  // the preceding kernel, dependents released at once
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w = blockIdx.x * 4 + warp;
  if (w >= n_kv + n_heads) return;
  const int pos = position_holder[0];
  if (pos < 0 || pos >= context_length) {
    if (lane == 0) atomicCAS(status, 0, GLA_ERR_INVALID_ARG);
    return;
  }
  const bool is_k = w < n_kv;
  const int h = is_k ? w : w - n_kv;
  float* x = (is_k ? k : q) + (int64_t)h * hd;
  for (int ic = lane; ic < hd / 2; ic += 32) {
    float fcr, fci;
    rope_cos_sin(pos, ic, hd, theta, &fcr, &fci);
    int i0, i1;
    rope_pair(style, ic, hd, &i0, &i1);
    float o0, o1;
    rope_rotate(x[i0], x[i1], fcr, fci, &o0, &o1);
    x[i0] = o0;
    x[i1] = o1;
    if (is_k) {
      s_row[warp][i0] = o0;
      s_row[warp][i1] = o1;
    }
  }
  if (!is_k) return;
  __syncwarp();
  const int64_t row = (int64_t)pos * n_kv * hd + (int64_t)h * hd;
  const int nb = hd / 32;
  const uint16_t ks = quantize_head_row(s_row[warp], kq + row, nb, lane);
  const uint16_t vs = quantize_head_row(v + (int64_t)h * hd, vq + row, nb, lane);
  uint16_t* srow = scales + ((int64_t)pos * n_kv + h) * kQ8ScaleHalves;
  if (lane < 4) {
    srow[lane] = lane < nb ? ks : (uint16_t)0;
    srow[4 + lane] = lane < nb ? vs : (uint16_t)0;
  }
}

}  // namespace

int launch_rope_append_q8(float* q, float* k, const float* v, int8_t* kq, int8_t* vq,
                          uint16_t* scales, int32_t n_heads, int32_t n_kv, int32_t hd,
                          const int32_t* position_holder, int32_t context_length, float theta,
                          int32_t rope_style, int32_t* status, cudaStream_t stream,
                          std::string* err) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((n_kv + n_heads + 3) / 4);
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, rope_append_q8_kernel, q, k, v, kq, vq, scales, n_heads,
                                     n_kv, hd, position_holder, context_length, (double)theta,
                                     rope_style, status);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("rope/Q8 append launch failed: ") + cudaGetErrorString(e);
    return GLA_ERR_CUDA;
  }
  return GLA_OK;
}

int launch_quantize_q8(const float* k, const float* v, int64_t src_stride, int32_t n_rows,
                       int32_t n_kv, int32_t hd, int8_t* kq, int8_t* vq, int64_t kv_stride,
                       uint16_t* scales, cudaStream_t stream, std::string* err) {
  const int64_t threads = (int64_t)n_rows * n_kv * 32;
  const int64_t blocks = (threads + 255) / 256;
  if (blocks > INT32_MAX) {
    *err = "too many rows to quantise in one call";
    return GLA_ERR_INVALID_ARG;
  }
  quantize_q8_kernel<<<(unsigned)blocks, 256, 0, stream>>>(k, v, src_stride, n_rows, n_kv, hd, kq,
                                                           vq, kv_stride, scales);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("quantise launch failed: ") + cudaGetErrorString(e);
    return GLA_ERR_CUDA;
  }
  return GLA_OK;
}

}  // namespace gla
