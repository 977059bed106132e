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
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
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

}  // namespace

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
