// gla_rope.cuh - RoPE arithmetic shared by the RoPE+append kernel and the
// fused RoPE+append+attention decode, so both produce the same bits.
//
// Frequencies follow RoPE.precomputeFreqsCis (RoPE.java:6-37):
//   freq_i = (float)(1 / theta^(2i/head_dim)),  angle = (float)pos * freq_i,
//   fcr = (float)cos(angle), fci = (float)sin(angle)   (double evaluation);
// the rotation uses explicitly rounded FP32 products and sums so no FMA
// changes the result.
#pragma once

#include "gla_common.cuh"

namespace gla {

__device__ __forceinline__ void rope_cos_sin(int pos, int ic, int head_dim, double theta,
                                             float* fcr, float* fci) {
  const float freq = (float)(1.0 / pow(theta, (double)(2 * ic) / (double)head_dim));
  const float ang = __fmul_rn((float)pos, freq);
  *fcr = (float)cos((double)ang);
  *fci = (float)sin((double)ang);
}

// Elements (i0, i1) of pair ic inside a head: adjacent (interleaved, Llama)
// or half a head apart (NeoX: Qwen, Phi-3).
__device__ __forceinline__ void rope_pair(int style, int ic, int head_dim, int* i0, int* i1) {
  if (style == GLA_ROPE_INTERLEAVED) {
    *i0 = 2 * ic;
    *i1 = *i0 + 1;
  } else {
    *i0 = ic;
    *i1 = ic + head_dim / 2;
  }
}

__device__ __forceinline__ void rope_rotate(float v0, float v1, float fcr, float fci, float* o0,
                                            float* o1) {
  *o0 = __fsub_rn(__fmul_rn(v0, fcr), __fmul_rn(v1, fci));
  *o1 = __fadd_rn(__fmul_rn(v0, fci), __fmul_rn(v1, fcr));
}

}  // namespace gla
