// ingest.cu - batched prompt ingestion for one layer: L new positions at once.
//
// The reference ingests a prompt one position at a time
// (InferenceEngine.java:88-99 on the CPU, :309-327 on the GPU): every
// position runs InferenceCore.forwardJava's RoPE (:82-94 Llama, :210-225
// Qwen/Phi), KV append (:99-100) and attention block (:105-144).  Given the
// q/k/v rows of L consecutive positions (a batched QKV projection), this
// file does the same for all of them in two launches:
//
//   1. ingest_prep_kernel - one CTA per new row: the row's cos/sin pairs
//      (RoPE.java:6-37 formula, double evaluation) once into shared memory,
//      q/k in units of 4 rotation pairs (two float4 loads each), then the
//      rotated k and the v row into the layer cache at row
//      start_pos + i (FP32 or FP16), and FP16 copies of the rotated q (and,
//      for an FP32 cache, of k and v) for the tensor cores.  q/k/v are only
//      read: the reference's in-place rotation of state.q/state.k is an
//      intermediate nothing reads after the attention block.  For an FP32
//      cache with start_pos > 0, convert_rows_kernel first copies the cached
//      prefix rows 0..start_pos-1 to the FP16 workspace.
//   2. the tcgen05 prefill kernel (prefill.cu) with a query offset: row i
//      attends to key rows 0..start_pos+i, reading the FP16 cache directly or
//      the FP16 workspace.
//
// Every q/k element is rotated by the same explicitly rounded products as the
// single-position RoPE kernel (rope.cu), so the cache rows are identical to
// the ones L calls of gla_rope_append_f32 would write.
#include <cuda_fp16.h>

#include "gla_common.cuh"
#include "gla_internal.h"
#include "gla_rope.cuh"

namespace gla {

namespace {

constexpr int kPrepThreads = 256;
constexpr int kU = 2;        // q and k units a thread loads per round
constexpr int kUV = 2 * kU;  // v float4s a thread loads per round (kv_dim/4 = 2 k units)

// A unit is 8 elements of one head holding the 4 rotation pairs ic = 4j..4j+3:
// interleaved pairs (2ic, 2ic+1) are elements 8j..8j+7, NeoX pairs
// (ic, ic+hd/2) are elements 4j..4j+3 and hd/2+4j..hd/2+4j+3.  Both halves
// are float4 loads (head_dim/2 is a multiple of 4 for head_dim 64/96/128).
template <int HD>
__device__ __forceinline__ void unit_offsets(int style, int j, int* o0, int* o1) {
  if (style == GLA_ROPE_INTERLEAVED) {
    *o0 = 8 * j;
    *o1 = 8 * j + 4;
  } else {
    *o0 = 4 * j;
    *o1 = HD / 2 + 4 * j;
  }
}

__device__ __forceinline__ void rotate_unit(int style, float4& a, float4& b, float4 c, float4 s) {
  if (style == GLA_ROPE_INTERLEAVED) {
    rope_rotate(a.x, a.y, c.x, s.x, &a.x, &a.y);
    rope_rotate(a.z, a.w, c.y, s.y, &a.z, &a.w);
    rope_rotate(b.x, b.y, c.z, s.z, &b.x, &b.y);
    rope_rotate(b.z, b.w, c.w, s.w, &b.z, &b.w);
  } else {
    rope_rotate(a.x, b.x, c.x, s.x, &a.x, &b.x);
    rope_rotate(a.y, b.y, c.y, s.y, &a.y, &b.y);
    rope_rotate(a.z, b.z, c.z, s.z, &a.z, &b.z);
    rope_rotate(a.w, b.w, c.w, s.w, &a.w, &b.w);
  }
}

__device__ __forceinline__ void store_h4(__half* p, float4 x) {
  const __half2 lo = __floats2half2_rn(x.x, x.y), hi = __floats2half2_rn(x.z, x.w);
  *reinterpret_cast<uint2*>(p) =
      make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

// One CTA per new row.  Every thread first issues the loads of its q and k
// units and v float4s of the round (one memory round trip), threads < HD/2
// meanwhile compute the row's cos/sin pairs into shared memory; then the
// rotations and the stores.  A round covers 2 * 256 units (up to 64 heads of
// head_dim 64, 42 of 96, 32 of 128); longer rows take more rounds.
template <int HD, bool F16Cache>
__global__ void __launch_bounds__(kPrepThreads)
    ingest_prep_kernel(const float* __restrict__ q, const float* __restrict__ k,
                       const float* __restrict__ v, void* __restrict__ key_cache,
                       void* __restrict__ value_cache, __half* __restrict__ q16,
                       __half* __restrict__ k16, __half* __restrict__ v16, int32_t start_pos,
                       int32_t n_heads, int32_t n_kv_heads, double theta, int32_t style) {
  constexpr int kPerHead = HD / 8;  // units per head
  __shared__ __align__(16) float s_cos[HD / 2];
  __shared__ __align__(16) float s_sin[HD / 2];
  const int i = blockIdx.x, tid = threadIdx.x;
  const int pos = start_pos + i;
  const int nq = n_heads * kPerHead, nk = n_kv_heads * kPerHead, nv = 2 * nk;
  const int64_t qw = (int64_t)n_heads * HD, kvw = (int64_t)n_kv_heads * HD;
  const float* qr = q + (int64_t)i * qw;
  __half* q16r = q16 + (int64_t)i * qw;
  const float* kr = k + (int64_t)i * kvw;
  const float4* vr = reinterpret_cast<const float4*>(v + (int64_t)i * kvw);
  const int64_t crow = (int64_t)pos * kvw;
  const int rounds = (max(nq, nk) + kU * kPrepThreads - 1) / (kU * kPrepThreads);
  for (int rd = 0; rd < rounds; ++rd) {
    const int b = rd * kU * kPrepThreads + tid, bv = rd * kUV * kPrepThreads + tid;
    float4 qa[kU], qb[kU], ka[kU], kb[kU], vx[kUV];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int e = b + u * kPrepThreads;
      int o0, o1;
      if (e < nq) {
        const int h = e / kPerHead;
        unit_offsets<HD>(style, e - h * kPerHead, &o0, &o1);
        qa[u] = *reinterpret_cast<const float4*>(qr + h * HD + o0);
        qb[u] = *reinterpret_cast<const float4*>(qr + h * HD + o1);
      }
      if (e < nk) {
        const int g = e / kPerHead;
        unit_offsets<HD>(style, e - g * kPerHead, &o0, &o1);
        ka[u] = *reinterpret_cast<const float4*>(kr + g * HD + o0);
        kb[u] = *reinterpret_cast<const float4*>(kr + g * HD + o1);
      }
    }
#pragma unroll
    for (int u = 0; u < kUV; ++u)
      if (bv + u * kPrepThreads < nv) vx[u] = vr[bv + u * kPrepThreads];
    if (rd == 0) {
      if (tid < HD / 2) rope_cos_sin(pos, tid, HD, theta, &s_cos[tid], &s_sin[tid]);
      __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int e = b + u * kPrepThreads;
      int o0, o1;
      if (e < nq) {
        const int h = e / kPerHead, jj = e - h * kPerHead;
        unit_offsets<HD>(style, jj, &o0, &o1);
        const float4 c = reinterpret_cast<const float4*>(s_cos)[jj];
        const float4 sn = reinterpret_cast<const float4*>(s_sin)[jj];
        rotate_unit(style, qa[u], qb[u], c, sn);
        store_h4(q16r + h * HD + o0, qa[u]);
        store_h4(q16r + h * HD + o1, qb[u]);
      }
      if (e < nk) {
        const int g = e / kPerHead, jj = e - g * kPerHead;
        unit_offsets<HD>(style, jj, &o0, &o1);
        const float4 c = reinterpret_cast<const float4*>(s_cos)[jj];
        const float4 sn = reinterpret_cast<const float4*>(s_sin)[jj];
        rotate_unit(style, ka[u], kb[u], c, sn);
        const int64_t at = crow + g * HD;
        if constexpr (F16Cache) {
          store_h4(static_cast<__half*>(key_cache) + at + o0, ka[u]);
          store_h4(static_cast<__half*>(key_cache) + at + o1, kb[u]);
        } else {
          *reinterpret_cast<float4*>(static_cast<float*>(key_cache) + at + o0) = ka[u];
          *reinterpret_cast<float4*>(static_cast<float*>(key_cache) + at + o1) = kb[u];
          store_h4(k16 + at + o0, ka[u]);
          store_h4(k16 + at + o1, kb[u]);
        }
      }
    }
    // v: the row as it is
#pragma unroll
    for (int u = 0; u < kUV; ++u) {
      const int e = bv + u * kPrepThreads;
      if (e >= nv) continue;
      if constexpr (F16Cache) {
        store_h4(static_cast<__half*>(value_cache) + crow + 4 * e, vx[u]);
      } else {
        reinterpret_cast<float4*>(static_cast<float*>(value_cache) + crow)[e] = vx[u];
        store_h4(v16 + crow + 4 * e, vx[u]);
      }
    }
  }
}

template <bool F16Cache>
void launch_prep(int hd, int n_rows, cudaStream_t stream, const float* q, const float* k,
                 const float* v, void* key_cache, void* value_cache, __half* q16, __half* k16,
                 __half* v16, int32_t start_pos, int32_t n_heads, int32_t n_kv_heads,
                 double theta, int32_t style) {
  auto go = [&](auto kernel) {
    kernel<<<n_rows, kPrepThreads, 0, stream>>>(q, k, v, key_cache, value_cache, q16, k16, v16,
                                                start_pos, n_heads, n_kv_heads, theta, style);
  };
  if (hd == 64) go(ingest_prep_kernel<64, F16Cache>);
  else if (hd == 96) go(ingest_prep_kernel<96, F16Cache>);
  else go(ingest_prep_kernel<128, F16Cache>);
}

// FP32 cache rows 0..n_rows-1 (kvw floats each, a multiple of 4) to FP16.
__global__ void convert_rows_kernel(const float* __restrict__ key_cache,
                                    const float* __restrict__ value_cache,
                                    __half* __restrict__ k16, __half* __restrict__ v16,
                                    int64_t n4) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n4; j += stride) {
    const float4 kk = ld_cg4(key_cache + 4 * j);
    const float4 vv = ld_cg4(value_cache + 4 * j);
    reinterpret_cast<__half2*>(k16)[2 * j] = __floats2half2_rn(kk.x, kk.y);
    reinterpret_cast<__half2*>(k16)[2 * j + 1] = __floats2half2_rn(kk.z, kk.w);
    reinterpret_cast<__half2*>(v16)[2 * j] = __floats2half2_rn(vv.x, vv.y);
    reinterpret_cast<__half2*>(v16)[2 * j + 1] = __floats2half2_rn(vv.z, vv.w);
  }
}

int check_launch(const char* what, std::string* err) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string(what) + " launch failed: " + cudaGetErrorString(e);
    return GLA_ERR_CUDA;
  }
  return GLA_OK;
}

}  // namespace

size_t ingest_workspace_halves(bool f16_cache, int32_t start_pos, int32_t n_rows,
                               int32_t n_heads, int32_t n_kv_heads, int32_t head_dim) {
  // q16 [n_rows][n_heads*hd]; FP32 cache: k16, v16 [start_pos+n_rows][kv_dim];
  // each part rounded up to 8 halves (16 bytes)
  auto up8 = [](size_t x) { return (x + 7) & ~(size_t)7; };
  size_t n = up8((size_t)n_rows * n_heads * head_dim);
  if (!f16_cache) n += 2 * up8(((size_t)start_pos + n_rows) * n_kv_heads * head_dim);
  return n;
}

int launch_ingest(bool f16_cache, const float* q, const float* k, const float* v, void* key_cache,
                  void* value_cache, float* xb, uint16_t* ws, int32_t start_pos, int32_t n_rows,
                  int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, float theta,
                  int32_t rope_style, int32_t* status, const DeviceInfo& dev,
                  cudaStream_t stream, std::string* err) {
  auto up8 = [](size_t x) { return (x + 7) & ~(size_t)7; };
  const int64_t kvw = (int64_t)n_kv_heads * head_dim;
  __half* q16 = reinterpret_cast<__half*>(ws);
  __half* k16 = q16 + up8((size_t)n_rows * n_heads * head_dim);
  __half* v16 = k16 + up8(((size_t)start_pos + n_rows) * kvw);
  if (!f16_cache && start_pos > 0) {
    const int64_t n4 = (int64_t)start_pos * kvw / 4;
    const int blocks = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)dev.sms * 8);
    convert_rows_kernel<<<blocks, 256, 0, stream>>>(static_cast<const float*>(key_cache),
                                                    static_cast<const float*>(value_cache), k16,
                                                    v16, n4);
    if (int rc = check_launch("prefix conversion", err)) return rc;
  }
  if (f16_cache)
    launch_prep<true>(head_dim, n_rows, stream, q, k, v, key_cache, value_cache, q16, nullptr,
                      nullptr, start_pos, n_heads, n_kv_heads, (double)theta, rope_style);
  else
    launch_prep<false>(head_dim, n_rows, stream, q, k, v, key_cache, value_cache, q16, k16, v16,
                       start_pos, n_heads, n_kv_heads, (double)theta, rope_style);
  if (int rc = check_launch("ingest RoPE/append", err)) return rc;
  const uint16_t* kk = f16_cache ? static_cast<const uint16_t*>(key_cache)
                                 : reinterpret_cast<const uint16_t*>(k16);
  const uint16_t* vv = f16_cache ? static_cast<const uint16_t*>(value_cache)
                                 : reinterpret_cast<const uint16_t*>(v16);
  return launch_prefill_f16(reinterpret_cast<const uint16_t*>(q16), kk, vv, xb, n_rows,
                            start_pos, kvw, n_heads, n_kv_heads, head_dim,
                            1.0f / sqrtf((float)head_dim), status, dev, stream, err);
}

}  // namespace gla
