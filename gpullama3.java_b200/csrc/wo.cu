// wo.cu - output projection with the residual add, the step after attention:
//
//   x[i] = x[i] + sum_j w[i][j] * xb[j],   w FP16 [d][n] row-major, xb/x FP32
//
// (matrixVectorGenericWithResidual, TransformerComputeKernelsLayered.java:715-733,
// the "matmul1" task of LlamaFP16FFNLayers.java:131; InferenceCore.java:147-150
// on the CPU).  Batch 1, so an HBM-bound GEMV: 2 bytes of weight per
// multiply-add, d*n*2 bytes a call (Llama-3.2-3B wo: 18.9 MB).
//
// One warp per row (CTAs of 8 warps); a lane owns 16-byte chunks (8 halves)
// lane, lane+32, ... of the row, so a warp's load instruction reads 512
// contiguous bytes, and all the chunks of a row pass (CH chunks a lane: the
// row rounded up to 1024/2048/3072/4096 halves) are loaded before the first
// multiply.  With CH sized to the row, a 3072 x 3072 matrix fits in one wave
// (3 CTAs an SM), every row in flight at once.  FP32 products
// and sums, lane partials joined by a shuffle tree.  xb is staged in shared
// memory once per CTA.
//
// Launched with programmatic dependent launch behind the attention kernel
// that writes xb: the weights are never written by the preceding kernel, so
// every warp loads its row's chunks into registers before griddepcontrol.wait;
// xb and x are read only after the wait.
#include <cuda_fp16.h>

#include "gla_common.cuh"
#include "gla_internal.h"

namespace gla {

namespace {

constexpr int kWoThreads = 256;
constexpr int kWoWarps = kWoThreads / 32;

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float dot8(uint4 wv, float4 a, float4 b, float acc) {
  const __half2* h = reinterpret_cast<const __half2*>(&wv);
  const float2 w0 = __half22float2(h[0]), w1 = __half22float2(h[1]);
  const float2 w2 = __half22float2(h[2]), w3 = __half22float2(h[3]);
  acc = fmaf(w0.x, a.x, acc);
  acc = fmaf(w0.y, a.y, acc);
  acc = fmaf(w1.x, a.z, acc);
  acc = fmaf(w1.y, a.w, acc);
  acc = fmaf(w2.x, b.x, acc);
  acc = fmaf(w2.y, b.y, acc);
  acc = fmaf(w3.x, b.z, acc);
  acc = fmaf(w3.y, b.w, acc);
  return acc;
}

template <int CH>  // 16-byte chunks a lane holds per row pass
__global__ void __launch_bounds__(kWoThreads)
    wo_residual_kernel(const uint16_t* __restrict__ w, const float* __restrict__ xb,
                       float* __restrict__ x, int32_t n, int32_t d) {
  extern __shared__ float4 s_xb[];  // n / 4
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kWoWarps + warp, nw = gridDim.x * kWoWarps;
  const int nch = n >> 3;  // 16-byte chunks a row
  uint4 c[CH];
  auto load_pass = [&](int r, int base) {
    const uint4* wr = reinterpret_cast<const uint4*>(w + (int64_t)r * n);
#pragma unroll
    for (int u = 0; u < CH; ++u) {
      const int ch = base + lane + 32 * u;
      if (ch < nch) c[u] = ld_stream16(wr + ch);
    }
  };
  if (gw < d) load_pass(gw, 0);
  // xb and x are written by the preceding kernels
  pdl_wait();
  pdl_launch_dependents();
  const float4* xb4 = reinterpret_cast<const float4*>(xb);
  for (int i = threadIdx.x; i < (n >> 2); i += kWoThreads) s_xb[i] = xb4[i];
  __syncthreads();
  for (int r = gw; r < d; r += nw) {
    float acc = 0.f;
    for (int base = 0; base < nch; base += 32 * CH) {
      if (r != gw || base != 0) load_pass(r, base);
#pragma unroll
      for (int u = 0; u < CH; ++u) {
        const int ch = base + lane + 32 * u;
        if (ch < nch) acc = dot8(c[u], s_xb[2 * ch], s_xb[2 * ch + 1], acc);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    if (lane == 0) x[r] = x[r] + acc;
  }
}

}  // namespace

int launch_wo_residual_f16(const uint16_t* w, const float* xb, float* x, int32_t n, int32_t d,
                           const DeviceInfo& dev, cudaStream_t stream, std::string* err) {
  const size_t smem = (size_t)n * sizeof(float);
  if (smem > (size_t)dev.smem_optin) {
    *err = "wo input dimension too large for shared memory";
    return GLA_ERR_NOT_SUPPORTED;
  }
  // one row a warp (rows past the resident CTAs wait for a free slot)
  const int grid = (d + kWoWarps - 1) / kWoWarps;
  const int per_lane = (n / 8 + 31) / 32;  // chunks a lane owns in the whole row
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWoThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto go = [&](auto kern) {
    static std::atomic<uint64_t> smem_set{0};
    ensure_smem_attr(kern, smem, smem_set);
    return cudaLaunchKernelEx(&cfg, kern, w, xb, x, n, d);
  };
  cudaError_t e = per_lane <= 4    ? go(wo_residual_kernel<4>)
                  : per_lane <= 8  ? go(wo_residual_kernel<8>)
                  : per_lane <= 12 ? go(wo_residual_kernel<12>)
                                   : go(wo_residual_kernel<16>);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("wo launch failed: ") + cudaGetErrorString(e);
    return GLA_ERR_CUDA;
  }
  return GLA_OK;
}

}  // namespace gla
