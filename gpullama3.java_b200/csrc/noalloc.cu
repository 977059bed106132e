// noalloc.cu - gla_decode_f32kv_noalloc: FP32-cache decode attention that
// allocates no device memory.
//
// Some callers cannot allocate device memory at the point where they need
// attention: a JVM thread that was handed device buffers by another owner
// (TornadoVM owns every device allocation on the reference's GPU path), code
// running under an allocator that forbids growth mid-step, or an embedder
// that must not call cudaMalloc/cudaFree because they synchronise the device.
// gla_create allocates the context workspace, so those callers use this entry
// point instead: it needs no context, and its split-KV scratch (the per-CTA
// partial records, the per-kv-head arrival counters and the device status
// word) lives in the file-scope array g_noalloc_scratch below, which every
// GPU that loads this library holds until the process exits.
//
// Set-up: the first call on a device (with that device current) looks up the
// array's device address with cudaGetSymbolAddress and caches it; make that
// first call before any stream capture on the device.
//
// Sharing: every call on a device uses the same array and it keeps the last
// call's contents.  Each call clears the status word and the counters it uses
// (one cudaMemsetAsync on the caller's stream) before its kernel.  The
// partial records need no clearing: each word carries the epoch of the call
// that wrote it, and the epoch word (never cleared; zero when the library is
// loaded) gives every call a larger one.  Calls whose kernels overlap on the
// GPU (different streams without ordering, or threads racing on one device)
// race on the array and give wrong results.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>
#include <string>

#include "gla_common.cuh"
#include "gla_internal.h"
#include "gpullama_attn.h"

namespace {

// Layout of the scratch array: [0, 4) status word, [16, 16 + 4 * kMaxCounters)
// arrival counters, [kEpochOffset, +8) the call-epoch word,
// [kHeaderBytes, kHeaderBytes + kSlotBytes) partial records.
constexpr size_t kMaxCounters = 1024;                // kv heads of one call
constexpr size_t kCounterOffset = 16;
constexpr size_t kEpochOffset = 8184;
constexpr size_t kHeaderBytes = 8192;                // status, counters, epoch
constexpr size_t kSlotBytes = size_t(1) << 20;       // 1 MiB of partial records
static_assert(kCounterOffset + 4 * kMaxCounters <= kEpochOffset, "header layout");
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kHeaderBytes + kSlotBytes];

struct DeviceScratch {
  bool ready = false;
  unsigned char* base = nullptr;  // device address of g_noalloc_scratch
  gla::DeviceInfo info{};
};

std::mutex g_mu;
DeviceScratch g_dev[kMaxDevices];

// Resolves (once per device, with that device current) the device address of
// the scratch array and the device properties the launch plan needs.
int scratch_for_current_device(DeviceScratch** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return GLA_ERR_NO_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceScratch& d = g_dev[dev];
  if (!d.ready) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return GLA_ERR_CUDA;
    }
    if (cudaDeviceGetAttribute(&d.info.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.info.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                               dev) != cudaSuccess) {
      cudaGetLastError();
      return GLA_ERR_CUDA;
    }
    d.base = static_cast<unsigned char*>(p);
    d.ready = true;
  }
  *out = &d;
  return GLA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int32_t gla_decode_f32kv_noalloc(const float* q, const float* k, const float* v,
                                            float* xb, int32_t n_heads, int32_t n_kv_heads,
                                            int32_t head_dim, int64_t kv_stride, int32_t n_pos,
                                            float scale, void* cuda_stream) {
  if (!q || !k || !v || !xb) return GLA_ERR_INVALID_ARG;
  if (n_pos < 1 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0) return GLA_ERR_INVALID_ARG;
  if (n_heads % n_kv_heads != 0) return GLA_ERR_INVALID_ARG;
  if (kv_stride < (int64_t)n_kv_heads * head_dim) return GLA_ERR_INVALID_ARG;
  if (!std::isfinite(scale)) return GLA_ERR_INVALID_ARG;
  if ((kv_stride * 4) % 16 != 0 || ((int64_t)head_dim * 4) % 16 != 0) return GLA_ERR_ALIGNMENT;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(xb)) return GLA_ERR_ALIGNMENT;

  DeviceScratch* d = nullptr;
  int rc = scratch_for_current_device(&d);
  if (rc != GLA_OK) return rc;

  gla::DecodeRequest req{};
  req.dtype = GLA_DTYPE_F32;
  req.q = q;
  req.k = k;
  req.v = v;
  req.kv_stride = kv_stride;
  req.n_pos = n_pos;
  req.n_pos_cap = n_pos;
  req.max_n_pos = n_pos;
  req.batch = 1;
  req.n_heads = n_heads;
  req.n_kv = n_kv_heads;
  req.head_dim = head_dim;
  req.scale = scale;
  req.out = xb;
  req.record_mode = 0;
  req.early_kv = 1;  // n_pos comes from the host: the same kernel path as gla_decode_f32kv

  std::string err;
  gla::DecodePlan plan;
  rc = gla::plan_decode(req, d->info, &plan, &err);
  if (rc != GLA_OK) return rc;
  // the scratch has a fixed size: refuse calls that need more
  if (plan.counters > kMaxCounters || plan.part_words * sizeof(uint64_t) > kSlotBytes)
    return GLA_ERR_NOT_SUPPORTED;

  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  gla::DecodeWorkspace ws;
  ws.status = reinterpret_cast<int32_t*>(d->base);
  ws.counter = reinterpret_cast<int32_t*>(d->base + kCounterOffset);
  ws.epoch = reinterpret_cast<unsigned long long*>(d->base + kEpochOffset);
  ws.part = reinterpret_cast<uint64_t*>(d->base + kHeaderBytes);
  // status word and this call's counters start at zero (the epoch word stays)
  if (cudaMemsetAsync(d->base, 0, kCounterOffset + plan.counters * sizeof(int32_t), stream) !=
      cudaSuccess) {
    cudaGetLastError();
    return GLA_ERR_CUDA;
  }
  return gla::launch_decode(req, plan, ws, stream, &err);
}
