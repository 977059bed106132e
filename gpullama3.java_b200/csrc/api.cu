// api.cu - the C ABI of libgpullama_attn (include/gpullama_attn.h).
//
// Argument checking, the context (device, stream, workspace, status word,
// communicator) and dispatch to the kernel launchers.  Every entry point
// returns a status code; no exception crosses the ABI.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "gpullama_attn.h"
#include "gla_common.cuh"
#include "gla_internal.h"
#include "gla_comm.h"
#include "gla_peer.h"
#include "gla_xch.h"

struct gla_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  gla::DeviceInfo dev{};
  int32_t* status = nullptr;        // device status word
  int32_t* counters = nullptr;      // piece counters (zero between calls)
  size_t counters_cap = 0;
  uint64_t* parts = nullptr;        // piece slots (tagged 64-bit words, zeroed at allocation)
  size_t parts_cap = 0;             // words
  uint64_t* trace = nullptr;        // GLA_OPT_TRACE: per-CTA phase stamps of the last decode
  size_t trace_words = 0;
  float* records = nullptr;         // sharded decode: local records
  float* gathered = nullptr;        // sharded decode: all ranks' records
  size_t records_cap = 0;           // floats per rank
  uint16_t* ingest_ws = nullptr;    // prompt ingestion: FP16 q (and K/V) copies
  size_t ingest_cap = 0;            // halves
  gla::Comm comm;
  gla::PeerExchange xch;            // sharded decode: peer exchange buffers
  int32_t opt_early_kv = 2;         // GLA_OPT_EARLY_KV_PREFETCH
  int32_t opt_shard_exchange = 1;   // GLA_OPT_SHARD_EXCHANGE
  std::string last_error;
};

namespace {

int fail(gla_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}

int cuda_fail(gla_ctx* ctx, cudaError_t e, const char* what) {
  return fail(ctx, GLA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The context's 256-byte status block: the device status word at 0, the
// decode call-epoch word (see DecodeWorkspace) at kEpochOffset.
constexpr size_t kEpochOffset = 64;

// Makes the context's device current for the duration of a call.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

bool stream_capturing(cudaStream_t s) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &st) != cudaSuccess) return false;
  return st != cudaStreamCaptureStatusNone;
}

// Grows the piece workspace; never during stream capture.
int ensure_workspace(gla_ctx* ctx, size_t part_words, size_t counters) {
  if (part_words <= ctx->parts_cap && counters <= ctx->counters_cap) return GLA_OK;
  if (stream_capturing(ctx->stream))
    return fail(ctx, GLA_ERR_INVALID_ARG,
                "decode workspace must grow; call gla_reserve before stream capture");
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaStreamSynchronize");
  if (part_words > ctx->parts_cap) {
    size_t cap = std::max(part_words, ctx->parts_cap * 2);
    cudaFree(ctx->parts);
    ctx->parts = nullptr;
    ctx->parts_cap = 0;
    e = cudaMalloc(&ctx->parts, cap * sizeof(uint64_t));
    if (e != cudaSuccess) return fail(ctx, GLA_ERR_OUT_OF_MEMORY, "workspace allocation failed");
    // epoch 0 on every word: no call uses epoch 0
    e = cudaMemsetAsync(ctx->parts, 0, cap * sizeof(uint64_t), ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemsetAsync");
    ctx->parts_cap = cap;
  }
  if (counters > ctx->counters_cap) {
    size_t cap = std::max(counters, ctx->counters_cap * 2);
    cudaFree(ctx->counters);
    ctx->counters = nullptr;
    ctx->counters_cap = 0;
    e = cudaMalloc(&ctx->counters, cap * sizeof(int32_t));
    if (e != cudaSuccess) return fail(ctx, GLA_ERR_OUT_OF_MEMORY, "workspace allocation failed");
    e = cudaMemsetAsync(ctx->counters, 0, cap * sizeof(int32_t), ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemsetAsync");
    ctx->counters_cap = cap;
  }
  return GLA_OK;
}

int check_decode_shape(gla_ctx* ctx, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                       int64_t kv_stride, int esize) {
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0)
    return fail(ctx, GLA_ERR_INVALID_ARG, "n_heads, n_kv_heads and head_dim must be positive");
  if (n_heads % n_kv_heads != 0)
    return fail(ctx, GLA_ERR_INVALID_ARG, "n_heads must be a multiple of n_kv_heads");
  if (kv_stride < (int64_t)n_kv_heads * head_dim)
    return fail(ctx, GLA_ERR_INVALID_ARG, "kv_stride must be >= n_kv_heads * head_dim");
  if ((kv_stride * esize) % 16 != 0 || ((int64_t)head_dim * esize) % 16 != 0)
    return fail(ctx, GLA_ERR_ALIGNMENT, "kv_stride and head_dim must be multiples of 16 bytes");
  return GLA_OK;
}

int run_decode(gla_ctx* ctx, gla::DecodeRequest& req) {
  req.early_kv = ctx->opt_early_kv;  // every context entry point honours the option
  std::string err;
  gla::DecodePlan plan;
  int rc = gla::plan_decode(req, ctx->dev, &plan, &err);
  if (rc != GLA_OK) return fail(ctx, rc, err);
  rc = ensure_workspace(ctx, plan.part_words, plan.counters);
  if (rc != GLA_OK) return rc;
  gla::DecodeWorkspace ws;
  ws.part = ctx->parts;
  ws.counter = ctx->counters;
  ws.epoch = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(ctx->status) +
                                                    kEpochOffset);
  ws.status = ctx->status;
  ws.trace = (ctx->trace && (size_t)plan.grid * gla::kTraceWordsPerCta <= ctx->trace_words)
                 ? ctx->trace
                 : nullptr;
  rc = gla::launch_decode(req, plan, ws, ctx->stream, &err);
  if (rc != GLA_OK) return fail(ctx, rc, err);
  return GLA_OK;
}

int decode_single(gla_ctx* ctx, int dtype, const float* q, const void* k, const void* v,
                  float* out, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                  int64_t kv_stride, int32_t n_pos, float scale, int32_t record_mode) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!q || !k || !v || !out) return fail(ctx, GLA_ERR_INVALID_ARG, "null tensor pointer");
  if (n_pos < 1) return fail(ctx, GLA_ERR_INVALID_ARG, "n_pos must be >= 1");
  if (!std::isfinite(scale)) return fail(ctx, GLA_ERR_INVALID_ARG, "scale must be finite");
  const int esize = dtype == GLA_DTYPE_F32 ? 4 : 2;
  int rc = check_decode_shape(ctx, n_heads, n_kv_heads, head_dim, kv_stride, esize);
  if (rc != GLA_OK) return rc;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(ctx, GLA_ERR_ALIGNMENT, "q, k, v and the output must be 16-byte aligned");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, GLA_ERR_CUDA, "cudaSetDevice failed");
  gla::DecodeRequest req{};
  req.dtype = dtype;
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
  req.out = out;
  req.record_mode = record_mode;
  return run_decode(ctx, req);
}

int decode_batched(gla_ctx* ctx, int dtype, const float* q, const void* const* k_ptrs,
                   const void* const* v_ptrs, const int32_t* n_pos, int32_t max_n_pos,
                   float* xb, int32_t batch, int32_t n_heads, int32_t n_kv_heads,
                   int32_t head_dim, int64_t kv_stride, float scale) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!q || !k_ptrs || !v_ptrs || !n_pos || !xb)
    return fail(ctx, GLA_ERR_INVALID_ARG, "null pointer");
  if (batch < 1) return fail(ctx, GLA_ERR_INVALID_ARG, "batch must be >= 1");
  if (max_n_pos < 1) return fail(ctx, GLA_ERR_INVALID_ARG, "max_n_pos must be >= 1");
  if (!std::isfinite(scale)) return fail(ctx, GLA_ERR_INVALID_ARG, "scale must be finite");
  const int esize = dtype == GLA_DTYPE_F32 ? 4 : 2;
  int rc = check_decode_shape(ctx, n_heads, n_kv_heads, head_dim, kv_stride, esize);
  if (rc != GLA_OK) return rc;
  if (!aligned16(q) || !aligned16(xb))
    return fail(ctx, GLA_ERR_ALIGNMENT, "q and xb must be 16-byte aligned");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, GLA_ERR_CUDA, "cudaSetDevice failed");
  gla::DecodeRequest req{};
  req.dtype = dtype;
  req.q = q;
  req.k_ptrs = k_ptrs;
  req.v_ptrs = v_ptrs;
  req.kv_stride = kv_stride;
  req.n_pos_dev = n_pos;
  req.n_pos_add = 0;
  req.n_pos_cap = max_n_pos;
  req.max_n_pos = max_n_pos;
  req.batch = batch;
  req.n_heads = n_heads;
  req.n_kv = n_kv_heads;
  req.head_dim = head_dim;
  req.scale = scale;
  req.out = xb;
  req.record_mode = 0;
  return run_decode(ctx, req);
}

struct RopeAppend {
  const float* k = nullptr;  // new key row [kvDim], unrotated
  const float* v = nullptr;  // new value row [kvDim]
  float theta = 0.f;
  int32_t style = 0;
};

int process_heads(gla_ctx* ctx, int dtype, const float* q, const void* key_cache,
                  const void* value_cache, float* xb, int32_t n_heads, int32_t head_size,
                  int32_t kv_dim, int32_t kv_mul, const int32_t* position_holder, int32_t layer,
                  int32_t context_length, const RopeAppend* rope = nullptr) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!q || !key_cache || !value_cache || !xb || !position_holder)
    return fail(ctx, GLA_ERR_INVALID_ARG, "null pointer");
  if (kv_mul <= 0 || n_heads <= 0 || n_heads % kv_mul != 0)
    return fail(ctx, GLA_ERR_INVALID_ARG, "kvMul must divide nHeads");
  const int32_t n_kv = n_heads / kv_mul;
  if ((int64_t)n_kv * head_size != kv_dim)
    return fail(ctx, GLA_ERR_INVALID_ARG, "kvDim must equal (nHeads / kvMul) * headSize");
  if (layer < 0 || context_length < 1)
    return fail(ctx, GLA_ERR_INVALID_ARG, "layer must be >= 0 and contextLength >= 1");
  const int esize = dtype == GLA_DTYPE_F32 ? 4 : 2;
  int rc = check_decode_shape(ctx, n_heads, n_kv, head_size, kv_dim, esize);
  if (rc != GLA_OK) return rc;
  if (!aligned16(q) || !aligned16(key_cache) || !aligned16(value_cache) || !aligned16(xb))
    return fail(ctx, GLA_ERR_ALIGNMENT, "q, caches and xb must be 16-byte aligned");
  if (rope && (!rope->k || !rope->v)) return fail(ctx, GLA_ERR_INVALID_ARG, "null pointer");
  if (rope && (!aligned16(rope->k) || !aligned16(rope->v)))
    return fail(ctx, GLA_ERR_ALIGNMENT, "k and v must be 16-byte aligned");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, GLA_ERR_CUDA, "cudaSetDevice failed");
  const int64_t loff = (int64_t)layer * context_length * kv_dim * esize;  // 64-bit layer offset
  gla::DecodeRequest req{};
  req.dtype = dtype;
  req.q = q;
  req.k = static_cast<const char*>(key_cache) + loff;
  req.v = static_cast<const char*>(value_cache) + loff;
  req.kv_stride = kv_dim;
  req.n_pos_dev = position_holder;
  req.n_pos_add = 1;
  req.n_pos_cap = context_length;
  req.max_n_pos = context_length;
  req.batch = 1;
  req.n_heads = n_heads;
  req.n_kv = n_kv;
  req.head_dim = head_size;
  req.scale = (float)(1.0 / std::sqrt((double)head_size));
  req.out = xb;
  req.record_mode = 0;
  if (rope) {
    if (!rope->k || !rope->v) return fail(ctx, GLA_ERR_INVALID_ARG, "null new key/value row");
    if (rope->style != GLA_ROPE_INTERLEAVED && rope->style != GLA_ROPE_NEOX)
      return fail(ctx, GLA_ERR_INVALID_ARG, "unknown rope_style");
    if (!(rope->theta > 0.f) || !std::isfinite(rope->theta))
      return fail(ctx, GLA_ERR_INVALID_ARG, "theta must be positive");
    req.rope = 1;
    req.rope_k = rope->k;
    req.rope_v = rope->v;
    req.rope_theta = (double)rope->theta;
    req.rope_style = rope->style;
  }
  return run_decode(ctx, req);
}

int sharded(gla_ctx* ctx, int dtype, const float* q, const void* k, const void* v, float* xb,
            int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int64_t kv_stride,
            int32_t n_pos_local, float scale) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!ctx->comm.active() && !ctx->xch.loopback())
    return fail(ctx, GLA_ERR_COMM, "gla_comm_init has not been called on this context");
  if (!xb) return fail(ctx, GLA_ERR_INVALID_ARG, "null xb");
  const size_t rec = (size_t)n_heads * (head_dim + 2);
  if (rec > ctx->records_cap) {
    if (stream_capturing(ctx->stream))
      return fail(ctx, GLA_ERR_INVALID_ARG, "record buffers must grow outside stream capture");
    DeviceGuard dg(ctx->device);
    std::string werr;
    int wrc = ctx->comm.wait(ctx->stream, &werr);
    if (wrc != GLA_OK) {
      ctx->xch.teardown();
      return fail(ctx, wrc, werr);
    }
    cudaFree(ctx->records);
    cudaFree(ctx->gathered);
    ctx->records = ctx->gathered = nullptr;
    ctx->records_cap = 0;
    if (cudaMalloc(&ctx->records, rec * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&ctx->gathered, rec * ctx->comm.nranks * sizeof(float)) != cudaSuccess)
      return fail(ctx, GLA_ERR_OUT_OF_MEMORY, "record buffer allocation failed");
    ctx->records_cap = rec;
  }
  int rc;
  if (ctx->opt_shard_exchange && ctx->xch.active() &&
      (size_t)n_heads * (head_dim + 4) <= (size_t)gla::kXchRecWords &&
      n_kv_heads <= gla::kXchMaxSeg) {
    // one kernel: shard attention, records to every rank over peer memory,
    // merge; an empty shard (n_pos_local == 0) still publishes empty records
    if (!q || !k || !v) return fail(ctx, GLA_ERR_INVALID_ARG, "null tensor pointer");
    if (n_pos_local < 0) return fail(ctx, GLA_ERR_INVALID_ARG, "n_pos_local must be >= 0");
    if (!std::isfinite(scale)) return fail(ctx, GLA_ERR_INVALID_ARG, "scale must be finite");
    const int esize = dtype == GLA_DTYPE_F32 ? 4 : 2;
    rc = check_decode_shape(ctx, n_heads, n_kv_heads, head_dim, kv_stride, esize);
    if (rc != GLA_OK) return rc;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(xb))
      return fail(ctx, GLA_ERR_ALIGNMENT, "q, k, v and xb must be 16-byte aligned");
    DeviceGuard dg(ctx->device);
    gla::DecodeRequest req{};
    req.dtype = dtype;
    req.q = q;
    req.k = k;
    req.v = v;
    req.kv_stride = kv_stride;
    req.n_pos = n_pos_local;
    req.n_pos_cap = std::max(1, n_pos_local);
    req.max_n_pos = n_pos_local;
    req.batch = 1;
    req.n_heads = n_heads;
    req.n_kv = n_kv_heads;
    req.head_dim = head_dim;
    req.scale = scale;
    req.out = ctx->records;
    req.record_mode = 2;
    req.xch_bases = ctx->xch.bases();
    req.xch_local = ctx->xch.local();
    req.xch_out = xb;
    req.xch_world = ctx->xch.world;
    req.xch_rank = ctx->xch.rank;
    return run_decode(ctx, req);
  }
  if (n_pos_local >= 1) {
    rc = decode_single(ctx, dtype, q, k, v, ctx->records, n_heads, n_kv_heads, head_dim, kv_stride,
                       n_pos_local, scale, 1);
    if (rc != GLA_OK) return rc;
  } else {
    // an empty shard contributes l = 0 records
    DeviceGuard dg(ctx->device);
    cudaMemsetAsync(ctx->records, 0, rec * sizeof(float), ctx->stream);
  }
  DeviceGuard dg(ctx->device);
  std::string err;
  rc = ctx->comm.all_gather(ctx->records, ctx->gathered, rec, ctx->stream, &err);
  if (rc != GLA_OK) return fail(ctx, rc, err);
  rc = gla::launch_lse_combine(ctx->gathered, ctx->comm.nranks, n_heads, head_dim, xb,
                               ctx->stream, &err);
  if (rc != GLA_OK) return fail(ctx, rc, err);
  return GLA_OK;
}

// Collective end of the communicator's use before the peer exchange buffers
// are unmapped and freed: this rank's stream drains (bounded), then every
// rank meets at a barrier, so no rank's kernel still stores records into a
// buffer that is about to be freed.  If a rank does not arrive within the
// communicator timeout, the communicator is aborted (GLA_ERR_TIMEOUT) and
// the buffers are released anyway.
int quiesce_comm(gla_ctx* ctx) {
  if (!ctx->comm.active()) return GLA_OK;
  std::string err;
  int rc = ctx->comm.wait(ctx->stream, &err);
  if (rc == GLA_OK) rc = ctx->comm.barrier(ctx->stream, &err);
  if (rc != GLA_OK) fail(ctx, rc, err);
  return rc;
}

}  // namespace

extern "C" {

int32_t gla_version(void) { return GLA_VERSION; }

const char* gla_status_string(int32_t status) {
  switch (status) {
    case GLA_OK: return "GLA_OK";
    case GLA_ERR_INVALID_ARG: return "GLA_ERR_INVALID_ARG";
    case GLA_ERR_CUDA: return "GLA_ERR_CUDA";
    case GLA_ERR_NOT_SUPPORTED: return "GLA_ERR_NOT_SUPPORTED";
    case GLA_ERR_ALIGNMENT: return "GLA_ERR_ALIGNMENT";
    case GLA_ERR_TIMEOUT: return "GLA_ERR_TIMEOUT";
    case GLA_ERR_COMM: return "GLA_ERR_COMM";
    case GLA_ERR_NO_DEVICE: return "GLA_ERR_NO_DEVICE";
    case GLA_ERR_OUT_OF_MEMORY: return "GLA_ERR_OUT_OF_MEMORY";
    default: return "GLA_ERR_UNKNOWN";
  }
}

int32_t gla_create(int32_t device, void* cuda_stream, gla_ctx** out) {
  if (!out) return GLA_ERR_INVALID_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return GLA_ERR_NO_DEVICE;
  }
  if (device < 0 || device >= n) return GLA_ERR_NO_DEVICE;
  gla_ctx* ctx = nullptr;
  try {
    ctx = new gla_ctx();
  } catch (const std::exception&) {
    return GLA_ERR_OUT_OF_MEMORY;
  }
  ctx->device = device;
  ctx->stream = static_cast<cudaStream_t>(cuda_stream);
  DeviceGuard dg(device);
  if (!dg.ok) {
    delete ctx;
    return GLA_ERR_CUDA;
  }
  cudaDeviceGetAttribute(&ctx->dev.sms, cudaDevAttrMultiProcessorCount, device);
  cudaDeviceGetAttribute(&ctx->dev.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  cudaDeviceGetAttribute(&ctx->dev.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor,
                         device);
  if (cudaMalloc(&ctx->status, 256) != cudaSuccess) {
    delete ctx;
    return GLA_ERR_OUT_OF_MEMORY;
  }
  cudaMemset(ctx->status, 0, 256);
  *out = ctx;
  return GLA_OK;
}

int32_t gla_destroy(gla_ctx* ctx) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  int rc = GLA_OK;
  {
    DeviceGuard dg(ctx->device);
    rc = quiesce_comm(ctx);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    ctx->xch.teardown();
    ctx->comm.destroy();
    cudaFree(ctx->status);
    cudaFree(ctx->counters);
    cudaFree(ctx->parts);
    cudaFree(ctx->records);
    cudaFree(ctx->gathered);
    cudaFree(ctx->ingest_ws);
    cudaFree(ctx->trace);
  }
  delete ctx;
  return rc;
}

int32_t gla_set_stream(gla_ctx* ctx, void* cuda_stream) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  ctx->stream = static_cast<cudaStream_t>(cuda_stream);
  return GLA_OK;
}

const char* gla_last_error(const gla_ctx* ctx) { return ctx ? ctx->last_error.c_str() : ""; }

int32_t gla_device_status(gla_ctx* ctx, int32_t* device_status) {
  if (!ctx || !device_status) return GLA_ERR_INVALID_ARG;
  DeviceGuard dg(ctx->device);
  if (ctx->comm.active()) {
    // bounded: a collective that waits for a rank that left is ended by the
    // host watchdog (the communicator is aborted)
    std::string err;
    int rc = ctx->comm.wait(ctx->stream, &err);
    if (rc != GLA_OK) {
      ctx->xch.teardown();
      return fail(ctx, rc, err);
    }
  }
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaStreamSynchronize");
  int32_t v = 0;
  e = cudaMemcpy(&v, ctx->status, sizeof v, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpy");
  if (v != 0) {
    cudaMemset(ctx->status, 0, sizeof v);
    // a kernel that gave up may have left piece counters raised
    if (ctx->counters) cudaMemset(ctx->counters, 0, ctx->counters_cap * sizeof(int32_t));
  }
  *device_status = v;
  return GLA_OK;
}

int32_t gla_reserve(gla_ctx* ctx, int32_t max_batch, int32_t max_kv_heads, int32_t max_heads,
                    int32_t max_head_dim) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (max_batch < 1 || max_kv_heads < 1 || max_heads < 1 || max_head_dim < 1)
    return fail(ctx, GLA_ERR_INVALID_ARG, "reserve sizes must be positive");
  const int group = std::max(1, max_heads / max_kv_heads);
  DeviceGuard dg(ctx->device);
  // grids run up to two CTAs an SM (batched FP16 decode)
  const size_t part = (size_t)(2 * ctx->dev.sms + (size_t)max_batch * max_kv_heads) * group *
                      (max_head_dim + 4);
  return ensure_workspace(ctx, part, (size_t)max_batch * max_kv_heads);
}

int32_t gla_num_sms(const gla_ctx* ctx) { return ctx ? ctx->dev.sms : 0; }

int32_t gla_set_option(gla_ctx* ctx, int32_t option, int32_t value) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  switch (option) {
    case GLA_OPT_SHARD_EXCHANGE:
      if (value < 0 || value > 1) return fail(ctx, GLA_ERR_INVALID_ARG, "value must be 0 or 1");
      ctx->opt_shard_exchange = value;
      return GLA_OK;
    case GLA_OPT_EARLY_KV_PREFETCH:
      if (value < 0 || value > 2) return fail(ctx, GLA_ERR_INVALID_ARG, "value must be 0, 1 or 2");
      ctx->opt_early_kv = value;
      return GLA_OK;
    case GLA_OPT_TRACE: {
      if (value < 0 || value > 1) return fail(ctx, GLA_ERR_INVALID_ARG, "value must be 0 or 1");
      if (value == 0) {
        DeviceGuard dg(ctx->device);
        cudaStreamSynchronize(ctx->stream);
        cudaFree(ctx->trace);
        ctx->trace = nullptr;
        ctx->trace_words = 0;
        return GLA_OK;
      }
      if (ctx->trace) return GLA_OK;
      if (stream_capturing(ctx->stream))
        return fail(ctx, GLA_ERR_INVALID_ARG, "turn tracing on outside stream capture");
      DeviceGuard dg(ctx->device);
      const size_t words = (size_t)2 * ctx->dev.sms * gla::kTraceWordsPerCta;
      if (cudaMalloc(&ctx->trace, words * sizeof(uint64_t)) != cudaSuccess) {
        cudaGetLastError();
        ctx->trace = nullptr;
        return fail(ctx, GLA_ERR_OUT_OF_MEMORY, "trace buffer allocation failed");
      }
      cudaMemsetAsync(ctx->trace, 0, words * sizeof(uint64_t), ctx->stream);
      ctx->trace_words = words;
      return GLA_OK;
    }
    case GLA_OPT_COMM_TIMEOUT_MS:
      if (value < 1) return fail(ctx, GLA_ERR_INVALID_ARG, "timeout must be >= 1 ms");
      ctx->comm.timeout_ms = value;
      return GLA_OK;
    default:
      return fail(ctx, GLA_ERR_INVALID_ARG, "unknown option");
  }
}

int32_t gla_kv_cache_alloc(gla_ctx* ctx, int32_t n_layers, int32_t context_length, int32_t kv_dim,
                           int32_t dtype, void** key_cache, void** value_cache) {
  if (!ctx || !key_cache || !value_cache) return GLA_ERR_INVALID_ARG;
  *key_cache = *value_cache = nullptr;
  if (n_layers < 1 || context_length < 1 || kv_dim < 1)
    return fail(ctx, GLA_ERR_INVALID_ARG, "cache dimensions must be positive");
  if (dtype != GLA_DTYPE_F32 && dtype != GLA_DTYPE_F16)
    return fail(ctx, GLA_ERR_INVALID_ARG, "dtype must be GLA_DTYPE_F32 or GLA_DTYPE_F16");
  const size_t bytes =
      (size_t)n_layers * context_length * kv_dim * (dtype == GLA_DTYPE_F32 ? 4 : 2);
  DeviceGuard dg(ctx->device);
  void* k = nullptr;
  void* v = nullptr;
  if (cudaMalloc(&k, bytes) != cudaSuccess || cudaMalloc(&v, bytes) != cudaSuccess) {
    cudaFree(k);
    cudaGetLastError();
    return fail(ctx, GLA_ERR_OUT_OF_MEMORY, "KV cache allocation failed");
  }
  cudaMemsetAsync(k, 0, bytes, ctx->stream);
  cudaMemsetAsync(v, 0, bytes, ctx->stream);
  *key_cache = k;
  *value_cache = v;
  return GLA_OK;
}

int32_t gla_kv_cache_free(gla_ctx* ctx, void* key_cache, void* value_cache) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  DeviceGuard dg(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  cudaFree(key_cache);
  cudaFree(value_cache);
  return GLA_OK;
}

int32_t gla_process_heads_flash_attention(gla_ctx* ctx, const float* q, const float* key_cache,
                                          const float* value_cache, float* xb, int32_t n_heads,
                                          int32_t head_size, int32_t kv_dim, int32_t kv_mul,
                                          const int32_t* position_holder, int32_t layer,
                                          int32_t context_length) {
  return process_heads(ctx, GLA_DTYPE_F32, q, key_cache, value_cache, xb, n_heads, head_size,
                       kv_dim, kv_mul, position_holder, layer, context_length);
}

int32_t gla_rope_append_attention_f32(gla_ctx* ctx, const float* q, const float* k,
                                      const float* v, float* key_cache, float* value_cache,
                                      float* xb, int32_t n_heads, int32_t head_size,
                                      int32_t kv_dim, int32_t kv_mul,
                                      const int32_t* position_holder, int32_t layer,
                                      int32_t context_length, float theta, int32_t rope_style) {
  RopeAppend ra;
  ra.k = k;
  ra.v = v;
  ra.theta = theta;
  ra.style = rope_style;
  return process_heads(ctx, GLA_DTYPE_F32, q, key_cache, value_cache, xb, n_heads, head_size,
                       kv_dim, kv_mul, position_holder, layer, context_length, &ra);
}

int32_t gla_process_heads_flash_attention_f16kv(gla_ctx* ctx, const float* q,
                                                const uint16_t* key_cache,
                                                const uint16_t* value_cache, float* xb,
                                                int32_t n_heads, int32_t head_size, int32_t kv_dim,
                                                int32_t kv_mul, const int32_t* position_holder,
                                                int32_t layer, int32_t context_length) {
  return process_heads(ctx, GLA_DTYPE_F16, q, key_cache, value_cache, xb, n_heads, head_size,
                       kv_dim, kv_mul, position_holder, layer, context_length);
}

int32_t gla_decode_f32kv(gla_ctx* ctx, const float* q, const float* k, const float* v, float* xb,
                         int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int64_t kv_stride,
                         int32_t n_pos, float scale) {
  return decode_single(ctx, GLA_DTYPE_F32, q, k, v, xb, n_heads, n_kv_heads, head_dim, kv_stride,
                       n_pos, scale, 0);
}

int32_t gla_decode_f16kv(gla_ctx* ctx, const float* q, const uint16_t* k, const uint16_t* v,
                         float* xb, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                         int64_t kv_stride, int32_t n_pos, float scale) {
  return decode_single(ctx, GLA_DTYPE_F16, q, k, v, xb, n_heads, n_kv_heads, head_dim, kv_stride,
                       n_pos, scale, 0);
}

int32_t gla_decode_q8kv(gla_ctx* ctx, const float* q, const int8_t* k, const int8_t* v,
                        const uint16_t* scales, float* xb, int32_t n_heads, int32_t n_kv_heads,
                        int32_t head_dim, int64_t kv_stride, int32_t n_pos, float scale) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!q || !k || !v || !scales || !xb) return fail(ctx, GLA_ERR_INVALID_ARG, "null pointer");
  if (n_pos < 1) return fail(ctx, GLA_ERR_INVALID_ARG, "n_pos must be >= 1");
  if (!std::isfinite(scale)) return fail(ctx, GLA_ERR_INVALID_ARG, "scale must be finite");
  int rc = check_decode_shape(ctx, n_heads, n_kv_heads, head_dim, kv_stride, 1);
  if (rc != GLA_OK) return rc;
  if (head_dim != 64 && head_dim != 128)
    return fail(ctx, GLA_ERR_NOT_SUPPORTED, "Q8 cache: head_dim 64 or 128");
  if (kv_stride % 16 != 0) return fail(ctx, GLA_ERR_ALIGNMENT, "Q8 kv_stride must be a multiple of 16");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(scales) || !aligned16(xb))
    return fail(ctx, GLA_ERR_ALIGNMENT, "q, k, v, scales and xb must be 16-byte aligned");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, GLA_ERR_CUDA, "cudaSetDevice failed");
  gla::DecodeRequest req{};
  req.dtype = GLA_DTYPE_Q8;
  req.q = q;
  req.k = k;
  req.v = v;
  req.scales = scales;
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
  return run_decode(ctx, req);
}

int32_t gla_kv_quantize_q8(gla_ctx* ctx, const float* k, const float* v, int64_t src_stride,
                           int32_t n_rows, int32_t n_kv_heads, int32_t head_dim, int8_t* kq,
                           int8_t* vq, int64_t kv_stride, uint16_t* scales) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!k || !v || !kq || !vq || !scales) return fail(ctx, GLA_ERR_INVALID_ARG, "null pointer");
  if (n_rows < 1 || n_kv_heads < 1 || head_dim < 32 || head_dim > 128 || head_dim % 32 != 0)
    return fail(ctx, GLA_ERR_INVALID_ARG, "bad quantisation shape");
  if (src_stride < (int64_t)n_kv_heads * head_dim || kv_stride < (int64_t)n_kv_heads * head_dim)
    return fail(ctx, GLA_ERR_INVALID_ARG, "row strides shorter than n_kv_heads * head_dim");
  DeviceGuard dg(ctx->device);
  std::string err;
  int rc = gla::launch_quantize_q8(k, v, src_stride, n_rows, n_kv_heads, head_dim, kq, vq,
                                   kv_stride, scales, ctx->stream, &err);
  return rc == GLA_OK ? GLA_OK : fail(ctx, rc, err);
}

int32_t gla_kv_cache_alloc_q8(gla_ctx* ctx, int32_t n_layers, int32_t context_length,
                              int32_t n_kv_heads, int32_t head_dim, int8_t** key_cache,
                              int8_t** value_cache, uint16_t** scales) {
  if (!ctx || !key_cache || !value_cache || !scales) return GLA_ERR_INVALID_ARG;
  *key_cache = *value_cache = nullptr;
  *scales = nullptr;
  if (n_layers < 1 || context_length < 1 || n_kv_heads < 1)
    return fail(ctx, GLA_ERR_INVALID_ARG, "cache dimensions must be positive");
  if (head_dim != 64 && head_dim != 128)
    return fail(ctx, GLA_ERR_NOT_SUPPORTED, "Q8 cache: head_dim 64 or 128");
  const size_t rows = (size_t)n_layers * context_length;
  const size_t vbytes = rows * n_kv_heads * head_dim;
  const size_t sbytes = rows * n_kv_heads * 8 * sizeof(uint16_t);
  DeviceGuard dg(ctx->device);
  void *k = nullptr, *v = nullptr, *sc = nullptr;
  if (cudaMalloc(&k, vbytes) != cudaSuccess || cudaMalloc(&v, vbytes) != cudaSuccess ||
      cudaMalloc(&sc, sbytes) != cudaSuccess) {
    cudaFree(k);
    cudaFree(v);
    cudaGetLastError();
    return fail(ctx, GLA_ERR_OUT_OF_MEMORY, "Q8 KV cache allocation failed");
  }
  cudaMemsetAsync(k, 0, vbytes, ctx->stream);
  cudaMemsetAsync(v, 0, vbytes, ctx->stream);
  cudaMemsetAsync(sc, 0, sbytes, ctx->stream);
  *key_cache = static_cast<int8_t*>(k);
  *value_cache = static_cast<int8_t*>(v);
  *scales = static_cast<uint16_t*>(sc);
  return GLA_OK;
}

int32_t gla_kv_cache_free_q8(gla_ctx* ctx, int8_t* key_cache, int8_t* value_cache,
                             uint16_t* scales) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  DeviceGuard dg(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  cudaFree(key_cache);
  cudaFree(value_cache);
  cudaFree(scales);
  return GLA_OK;
}

int32_t gla_rope_append_q8(gla_ctx* ctx, float* q, float* k, const float* v, int8_t* key_cache,
                           int8_t* value_cache, uint16_t* scales, int32_t n_heads,
                           int32_t n_kv_heads, int32_t head_dim, const int32_t* position_holder,
                           int32_t context_length, float theta, int32_t rope_style) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!q || !k || !v || !key_cache || !value_cache || !scales || !position_holder)
    return fail(ctx, GLA_ERR_INVALID_ARG, "null pointer");
  if (n_heads < 1 || n_kv_heads < 1 || n_kv_heads > n_heads || context_length < 1)
    return fail(ctx, GLA_ERR_INVALID_ARG, "bad RoPE shape");
  if (head_dim != 64 && head_dim != 128)
    return fail(ctx, GLA_ERR_NOT_SUPPORTED, "Q8 cache: head_dim 64 or 128");
  if (rope_style != GLA_ROPE_INTERLEAVED && rope_style != GLA_ROPE_NEOX)
    return fail(ctx, GLA_ERR_INVALID_ARG, "unknown rope_style");
  if (!(theta > 0.f)) return fail(ctx, GLA_ERR_INVALID_ARG, "theta must be positive");
  DeviceGuard dg(ctx->device);
  std::string err;
  int rc = gla::launch_rope_append_q8(q, k, v, key_cache, value_cache, scales, n_heads, n_kv_heads,
                                      head_dim, position_holder, context_length, theta,
                                      rope_style, ctx->status, ctx->stream, &err);
  return rc == GLA_OK ? GLA_OK : fail(ctx, rc, err);
}

int32_t gla_decode_batched_f32kv(gla_ctx* ctx, const float* q, const float* const* k_ptrs,
                                 const float* const* v_ptrs, const int32_t* n_pos,
                                 int32_t max_n_pos, float* xb, int32_t batch, int32_t n_heads,
                                 int32_t n_kv_heads, int32_t head_dim, int64_t kv_stride,
                                 float scale) {
  return decode_batched(ctx, GLA_DTYPE_F32, q, reinterpret_cast<const void* const*>(k_ptrs),
                        reinterpret_cast<const void* const*>(v_ptrs), n_pos, max_n_pos, xb, batch,
                        n_heads, n_kv_heads, head_dim, kv_stride, scale);
}

int32_t gla_decode_batched_f16kv(gla_ctx* ctx, const float* q, const uint16_t* const* k_ptrs,
                                 const uint16_t* const* v_ptrs, const int32_t* n_pos,
                                 int32_t max_n_pos, float* xb, int32_t batch, int32_t n_heads,
                                 int32_t n_kv_heads, int32_t head_dim, int64_t kv_stride,
                                 float scale) {
  return decode_batched(ctx, GLA_DTYPE_F16, q, reinterpret_cast<const void* const*>(k_ptrs),
                        reinterpret_cast<const void* const*>(v_ptrs), n_pos, max_n_pos, xb, batch,
                        n_heads, n_kv_heads, head_dim, kv_stride, scale);
}

int32_t gla_decode_partial_f32kv(gla_ctx* ctx, const float* q, const float* k, const float* v,
                                 float* part, int32_t n_heads, int32_t n_kv_heads,
                                 int32_t head_dim, int64_t kv_stride, int32_t n_pos, float scale) {
  return decode_single(ctx, GLA_DTYPE_F32, q, k, v, part, n_heads, n_kv_heads, head_dim,
                       kv_stride, n_pos, scale, 1);
}

int32_t gla_decode_partial_f16kv(gla_ctx* ctx, const float* q, const uint16_t* k,
                                 const uint16_t* v, float* part, int32_t n_heads,
                                 int32_t n_kv_heads, int32_t head_dim, int64_t kv_stride,
                                 int32_t n_pos, float scale) {
  return decode_single(ctx, GLA_DTYPE_F16, q, k, v, part, n_heads, n_kv_heads, head_dim,
                       kv_stride, n_pos, scale, 1);
}

int32_t gla_lse_combine(gla_ctx* ctx, const float* parts, int32_t n_parts, int32_t n_heads,
                        int32_t head_dim, float* xb) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!parts || !xb) return fail(ctx, GLA_ERR_INVALID_ARG, "null pointer");
  if (n_parts < 1 || n_heads < 1 || head_dim < 1)
    return fail(ctx, GLA_ERR_INVALID_ARG, "n_parts, n_heads and head_dim must be positive");
  DeviceGuard dg(ctx->device);
  std::string err;
  int rc = gla::launch_lse_combine(parts, n_parts, n_heads, head_dim, xb, ctx->stream, &err);
  return rc == GLA_OK ? GLA_OK : fail(ctx, rc, err);
}

int32_t gla_comm_unique_id_size(void) { return gla::Comm::unique_id_size(); }

int32_t gla_comm_get_unique_id(void* unique_id) {
  if (!unique_id) return GLA_ERR_INVALID_ARG;
  std::string err;
  return gla::Comm::get_unique_id(unique_id, &err);
}

int32_t gla_comm_init(gla_ctx* ctx, int32_t nranks, int32_t rank, const void* unique_id) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!unique_id || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(ctx, GLA_ERR_INVALID_ARG, "bad communicator arguments");
  DeviceGuard dg(ctx->device);
  std::string err;
  quiesce_comm(ctx);  // a previous communicator: collective end of its use
  ctx->xch.teardown();
  int rc = ctx->comm.init(nranks, rank, unique_id, &err);
  if (rc != GLA_OK) return fail(ctx, rc, err);
  if (ctx->opt_shard_exchange && nranks > 1) {
    rc = ctx->xch.setup(ctx->comm, ctx->stream, &err);
    if (rc != GLA_OK) return fail(ctx, rc, err);
  }
  return GLA_OK;
}

int32_t gla_comm_peer_exchange(const gla_ctx* ctx) {
  return ctx && ctx->opt_shard_exchange && ctx->xch.active() ? 1 : 0;
}

int32_t gla_comm_wait(gla_ctx* ctx) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  DeviceGuard dg(ctx->device);
  std::string err;
  if (!ctx->comm.active()) {
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    return e == cudaSuccess ? GLA_OK : cuda_fail(ctx, e, "cudaStreamSynchronize");
  }
  int rc = ctx->comm.wait(ctx->stream, &err);
  if (rc != GLA_OK) {
    ctx->xch.teardown();  // the communicator was aborted
    return fail(ctx, rc, err);
  }
  return GLA_OK;
}

int32_t gla_comm_resync(gla_ctx* ctx) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!ctx->comm.active())
    return fail(ctx, GLA_ERR_COMM, "gla_comm_init has not been called on this context");
  DeviceGuard dg(ctx->device);
  std::string err;
  // 1. every rank's stream has drained: no kernel stores records any more
  int rc = ctx->comm.wait(ctx->stream, &err);
  if (rc == GLA_OK) rc = ctx->comm.barrier(ctx->stream, &err);
  // 2. records and epochs back to zero on every rank
  if (rc == GLA_OK) rc = ctx->xch.reset(ctx->stream, &err);
  int32_t* st = ctx->status;
  if (rc == GLA_OK && cudaMemsetAsync(st, 0, sizeof(int32_t), ctx->stream) != cudaSuccess) {
    cudaGetLastError();
    rc = GLA_ERR_CUDA;
    err = "status reset failed";
  }
  if (rc == GLA_OK && ctx->counters &&
      cudaMemsetAsync(ctx->counters, 0, ctx->counters_cap * sizeof(int32_t), ctx->stream) !=
          cudaSuccess) {
    cudaGetLastError();
    rc = GLA_ERR_CUDA;
    err = "counter reset failed";
  }
  // 3. nobody starts a new call before every rank has reset
  if (rc == GLA_OK) rc = ctx->comm.barrier(ctx->stream, &err);
  if (rc != GLA_OK) {
    if (!ctx->comm.active()) ctx->xch.teardown();
    return fail(ctx, rc, err);
  }
  return GLA_OK;
}

int32_t gla_decode_sharded_f16kv(gla_ctx* ctx, const float* q, const uint16_t* k,
                                 const uint16_t* v, float* xb, int32_t n_heads,
                                 int32_t n_kv_heads, int32_t head_dim, int64_t kv_stride,
                                 int32_t n_pos_local, float scale) {
  return sharded(ctx, GLA_DTYPE_F16, q, k, v, xb, n_heads, n_kv_heads, head_dim, kv_stride,
                 n_pos_local, scale);
}

int32_t gla_decode_sharded_f32kv(gla_ctx* ctx, const float* q, const float* k, const float* v,
                                 float* xb, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                 int64_t kv_stride, int32_t n_pos_local, float scale) {
  return sharded(ctx, GLA_DTYPE_F32, q, k, v, xb, n_heads, n_kv_heads, head_dim, kv_stride,
                 n_pos_local, scale);
}

int32_t gla_prefill_causal_f16(gla_ctx* ctx, const uint16_t* q, const uint16_t* k,
                               const uint16_t* v, float* out, int32_t L, int32_t n_heads,
                               int32_t n_kv_heads, int32_t head_dim, float scale) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!q || !k || !v || !out) return fail(ctx, GLA_ERR_INVALID_ARG, "null tensor pointer");
  if (L < 1 || n_heads < 1 || n_kv_heads < 1 || n_heads % n_kv_heads != 0)
    return fail(ctx, GLA_ERR_INVALID_ARG, "bad prefill shape");
  if (!std::isfinite(scale)) return fail(ctx, GLA_ERR_INVALID_ARG, "scale must be finite");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(ctx, GLA_ERR_ALIGNMENT, "prefill tensors must be 16-byte aligned");
  DeviceGuard dg(ctx->device);
  std::string err;
  int rc = gla::launch_prefill_f16(q, k, v, out, L, 0, (int64_t)n_kv_heads * head_dim, n_heads,
                                   n_kv_heads, head_dim, scale, ctx->status, ctx->dev,
                                   ctx->stream, &err);
  return rc == GLA_OK ? GLA_OK : fail(ctx, rc, err);
}

int32_t gla_rope_append_f32(gla_ctx* ctx, float* q, float* k, const float* v, float* key_cache,
                            float* value_cache, int32_t n_heads, int32_t n_kv_heads,
                            int32_t head_dim, const int32_t* position_holder, float theta,
                            int32_t rope_style) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!q || !k || !v || !key_cache || !value_cache || !position_holder)
    return fail(ctx, GLA_ERR_INVALID_ARG, "null pointer");
  if (n_heads < 1 || n_kv_heads < 1 || n_kv_heads > n_heads || head_dim < 2 || head_dim % 2)
    return fail(ctx, GLA_ERR_INVALID_ARG, "bad RoPE shape");
  if (rope_style != GLA_ROPE_INTERLEAVED && rope_style != GLA_ROPE_NEOX)
    return fail(ctx, GLA_ERR_INVALID_ARG, "unknown rope_style");
  if (!(theta > 0.f)) return fail(ctx, GLA_ERR_INVALID_ARG, "theta must be positive");
  DeviceGuard dg(ctx->device);
  std::string err;
  int rc = gla::launch_rope_append_f32(q, k, v, key_cache, value_cache, n_heads, n_kv_heads,
                                       head_dim, position_holder, theta, rope_style, ctx->stream,
                                       &err);
  return rc == GLA_OK ? GLA_OK : fail(ctx, rc, err);
}

namespace {

int ingest_prompt(gla_ctx* ctx, bool f16_cache, const float* q, const float* k, const float* v,
                  void* key_cache, void* value_cache, float* xb, int32_t start_pos,
                  int32_t n_rows, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                  int32_t context_length, float theta, int32_t rope_style) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!q || !k || !v || !key_cache || !value_cache || !xb)
    return fail(ctx, GLA_ERR_INVALID_ARG, "null pointer");
  if (n_rows < 1 || n_heads < 1 || n_kv_heads < 1 || n_heads % n_kv_heads != 0)
    return fail(ctx, GLA_ERR_INVALID_ARG, "bad ingestion shape");
  if (head_dim != 64 && head_dim != 96 && head_dim != 128)
    return fail(ctx, GLA_ERR_NOT_SUPPORTED, "prompt ingestion head_dim must be 64, 96 or 128");
  if (start_pos < 0 || context_length < 1 || (int64_t)start_pos + n_rows > context_length)
    return fail(ctx, GLA_ERR_INVALID_ARG, "positions past context_length");
  if (rope_style != GLA_ROPE_INTERLEAVED && rope_style != GLA_ROPE_NEOX)
    return fail(ctx, GLA_ERR_INVALID_ARG, "unknown rope_style");
  if (!(theta > 0.f)) return fail(ctx, GLA_ERR_INVALID_ARG, "theta must be positive");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(key_cache) ||
      !aligned16(value_cache))
    return fail(ctx, GLA_ERR_ALIGNMENT, "q, k, v and the caches must be 16-byte aligned");
  DeviceGuard dg(ctx->device);
  const size_t need = gla::ingest_workspace_halves(f16_cache, start_pos, n_rows, n_heads,
                                                   n_kv_heads, head_dim);
  if (need > ctx->ingest_cap) {
    if (stream_capturing(ctx->stream))
      return fail(ctx, GLA_ERR_INVALID_ARG,
                  "ingestion workspace must grow; run the largest call once before capture");
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaStreamSynchronize");
    cudaFree(ctx->ingest_ws);
    ctx->ingest_ws = nullptr;
    ctx->ingest_cap = 0;
    e = cudaMalloc(&ctx->ingest_ws, need * sizeof(uint16_t));
    if (e != cudaSuccess) {
      ctx->ingest_ws = nullptr;
      return cuda_fail(ctx, e, "cudaMalloc ingestion workspace");
    }
    ctx->ingest_cap = need;
  }
  std::string err;
  int rc = gla::launch_ingest(f16_cache, q, k, v, key_cache, value_cache, xb, ctx->ingest_ws,
                              start_pos, n_rows, n_heads, n_kv_heads, head_dim, theta,
                              rope_style, ctx->status, ctx->dev, ctx->stream, &err);
  return rc == GLA_OK ? GLA_OK : fail(ctx, rc, err);
}

}  // namespace

int32_t gla_wo_residual_f16(gla_ctx* ctx, const float* xb, float* x, const uint16_t* w, int32_t n,
                            int32_t d) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (!xb || !x || !w) return fail(ctx, GLA_ERR_INVALID_ARG, "null pointer");
  if (n < 8 || d < 1) return fail(ctx, GLA_ERR_INVALID_ARG, "bad wo shape");
  if (n % 8 != 0 || !aligned16(w) || !aligned16(xb))
    return fail(ctx, GLA_ERR_ALIGNMENT, "wo needs n % 8 == 0 and 16-byte aligned w and xb");
  DeviceGuard dg(ctx->device);
  std::string err;
  int rc = gla::launch_wo_residual_f16(w, xb, x, n, d, ctx->dev, ctx->stream, &err);
  return rc == GLA_OK ? GLA_OK : fail(ctx, rc, err);
}

int32_t gla_ingest_prompt_f32(gla_ctx* ctx, const float* q, const float* k, const float* v,
                              float* key_cache, float* value_cache, float* xb, int32_t start_pos,
                              int32_t n_rows, int32_t n_heads, int32_t n_kv_heads,
                              int32_t head_dim, int32_t context_length, float theta,
                              int32_t rope_style) {
  return ingest_prompt(ctx, false, q, k, v, key_cache, value_cache, xb, start_pos, n_rows,
                       n_heads, n_kv_heads, head_dim, context_length, theta, rope_style);
}

int32_t gla_ingest_prompt_f16kv(gla_ctx* ctx, const float* q, const float* k, const float* v,
                                uint16_t* key_cache, uint16_t* value_cache, float* xb,
                                int32_t start_pos, int32_t n_rows, int32_t n_heads,
                                int32_t n_kv_heads, int32_t head_dim, int32_t context_length,
                                float theta, int32_t rope_style) {
  return ingest_prompt(ctx, true, q, k, v, key_cache, value_cache, xb, start_pos, n_rows,
                       n_heads, n_kv_heads, head_dim, context_length, theta, rope_style);
}

int32_t gla_debug_advance_position(gla_ctx* ctx, int32_t* position_holder, int32_t delta,
                                   int32_t delay_us) {
  if (!ctx || !position_holder) return GLA_ERR_INVALID_ARG;
  DeviceGuard dg(ctx->device);
  std::string err;
  int rc = gla::launch_advance_position(position_holder, delta, delay_us, ctx->stream, &err);
  return rc == GLA_OK ? GLA_OK : fail(ctx, rc, err);
}

int32_t gla_debug_xch_loopback(gla_ctx* ctx, int32_t world) {
  if (!ctx) return GLA_ERR_INVALID_ARG;
  if (ctx->comm.active())
    return fail(ctx, GLA_ERR_INVALID_ARG, "the context has a communicator");
  DeviceGuard dg(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (world == 0) {
    ctx->xch.teardown();
    return GLA_OK;
  }
  std::string err;
  int rc = ctx->xch.setup_loopback(world, &err);
  return rc == GLA_OK ? GLA_OK : fail(ctx, rc, err);
}

int64_t gla_debug_trace(gla_ctx* ctx, uint64_t* out, int64_t capacity) {
  if (!ctx || !out || capacity < 0) return GLA_ERR_INVALID_ARG;
  if (!ctx->trace) return fail(ctx, GLA_ERR_INVALID_ARG, "tracing is off (GLA_OPT_TRACE)");
  DeviceGuard dg(ctx->device);
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaStreamSynchronize");
  const size_t n = std::min<size_t>((size_t)capacity, ctx->trace_words);
  e = cudaMemcpy(out, ctx->trace, n * sizeof(uint64_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMemcpy");
  return (int64_t)n;
}

int64_t gla_debug_partition(const int32_t* n_pos, int32_t n_seq, int32_t n_kv_heads, int32_t tile,
                            int32_t unit_rows, int32_t n_ctas, int32_t* cta, int32_t* seq,
                            int32_t* kv_head, int32_t* row0, int32_t* rows, int32_t* slot,
                            int32_t* first_cta, int32_t* npieces, int64_t capacity) {
  if (!n_pos || n_seq < 1 || n_kv_heads < 1 || n_ctas < 1 || unit_rows < 1 || tile < unit_rows ||
      tile % unit_rows != 0)
    return GLA_ERR_INVALID_ARG;
  std::vector<int32_t> nunits(n_seq), start(n_seq + 1), np(n_seq);
  int64_t acc = 0;
  for (int b = 0; b < n_seq; ++b) {
    np[b] = n_pos[b] < 0 ? 0 : n_pos[b];
    nunits[b] = gla::ceil_div(np[b], unit_rows);
    start[b] = (int32_t)(acc * n_kv_heads);
    acc += nunits[b];
  }
  start[n_seq] = (int32_t)(acc * n_kv_heads);
  const gla::Deal deal = gla::make_deal(start[n_seq], n_ctas, n_seq, n_kv_heads, nunits[0]);
  // walk each CTA's tiles exactly as the kernel's producer and consumers do
  int64_t n = 0;
  for (int32_t c = 0; c < n_ctas; ++c) {
    gla::CtaTiles ct = gla::cta_tiles_of(deal, c, start.data(), nunits.data(), n_seq);
    gla::Tile t;
    while (ct.next(nunits.data(), n_seq, n_kv_heads, tile / unit_rows, unit_rows, t)) {
      if (n >= capacity) return GLA_ERR_INVALID_ARG;
      cta[n] = c;
      seq[n] = t.b;
      kv_head[n] = t.g;
      row0[n] = t.row0;
      rows[n] = std::min(t.units * unit_rows, np[t.b] - t.row0);
      slot[n] = c + t.b * n_kv_heads + t.g;
      int32_t c0;
      const int32_t np_ = deal.pieces(start.data(), nunits.data(), t.b, t.g, &c0);
      first_cta[n] = c0;
      npieces[n] = np_;
      ++n;
    }
  }
  return n;
}

}  // extern "C"
