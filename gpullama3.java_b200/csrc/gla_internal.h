// gla_internal.h - interfaces between the C ABI layer (api.cu) and the kernel
// launchers.  Not installed; not part of the ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace gla {

// Everything a decode launch needs besides pointers checked by the caller.
struct DecodeRequest {
  int dtype;                   // GLA_DTYPE_F32 / GLA_DTYPE_F16 / GLA_DTYPE_Q8
  const float* q;
  const void* k;
  const void* v;
  const void* scales = nullptr;  // Q8: [rows][n_kv][8] halves (K, V block scales)
  const void* const* k_ptrs;
  const void* const* v_ptrs;
  int64_t kv_stride;
  const int32_t* n_pos_dev;
  int32_t n_pos;               // scalar rows (n_pos_dev == nullptr)
  int32_t n_pos_add;
  int32_t n_pos_cap;
  int32_t max_n_pos;           // host bound used to choose the tile
  int32_t batch;
  int32_t n_heads;
  int32_t n_kv;
  int32_t head_dim;
  float scale;
  float* out;
  int32_t record_mode;
  int32_t early_kv;            // GLA_OPT_EARLY_KV_PREFETCH value (0, 1 or 2)
  // record_mode 2 (peer exchange of a sharded sequence; gla_xch.h)
  const uint64_t* xch_bases = nullptr;  // device [world]
  char* xch_local = nullptr;
  float* xch_out = nullptr;
  int32_t xch_world = 0;
  int32_t xch_rank = 0;
  // fused RoPE + append (FP32 cache, one sequence, device position)
  int32_t rope = 0;
  int32_t rope_style = 0;
  double rope_theta = 0.0;
  const float* rope_k = nullptr;
  const float* rope_v = nullptr;
};

// Launch geometry chosen for a request.
struct DecodePlan {
  int32_t loader;              // 0: tensor-map loader (round-robin deal), 1: cp.async loader
  int32_t tile;
  int32_t stages;
  int32_t grid;
  int32_t threads;
  size_t smem;
  size_t part_words;           // workspace 64-bit words for piece slots (zeroed when allocated)
  size_t counters;             // workspace counters (zero between calls)
};

// Words of the per-CTA phase trace of a decode launch (DecodeWorkspace::trace).
constexpr int kTraceWordsPerCta = 16;

// Device memory a decode launch uses besides its inputs and outputs.
struct DecodeWorkspace {
  uint64_t* part = nullptr;        // plan.part_words tagged piece words, zeroed at allocation
  int32_t* counter = nullptr;      // plan.counters piece counters, zero between calls
  unsigned long long* epoch = nullptr;  // one word: call epoch << 32 | tickets of this call
  int32_t* status = nullptr;       // device status word
  uint64_t* trace = nullptr;       // optional [grid][16] phase stamps
};

// Device properties a plan depends on.
struct DeviceInfo {
  int sms;
  int smem_optin;              // max dynamic shared memory per block
  int smem_per_sm = 0;         // shared memory of an SM (0: plan one CTA an SM)
};

// Fills `plan` for `req`; returns GLA_OK or an error code with *err set.
int plan_decode(const DecodeRequest& req, const DeviceInfo& dev, DecodePlan* plan,
                std::string* err);

// Launches the decode kernel with a plan from plan_decode.
int launch_decode(const DecodeRequest& req, const DecodePlan& plan, const DecodeWorkspace& ws,
                  cudaStream_t stream, std::string* err);

// Log-sum-exp merge of records [n_parts][n_heads][head_dim+2] into xb.
int launch_lse_combine(const float* parts, int32_t n_parts, int32_t n_heads, int32_t head_dim,
                       float* xb, cudaStream_t stream, std::string* err);

// RoPE rotation of q/k at *position_holder followed by the KV append.
int launch_rope_append_f32(float* q, float* k, const float* v, float* key_cache,
                           float* value_cache, int32_t n_heads, int32_t n_kv_heads,
                           int32_t head_dim, const int32_t* position_holder, float theta,
                           int32_t rope_style, cudaStream_t stream, std::string* err);

// Causal prefill (tcgen05): L query rows at positions q_off..q_off+L-1 over
// key/value rows 0..q_off+L-1 (row stride kv_stride halves).
int launch_prefill_f16(const uint16_t* q, const uint16_t* k, const uint16_t* v, float* out,
                       int32_t L, int32_t q_off, int64_t kv_stride, int32_t n_heads,
                       int32_t n_kv_heads, int32_t head_dim, float scale, int32_t* status,
                       const DeviceInfo& dev, cudaStream_t stream, std::string* err);

// Q8 cache rows from FP32 K/V rows (q8.cu); scales [rows][n_kv][8] halves.
int launch_quantize_q8(const float* k, const float* v, int64_t src_stride, int32_t n_rows,
                       int32_t n_kv, int32_t hd, int8_t* kq, int8_t* vq, int64_t kv_stride,
                       uint16_t* scales, cudaStream_t stream, std::string* err);

// RoPE of the new token + its k/v quantised into a Q8 cache row (q8.cu).
int launch_rope_append_q8(float* q, float* k, const float* v, int8_t* kq, int8_t* vq,
                          uint16_t* scales, int32_t n_heads, int32_t n_kv, int32_t hd,
                          const int32_t* position_holder, int32_t context_length, float theta,
                          int32_t rope_style, int32_t* status, cudaStream_t stream,
                          std::string* err);

// Output projection + residual (wo.cu): x[i] += w[i][:] . xb, w FP16 [d][n].
int launch_wo_residual_f16(const uint16_t* w, const float* xb, float* x, int32_t n, int32_t d,
                           const DeviceInfo& dev, cudaStream_t stream, std::string* err);

// Batched prompt ingestion of one layer (ingest.cu): RoPE, KV append and
// causal attention of n_rows positions from start_pos.  ws holds
// ingest_workspace_halves(...) halves, 16-byte aligned.
size_t ingest_workspace_halves(bool f16_cache, int32_t start_pos, int32_t n_rows,
                               int32_t n_heads, int32_t n_kv_heads, int32_t head_dim);
int launch_ingest(bool f16_cache, const float* q, const float* k, const float* v, void* key_cache,
                  void* value_cache, float* xb, uint16_t* ws, int32_t start_pos, int32_t n_rows,
                  int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, float theta,
                  int32_t rope_style, int32_t* status, const DeviceInfo& dev,
                  cudaStream_t stream, std::string* err);

// Test hook (debug.cu): a PDL kernel that releases its dependents at once,
// spins delay_us (at most 1000) and then adds delta to *position_holder.
int launch_advance_position(int32_t* position_holder, int32_t delta, int32_t delay_us,
                            cudaStream_t stream, std::string* err);

}  // namespace gla
