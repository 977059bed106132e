/*
 * gpullama_attn.h - C ABI of libgpullama_attn, a B200 (sm_100a) attention
 * library that replaces the per-layer attention task of GPULlama3.java.
 *
 * Conventions (all entry points):
 *  - Every tensor pointer is a caller-owned DEVICE pointer on the context's
 *    device (Java passes MemorySegment.address() of a device segment).
 *  - Calls are asynchronous and ordered on the context's CUDA stream.
 *  - Return value: GLA_OK (0) or a negative GLA_ERR_* code.  Nothing aborts and
 *    no C++ exception crosses the ABI.  gla_last_error() describes the last
 *    failure of a context.  Errors found by a kernel while it runs (a bounded
 *    wait that gave up) are latched in a device status word that
 *    gla_device_status() reads back.
 *  - A context is not thread-safe: use one per (device, host thread).
 *  - All element offsets are 64-bit.
 *  - Layouts follow the reference:
 *      q   [n_heads][head_dim]              FP32 (one token)
 *      K/V [position][kv_stride] per layer  (kv_stride = n_kv_heads*head_dim
 *                                            for the reference layout)
 *      xb  [n_heads][head_dim]              FP32
 *    q head h reads kv head h / (n_heads / n_kv_heads)  (GQA, kvMul).
 *  - FP16 tensors are IEEE binary16 passed as uint16_t.
 */
#ifndef GPULLAMA_ATTN_H
#define GPULLAMA_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GLA_VERSION 100 /* 1.0.0 */

/* status codes */
#define GLA_OK 0
#define GLA_ERR_INVALID_ARG (-1)   /* null pointer, bad size, bad shape        */
#define GLA_ERR_CUDA (-2)          /* a CUDA runtime call failed              */
#define GLA_ERR_NOT_SUPPORTED (-3) /* shape outside the compiled variants      */
#define GLA_ERR_ALIGNMENT (-4)     /* pointer/stride not 16-byte aligned       */
#define GLA_ERR_TIMEOUT (-5)       /* a bounded device or host wait gave up    */
#define GLA_ERR_COMM (-6)          /* NCCL failure or communicator missing     */
#define GLA_ERR_NO_DEVICE (-7)     /* no CUDA device / wrong device id         */
#define GLA_ERR_OUT_OF_MEMORY (-8) /* device allocation failed                 */

/* element types */
#define GLA_DTYPE_F32 0
#define GLA_DTYPE_F16 1
#define GLA_DTYPE_Q8 2 /* int8 values + FP16 scale per 32 (see gla_decode_q8kv) */

typedef struct gla_ctx gla_ctx;

/* ------------------------------------------------------------------------ */
/* Library / context                                                         */
/* ------------------------------------------------------------------------ */

/* Library version (GLA_VERSION of the build). */
int32_t gla_version(void);

/* Human-readable name of a status code (static string). */
const char* gla_status_string(int32_t status);

/* Creates a context on `device` that launches on `cuda_stream` (a cudaStream_t;
 * NULL = the legacy default stream).  Allocates the context's device
 * workspace.  Replaces the per-plan device set-up of
 * tornadovm/TornadoVMMasterPlan.java:37-79 (initializeTornadoVMPlan) for the
 * attention task. */
int32_t gla_create(int32_t device, void* cuda_stream, gla_ctx** out);

/* Frees the context, its workspace and its communicator (if any).
 * Collective for a context with a communicator (gla_comm_init): every rank
 * calls it; the ranks meet at a bounded barrier before the peer exchange
 * buffers that other ranks store into are unmapped and freed.  Returns
 * GLA_ERR_TIMEOUT (after freeing everything) if a rank did not arrive within
 * the communicator timeout. */
int32_t gla_destroy(gla_ctx* ctx);

/* Re-targets the context to another stream of the same device. */
int32_t gla_set_stream(gla_ctx* ctx, void* cuda_stream);

/* Message of the context's last failure ("" if none).  Valid until the next
 * call on the context. */
const char* gla_last_error(const gla_ctx* ctx);

/* Synchronises the context's stream, then returns (and clears) the device
 * status word that kernels set when a bounded wait gives up
 * (GLA_OK or GLA_ERR_TIMEOUT), or GLA_ERR_CUDA if the stream itself failed. */
int32_t gla_device_status(gla_ctx* ctx, int32_t* device_status);

/* Grows the context workspace so that later decode calls of up to
 * `max_batch` sequences x `max_kv_heads` KV heads x `max_heads` q heads of
 * `max_head_dim` never allocate (call before CUDA-graph capture). */
int32_t gla_reserve(gla_ctx* ctx, int32_t max_batch, int32_t max_kv_heads, int32_t max_heads,
                    int32_t max_head_dim);

/* Number of streaming multiprocessors of the context's device. */
int32_t gla_num_sms(const gla_ctx* ctx);

/* Context options (gla_set_option). */
#define GLA_OPT_EARLY_KV_PREFETCH 1
/* GLA_OPT_EARLY_KV_PREFETCH (default 2).  Decode calls launch with
 * programmatic dependent launch and may start copying K/V tiles before the
 * kernel issued just before them on the stream has finished - only if that
 * kernel releases its dependents early (griddepcontrol.launch_dependents).
 * Which tiles a CTA copies does not depend on the length (kv head g's tiles
 * are dealt round robin to its CTA group); the length only bounds how many
 * are copied early:
 *   1 - calls that take n_pos from the host (gla_decode_*,
 *       gla_decode_partial_*, gla_decode_sharded_*);
 *   2 - also calls that read the position on the device
 *       (gla_process_heads_flash_attention*, gla_rope_append_attention_f32),
 *       which use the position read before the wait only as a hint: copies
 *       past the true length are dropped, tiles it does not cover are copied
 *       after the wait.
 * After the wait the two newest rows [n_pos - 2, n_pos) of every early tile
 * are read again (or, fused RoPE, the newest written), so a preceding kernel
 * that releases its dependents early may write the position holder and the
 * cache rows n_pos - 2 and n_pos - 1 (a KV append, the previous token's fused
 * append on the same cache); q and the workspace are read after the wait.
 * Use 0 if such a kernel writes older cache rows.  (Early copies apply to
 * single-sequence calls.) */
#define GLA_OPT_COMM_TIMEOUT_MS 3
/* GLA_OPT_COMM_TIMEOUT_MS (default 60000): host deadline of every step that
 * waits for other ranks - joining the communicator, enqueueing a collective,
 * gla_comm_wait / gla_device_status on a context with a communicator,
 * gla_comm_resync and the barrier of gla_destroy.  Past it the NCCL
 * communicator is aborted (ncclCommAbort ends its kernels), the call returns
 * GLA_ERR_TIMEOUT and sharded decode needs gla_comm_init again.  No
 * reference counterpart (the reference is single-device). */
#define GLA_OPT_TRACE 4
/* GLA_OPT_TRACE (default 0): 1 = every single-sequence or sharded decode
 * call on the context (batched calls leave none) writes
 * %globaltimer stamps of its phases (16 words per CTA: entry, dependency
 * wait, q loaded, first tile, last tile, piece counted, merged, published,
 * producer first/last copy, info, exit), read back with gla_debug_trace.
 * Turn it on outside stream capture.  No reference counterpart (the
 * reference's TornadoVM profiler flags, llama-tornado:93-134, time whole
 * tasks). */
#define GLA_OPT_SHARD_EXCHANGE 2
/* GLA_OPT_SHARD_EXCHANGE (default 1): 1 = sharded decode merges over the
 * peer exchange when gla_comm_init could set it up, 0 = always the NCCL
 * all-gather.  Set it to the same value on every rank (before
 * gla_comm_init to skip the mapping). */
int32_t gla_set_option(gla_ctx* ctx, int32_t option, int32_t value);

/* ------------------------------------------------------------------------ */
/* KV cache allocation (device MemorySegments of State)                      */
/* ------------------------------------------------------------------------ */

/* Allocates zero-initialised key and value caches of
 * n_layers * context_length * kv_dim elements of `dtype` each, laid out
 * [layer][position][kv_dim] like the flat wrapKeyCache/wrapValueCache of the
 * reference (inference/state/LlamaState.java:61-64, State.java:56-57), with
 * the per-layer CPU layout [position][kv_dim] (State.java:41-42) as each
 * layer's slice.  Replaces the zero-initialised host arrays that TornadoVM
 * copies to the device once (layers/type/fp16/LlamaFP16FFNLayers.java:145-165). */
int32_t gla_kv_cache_alloc(gla_ctx* ctx, int32_t n_layers, int32_t context_length, int32_t kv_dim,
                           int32_t dtype, void** key_cache, void** value_cache);

/* Frees caches from gla_kv_cache_alloc. */
int32_t gla_kv_cache_free(gla_ctx* ctx, void* key_cache, void* value_cache);

/* ------------------------------------------------------------------------ */
/* The reference task, argument for argument                                 */
/* ------------------------------------------------------------------------ */

/* Drop-in for the TornadoVM task "parallel-attention"
 *   TransformerComputeKernelsLayered.processHeadsFlashAttention(
 *       context, q, key_cache, value_cache, xb, nHeads, headSize, kvDim, kvMul,
 *       positionHolder, layer, contextLength)
 * (tornadovm/kernels/TransformerComputeKernelsLayered.java:336-458, wired at
 * tornadovm/layers/type/fp16/LlamaFP16FFNLayers.java:167-177).
 *  key_cache/value_cache: flat FP32 [layer][contextLength][kvDim] caches.
 *  position_holder: DEVICE int32 whose element 0 is the current position
 *  (IntArray positionHolder, State.java:58); attention covers positions
 *  0..position inclusive.  Scale is 1/sqrt(headSize) (InferenceCore.java:65,121).
 *  Because the position is read on the device, the call can be captured in a
 *  CUDA graph and replayed for every token. */
int32_t gla_process_heads_flash_attention(gla_ctx* ctx, const float* q, const float* key_cache,
                                          const float* value_cache, float* xb, int32_t n_heads,
                                          int32_t head_size, int32_t kv_dim, int32_t kv_mul,
                                          const int32_t* position_holder, int32_t layer,
                                          int32_t context_length);

/* One layer's attention step of a token in one launch: RoPE on q and on
 * the new key (as gla_rope_append_f32), the new key and value rows written
 * at row `position` of this layer's caches, then the attention of
 * gla_process_heads_flash_attention over rows 0..position -- the same bits
 * as those two calls in a row.  q and k are read, not rotated in place.
 * Replaces the rope, copyToCache and parallel-attention tasks of one layer
 * (TransformerComputeKernelsLayered.java:129-139, :179-205, :336-458); no
 * single reference counterpart.  k, v: [kvDim] rows of the new token; q, k,
 * v, the caches and xb 16-byte aligned. */
int32_t gla_rope_append_attention_f32(gla_ctx* ctx, const float* q, const float* k,
                                      const float* v, float* key_cache, float* value_cache,
                                      float* xb, int32_t n_heads, int32_t head_size,
                                      int32_t kv_dim, int32_t kv_mul,
                                      const int32_t* position_holder, int32_t layer,
                                      int32_t context_length, float theta, int32_t rope_style);

/* Same task over an FP16 cache (new capability; the reference KV is FP32). */
int32_t gla_process_heads_flash_attention_f16kv(gla_ctx* ctx, const float* q,
                                                const uint16_t* key_cache,
                                                const uint16_t* value_cache, float* xb,
                                                int32_t n_heads, int32_t head_size, int32_t kv_dim,
                                                int32_t kv_mul, const int32_t* position_holder,
                                                int32_t layer, int32_t context_length);

/* ------------------------------------------------------------------------ */
/* Decode attention (one new token per sequence), explicit pointers          */
/* ------------------------------------------------------------------------ */

/* Single-sequence decode over an FP32 cache.  k/v point at the LAYER base
 * (row 0); row t of kv head g starts at k + t*kv_stride + g*head_dim.
 * n_pos = position + 1 rows are attended.  scale multiplies q.k (the
 * reference divides by sqrt(head_dim): InferenceCore.java:121).
 * Replaces the CPU block InferenceCore.java:105-144 (forwardJava; also
 * forwardJavaQwen2 :233-272, forwardJavaQwen3 :375-407, forwardJavaPhi3
 * :495-517) and the GPU kernels TransformerComputeKernelsLayered.java:336-458,
 * :463-628, :278-334/:1091-1103, Qwen2Kernels.java:10-130,
 * Qwen3Kernels.java:193-293. */
int32_t gla_decode_f32kv(gla_ctx* ctx, const float* q, const float* k, const float* v, float* xb,
                         int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int64_t kv_stride,
                         int32_t n_pos, float scale);

/* Same over an FP16 cache; FP32 softmax and accumulation. */
int32_t gla_decode_f16kv(gla_ctx* ctx, const float* q, const uint16_t* k, const uint16_t* v,
                         float* xb, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                         int64_t kv_stride, int32_t n_pos, float scale);

/* Q8 cache (an addition: the reference's caches are FP32; the block shape is
 * that of its quantised weight type Q8_0, tensor/GGMLType.java:13):
 *   k, v    int8 [n_pos][kv_stride] (kv head g at column g*head_dim),
 *   scales  FP16 bits [n_pos][n_kv_heads][8]: the K scales of the head row's
 *           32-value blocks at [0, head_dim/32), the V scales at [4, ...);
 * element = q * (float)scale.  Attention is computed on those values with FP32
 * accuracy (int8 values and hi/lo-split q and p on FP16 tensor cores, scales
 * applied in FP32).  head_dim 64 or 128; kv_stride a multiple of 16; k, v,
 * scales, q, xb 16-byte aligned.  Half the bytes of an FP16 cache. */
int32_t gla_decode_q8kv(gla_ctx* ctx, const float* q, const int8_t* k, const int8_t* v,
                        const uint16_t* scales, float* xb, int32_t n_heads, int32_t n_kv_heads,
                        int32_t head_dim, int64_t kv_stride, int32_t n_pos, float scale);

/* Quantises n_rows FP32 rows of K and V ([n_rows][src_stride], n_kv_heads heads of
 * head_dim) into Q8 cache rows: per 32-value block d = amax/127, q = roundf(x/d)
 * computed as x * (1/d), d stored as FP16 (GGML's Q8_0 reference quantiser).
 * kq/vq/scales point at the first destination row. */
int32_t gla_kv_quantize_q8(gla_ctx* ctx, const float* k, const float* v, int64_t src_stride,
                           int32_t n_rows, int32_t n_kv_heads, int32_t head_dim, int8_t* kq,
                           int8_t* vq, int64_t kv_stride, uint16_t* scales);

/* Zero-initialised Q8 caches for n_layers layers (the Q8 counterpart of
 * gla_kv_cache_alloc, i.e. of the State allocation, state/LlamaState.java:45-46):
 * k, v int8 [layer][context_length][n_kv_heads*head_dim], scales FP16
 * [layer][context_length][n_kv_heads][8]; layer l starts at
 * l*context_length*n_kv_heads*head_dim (values) and l*context_length*n_kv_heads*8
 * (scales).  head_dim 64 or 128. */
int32_t gla_kv_cache_alloc_q8(gla_ctx* ctx, int32_t n_layers, int32_t context_length,
                              int32_t n_kv_heads, int32_t head_dim, int8_t** key_cache,
                              int8_t** value_cache, uint16_t** scales);
int32_t gla_kv_cache_free_q8(gla_ctx* ctx, int8_t* key_cache, int8_t* value_cache,
                             uint16_t* scales);

/* The new token into a Q8 cache layer: RoPE of q and k in place as
 * gla_rope_append_f32 does (same bits), then k and v quantised (as
 * gla_kv_quantize_q8) into row position_holder[0] of the layer's
 * key_cache/value_cache [context_length][kv_dim] and scales
 * [context_length][n_kv_heads][8].  A position outside [0, context_length)
 * writes nothing and latches GLA_ERR_INVALID_ARG in the device status. */
int32_t gla_rope_append_q8(gla_ctx* ctx, float* q, float* k, const float* v, int8_t* key_cache,
                           int8_t* value_cache, uint16_t* scales, int32_t n_heads,
                           int32_t n_kv_heads, int32_t head_dim, const int32_t* position_holder,
                           int32_t context_length, float theta, int32_t rope_style);

/* Batched decode: `batch` independent sequences, one new token each.
 *  q  [batch][n_heads][head_dim], xb [batch][n_heads][head_dim]
 *  k_ptrs/v_ptrs: DEVICE arrays of `batch` layer-base pointers
 *  n_pos: DEVICE int32 array [batch] (rows attended per sequence, >= 1)
 *  max_n_pos: host upper bound of n_pos[] (used only to pick the tile size).
 * No reference counterpart for batch > 1 (the reference decodes one
 * sequence: inference/InferenceEngine.java:67-141); each sequence computes
 * exactly what gla_decode_*kv computes for it. */
int32_t gla_decode_batched_f32kv(gla_ctx* ctx, const float* q, const float* const* k_ptrs,
                                 const float* const* v_ptrs, const int32_t* n_pos,
                                 int32_t max_n_pos, float* xb, int32_t batch, int32_t n_heads,
                                 int32_t n_kv_heads, int32_t head_dim, int64_t kv_stride,
                                 float scale);
int32_t gla_decode_batched_f16kv(gla_ctx* ctx, const float* q, const uint16_t* const* k_ptrs,
                                 const uint16_t* const* v_ptrs, const int32_t* n_pos,
                                 int32_t max_n_pos, float* xb, int32_t batch, int32_t n_heads,
                                 int32_t n_kv_heads, int32_t head_dim, int64_t kv_stride,
                                 float scale);

/* Partial decode over one contiguous KV shard (rows [0, n_pos) of k/v, which
 * hold some range of the global sequence).  Instead of xb it writes, per q
 * head h, the record part[h][0..head_dim+2):
 *     part[h][0..head_dim)  = sum_t exp(s_t - m) v_t / l   (normalised o)
 *     part[h][head_dim]     = m = max_t s_t                (natural log units)
 *     part[h][head_dim + 1] = l = sum_t exp(s_t - m)
 * where s_t = scale * q_h . k_t.  Records of disjoint shards merge exactly
 * with gla_lse_combine.  No reference counterpart (the reference is single
 * device, SchedulerDetectionService.java:13-26). */
int32_t gla_decode_partial_f32kv(gla_ctx* ctx, const float* q, const float* k, const float* v,
                                 float* part, int32_t n_heads, int32_t n_kv_heads,
                                 int32_t head_dim, int64_t kv_stride, int32_t n_pos, float scale);
int32_t gla_decode_partial_f16kv(gla_ctx* ctx, const float* q, const uint16_t* k,
                                 const uint16_t* v, float* part, int32_t n_heads,
                                 int32_t n_kv_heads, int32_t head_dim, int64_t kv_stride,
                                 int32_t n_pos, float scale);

/* Log-sum-exp merge of `n_parts` record sets parts[n_parts][n_heads][head_dim+2]
 * (layout above) into xb[n_heads][head_dim]:
 *     M = max_i m_i,  w_i = l_i exp(m_i - M),  xb = sum_i w_i o_i / sum_i w_i.
 * Records with l = 0 (empty shards) are ignored. */
int32_t gla_lse_combine(gla_ctx* ctx, const float* parts, int32_t n_parts, int32_t n_heads,
                        int32_t head_dim, float* xb);

/* Allocation-free FP32-cache decode.  No counterpart in the reference: it
 * serves callers that cannot allocate device memory where they need
 * attention (buffers owned by another runtime such as TornadoVM, allocators
 * that forbid growth mid-step, embedders that must not call cudaMalloc/cudaFree
 * because those synchronise the device) - gla_create allocates, this does not.
 * Same arguments and result as gla_decode_f32kv, on the CURRENT device and on
 * `cuda_stream` (a cudaStream_t; NULL = legacy default stream); no context.
 * Scratch: a fixed 1 MiB + 8 KiB static device array of the library, held by
 * every GPU that loads it until exit.  The first call on a device looks up
 * that array's address (cudaGetSymbolAddress): make it before any stream
 * capture.  Limits: (number of SMs + n_kv_heads) * kvMul * (head_dim + 4)
 * floats of partial records must fit in 1 MiB and n_kv_heads <= 1024, else
 * GLA_ERR_NOT_SUPPORTED; head_dim 64/96/128 and kvMul <= 8 as for
 * gla_decode_f32kv.  Every call shares the array (each call clears the
 * counters it uses first), so calls whose kernels overlap on the GPU race.
 * A bounded device wait that gives up is not reported (there is no context
 * to read it from). */
int32_t gla_decode_f32kv_noalloc(const float* q, const float* k, const float* v, float* xb,
                                 int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                 int64_t kv_stride, int32_t n_pos, float scale,
                                 void* cuda_stream);

/* ------------------------------------------------------------------------ */
/* Multi-GPU: KV-sequence sharded decode over NCCL                           */
/* ------------------------------------------------------------------------ */

/* Size in bytes of the opaque unique id used by gla_comm_init (ncclUniqueId). */
int32_t gla_comm_unique_id_size(void);

/* Writes a fresh unique id (rank 0 creates it and shares it out of band). */
int32_t gla_comm_get_unique_id(void* unique_id);

/* Joins an NCCL communicator of `nranks` ranks, one per GPU.  Collective.
 * With GLA_OPT_SHARD_EXCHANGE on (the default) it also maps every rank's
 * peer exchange buffer into every rank (CUDA IPC; the NCCL communicator
 * carries the handles); the exchange is used only if every rank succeeded. */
int32_t gla_comm_init(gla_ctx* ctx, int32_t nranks, int32_t rank, const void* unique_id);

/* 1 if sharded decode on this context runs the peer exchange, 0 if it uses
 * the NCCL all-gather.  No reference counterpart (introspection). */
int32_t gla_comm_peer_exchange(const gla_ctx* ctx);

/* Host watchdog: waits until the context's stream has drained, at most
 * GLA_OPT_COMM_TIMEOUT_MS.  A collective still waiting for a rank at the
 * deadline (a rank left, or skipped a call) is ended by aborting the
 * communicator: returns GLA_ERR_TIMEOUT and the context needs gla_comm_init
 * again (collectively, with the ranks still present).  Without a
 * communicator: a plain stream synchronisation.  No reference counterpart. */
int32_t gla_comm_wait(gla_ctx* ctx);

/* Collective recovery of the peer exchange after a sharded call returned
 * GLA_ERR_TIMEOUT in the device status (a rank skipped or lost a call, so
 * the ranks' per-kv-head call epochs differ): every rank drains its stream,
 * meets at a barrier, zeroes its exchange buffer (records and epochs), the
 * device status and the piece counters, and meets again.  Later calls
 * start from matching epochs.  Bounded like gla_comm_wait.  No reference
 * counterpart. */
int32_t gla_comm_resync(gla_ctx* ctx);

/* Decode of one sequence whose KV rows are sharded across the communicator's
 * ranks (this rank holds n_pos_local >= 0 rows).  Every rank ends with the
 * full xb.  Peer exchange (gla_comm_peer_exchange() == 1): one kernel
 * computes the shard's per-head records, stores them into every rank's
 * exchange buffer over NVLink, raises a flag per (rank, kv head) and merges
 * all ranks' records as they arrive (bounded waits: a rank that does not
 * take part within 1 s latches GLA_ERR_TIMEOUT).  Otherwise: partial record
 * kernel, NCCL all-gather, merge kernel.  Every rank must make the same
 * sequence of calls with the same shapes; capturable in a CUDA graph on the
 * peer path.  Needs gla_comm_init first. */
int32_t gla_decode_sharded_f16kv(gla_ctx* ctx, const float* q, const uint16_t* k,
                                 const uint16_t* v, float* xb, int32_t n_heads,
                                 int32_t n_kv_heads, int32_t head_dim, int64_t kv_stride,
                                 int32_t n_pos_local, float scale);
int32_t gla_decode_sharded_f32kv(gla_ctx* ctx, const float* q, const float* k, const float* v,
                                 float* xb, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                 int64_t kv_stride, int32_t n_pos_local, float scale);

/* ------------------------------------------------------------------------ */
/* Causal prefill (tcgen05 / TMEM)                                           */
/* ------------------------------------------------------------------------ */

/* Causal attention of a whole prompt: for every row p in [0, L) and head h,
 *   out[p][h] = softmax_t<=p(scale * q[p][h] . k[t][h/kvMul]) . v[t][h/kvMul]
 * q [L][n_heads*head_dim], k/v [L][n_kv_heads*head_dim] FP16 (row strides are
 * the packed widths), out [L][n_heads*head_dim] FP32.  Mathematically the
 * reference's prompt ingestion, which runs decode attention at positions
 * 0..L-1 one token at a time (inference/InferenceEngine.java:88-99, :309-327). */
int32_t gla_prefill_causal_f16(gla_ctx* ctx, const uint16_t* q, const uint16_t* k,
                               const uint16_t* v, float* out, int32_t L, int32_t n_heads,
                               int32_t n_kv_heads, int32_t head_dim, float scale);

/* Batched prompt ingestion of one layer: positions start_pos..start_pos+n_rows-1
 * at once.  The reference ingests a prompt one position at a time
 * (inference/InferenceEngine.java:88-99 CPU, :309-327 GPU), each position running
 * RoPE (InferenceCore.java:82-94 / :210-225), the KV append (:99-100) and the
 * attention block (:105-144); this call does the three for all rows, given the
 * rows of a batched QKV projection:
 *   q  [n_rows][n_heads*head_dim], k and v [n_rows][kv_dim] FP32, read only (the
 *      reference's in-place rotation of state.q/state.k is an intermediate that
 *      nothing reads after the attention block);
 *   key_cache/value_cache: the layer's [context_length][kv_dim] cache; rows
 *      start_pos+i receive k rotated for position start_pos+i and v (FP32, or
 *      FP16 for _f16kv), rows
 *      0..start_pos-1 hold earlier chunks (a prompt may be ingested in chunks);
 *   xb [n_rows][n_heads*head_dim] FP32: row i = attention of position start_pos+i
 *      over cache rows 0..start_pos+i, scale 1/sqrt(head_dim).
 * RoPE as gla_rope_append_f32 (same frequencies, same rounding: the cache rows
 * equal those of n_rows single-position calls).  Attention runs on the tcgen05
 * prefill kernel with FP16 operands (q, k, v rounded to FP16; FP32 softmax and
 * accumulation): the FP16 error bound applies to both variants, and both give
 * bit-identical xb.  head_dim 64, 96 or 128.  Uses a context workspace grown on
 * first use (not during stream capture). */
int32_t gla_ingest_prompt_f32(gla_ctx* ctx, const float* q, const float* k, const float* v,
                              float* key_cache, float* value_cache, float* xb, int32_t start_pos,
                              int32_t n_rows, int32_t n_heads, int32_t n_kv_heads,
                              int32_t head_dim, int32_t context_length, float theta,
                              int32_t rope_style);
int32_t gla_ingest_prompt_f16kv(gla_ctx* ctx, const float* q, const float* k, const float* v,
                                uint16_t* key_cache, uint16_t* value_cache, float* xb,
                                int32_t start_pos, int32_t n_rows, int32_t n_heads,
                                int32_t n_kv_heads, int32_t head_dim, int32_t context_length,
                                float theta, int32_t rope_style);

/* ------------------------------------------------------------------------ */
/* Output projection (the step after attention)                              */
/* ------------------------------------------------------------------------ */

/* x[i] = x[i] + sum_j w[i*n + j] * xb[j] for i in [0, d): the wo projection of
 * the attention output with the residual add, the reference's GPU task
 * "matmul1" = matrixVectorGenericWithResidual(context, xb, x, wo, n, d, 32)
 * (tornadovm/kernels/TransformerComputeKernelsLayered.java:715-733,
 * LlamaFP16FFNLayers.java:131; on the CPU InferenceCore.java:147-150).
 * w FP16 [d][n] row-major (HalfFloatArray), xb [n] and x [d] FP32; FP32
 * products and sums in a different order than the reference's 32-lane tree
 * (results agree to FP32 rounding, not bit for bit).  n % 8 == 0, w and xb
 * 16-byte aligned.  Launched with programmatic dependent launch: issued right
 * after an attention call on the same stream, it streams the weights while
 * the attention finishes and reads xb only once it has. */
int32_t gla_wo_residual_f16(gla_ctx* ctx, const float* xb, float* x, const uint16_t* w, int32_t n,
                            int32_t d);

/* ------------------------------------------------------------------------ */
/* Input producers: RoPE + KV append (the step before attention)             */
/* ------------------------------------------------------------------------ */

#define GLA_ROPE_INTERLEAVED 0 /* Llama/Mistral: pairs (2i, 2i+1), InferenceCore.java:82-94   */
#define GLA_ROPE_NEOX 1        /* Qwen2/Qwen3/Phi3: pairs (i, i+hd/2), InferenceCore.java:210-225 */

/* Rotates q (n_heads heads) and k (n_kv_heads heads) in place for `position`
 * with frequencies 1/theta^(2i/head_dim) (RoPE.java:6-37 without Llama-3.1
 * scaling), then appends k and v as row `position` of the FP32 layer caches
 * key_cache/value_cache ([position][kv_dim], InferenceCore.java:99-100;
 * copyToCache TransformerComputeKernelsLayered.java:129-139).  position is
 * read from the DEVICE int32 position_holder[0]. */
int32_t gla_rope_append_f32(gla_ctx* ctx, float* q, float* k, const float* v, float* key_cache,
                            float* value_cache, int32_t n_heads, int32_t n_kv_heads,
                            int32_t head_dim, const int32_t* position_holder, float theta,
                            int32_t rope_style);

/* ------------------------------------------------------------------------ */
/* Introspection used by the host tests (no device work)                     */
/* ------------------------------------------------------------------------ */

/* Test hook: launches on the context's stream a kernel standing in for a
 * caller's own position update - it releases its dependents at once
 * (programmatic dependent launch), spins delay_us (at most 1000), then adds
 * `delta` to position_holder[0].  A decode call behind it must attend to the
 * new position.  No reference counterpart. */
int32_t gla_debug_advance_position(gla_ctx* ctx, int32_t* position_holder, int32_t delta,
                                   int32_t delay_us);

/* Test hook: makes the context play rank 0 of a `world`-rank peer exchange
 * (2..8) whose other ranks' buffers are local allocations that nobody
 * writes, so a sharded call's bounded wait for their records runs out and
 * latches GLA_ERR_TIMEOUT in the device status.  world = 0 removes it.  Only
 * on a context without a communicator.  No reference counterpart. */
int32_t gla_debug_xch_loopback(gla_ctx* ctx, int32_t world);

/* Copies up to `capacity` words of the phase trace of the context's last
 * decode launch (GLA_OPT_TRACE) to host memory `out`, after synchronising
 * the stream: [CTA][16] uint64 (%globaltimer ns; word 10 = tiles | early
 * tiles << 16 | merger << 24 | SM id << 32).  Returns the words copied or a
 * negative status.  No reference counterpart. */
int64_t gla_debug_trace(gla_ctx* ctx, uint64_t* out, int64_t capacity);

/* Runs the decode kernels' work partition on the host: `n_seq` sequences with
 * n_pos[] rows, n_kv_heads segments each, dealt to `n_ctas` CTAs in units of
 * `unit_rows` rows and walked in tiles of up to `tile` rows (a multiple of
 * unit_rows; one sequence with n_kv_heads <= n_ctas: round robin, one unit a
 * tile).  Writes for every tile, in each CTA's walk order, its CTA, sequence,
 * kv head, first row, row count, partial-slot index, and the first CTA and
 * number of CTAs holding a piece of its segment (the merge's view) into the
 * eight arrays (each of length `capacity`); returns the tile count or a
 * negative status. */
int64_t gla_debug_partition(const int32_t* n_pos, int32_t n_seq, int32_t n_kv_heads, int32_t tile,
                            int32_t unit_rows, int32_t n_ctas, int32_t* cta, int32_t* seq,
                            int32_t* kv_head, int32_t* row0, int32_t* rows, int32_t* slot,
                            int32_t* first_cta, int32_t* npieces, int64_t capacity);

#ifdef __cplusplus
}
#endif

#endif /* GPULLAMA_ATTN_H */
