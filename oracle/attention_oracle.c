/*
 * attention_oracle.c - CPU restatement of GPULlama3.java's attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for
 * libgpullama_attn and the timed CPU baseline of bench.py; the product never
 * links, loads or calls it.
 *
 * PARITY UNPINNED: the reference ships no tests, fixtures or golden vectors
 * for attention, and its Java code cannot run here (no JDK, TornadoVM absent).
 * This restatement follows the Java source statement by statement instead:
 * same loop order, same FP32 operations in the same sequence (built with
 * -ffp-contract=off so no FMA is formed), Math.exp evaluated in double and
 * rounded to float, softmax normalised by a float division.  It is
 * self-checked by known-answer tests (uniform scores -> mean of V, one row ->
 * that row of V) and by a float64 restatement in the test-suite.
 *
 * Reference files (paths inside src/main/java/org/beehive/gpullama3/):
 *   inference/InferenceCore.java:105-144   per-head attention block (Llama)
 *   inference/InferenceCore.java:233-272   same block, Qwen2
 *   inference/InferenceCore.java:375-407   same block, Qwen3
 *   inference/InferenceCore.java:495-517   same block, Phi3
 *   tensor/standard/FloatTensor.java:86-92   scalarDot
 *   tensor/standard/FloatTensor.java:126-132 sum / max (reduce)
 *   tensor/standard/FloatTensor.java:167-173 mapInPlace
 *   tensor/standard/FloatTensor.java:203-227 divideInPlace, softmaxInPlace, saxpyInPlace
 *   tensor/standard/ArrayFloatTensor.java:49-52 fillInPlace
 *   auxiliary/Parallel.java:9-11            parallelFor over heads
 *   inference/operation/RoPE.java:6-37       precomputeFreqsCis
 *   inference/InferenceCore.java:82-94      interleaved RoPE rotation (Llama)
 *   inference/InferenceCore.java:210-225    NeoX RoPE rotation (Qwen2; Qwen3 :351-366, Phi3 :473-487)
 *   inference/InferenceEngine.java:88-99    prompt ingestion = decode at 0..L-1
 *   tornadovm/kernels/TransformerComputeKernelsLayered.java:715-733, :850-878
 *                                           wo projection + residual (GPU task "matmul1")
 *   tensor/GGMLType.java:13 (Q8_0 block shape) and GGML's published Q8_0 reference
 *   quantiser (ggml, quantize_row_q8_0_ref)  Q8 KV cache quantisation
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

/* Java's Math.max(float, float) (used by Float::max in FloatTensor.max):
 * NaN if either argument is NaN, otherwise the larger, with +0 > -0. */
static float java_fmax(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == 0.0f && b == 0.0f) return signbit(a) ? b : a;
  return a >= b ? a : b;
}

/* FloatTensor.scalarDot (FloatTensor.java:86-92): sequential FP32 sum of
 * products, j ascending, no fused multiply-add. */
static float scalar_dot(const float* a, const float* b, int size) {
  float result = 0.0f;
  for (int j = 0; j < size; j++) {
    float prod = a[j] * b[j];
    result = result + prod;
  }
  return result;
}

/* FloatTensor.softmaxInPlace (FloatTensor.java:211-219). */
static void softmax_inplace(float* x, int size) {
  float max_val = -INFINITY; /* reduce(..., NEGATIVE_INFINITY, Float::max) :130-132 */
  for (int i = 0; i < size; i++) max_val = java_fmax(max_val, x[i]);
  for (int i = 0; i < size; i++) x[i] = (float)exp((double)(x[i] - max_val)); /* mapInPlace :167-173 */
  float sum = 0.0f; /* reduce(..., 0f, Float::sum) :126-128 */
  for (int i = 0; i < size; i++) sum = sum + x[i];
  for (int i = 0; i < size; i++) x[i] = x[i] / sum; /* divideInPlace :203-205 */
}

/* FloatTensor.saxpyInPlace (FloatTensor.java:221-227):
 * this[i] = a * that[i] + this[i]. */
static void saxpy_inplace(float* x, const float* that, int size, float a) {
  for (int i = 0; i < size; i++) {
    float prod = a * that[i];
    x[i] = prod + x[i];
  }
}

/* IEEE binary16 -> binary32 (exact). */
static float half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        e++;
        mant <<= 1;
      } while ((mant & 0x400u) == 0);
      mant &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

void oracle_half_to_float(const uint16_t* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; i++) out[i] = half_to_float(in[i]);
}

/* Parallel.parallelFor(0, n, action) (auxiliary/Parallel.java:9-11): the
 * heads are independent, so the result does not depend on the thread count.
 * Threads take heads from a shared counter, like the ForkJoin pool's work
 * stealing. */
typedef struct {
  const float* q;
  const float* key_cache;
  const float* value_cache;
  float* xb;
  float* att;
  int n_heads, head_size, kv_mul, position;
  int64_t kv_stride;
  float divisor;
  int next; /* next head to take (atomic) */
} heads_job;

static void attention_head(const float* q, const float* key_cache, const float* value_cache,
                           float* xb, float* att, int h, int head_size, int64_t kv_stride,
                           int kv_mul, int position, float sqrt_head_size);

static void* heads_worker(void* arg) {
  heads_job* job = (heads_job*)arg;
  for (;;) {
    int h = __atomic_fetch_add(&job->next, 1, __ATOMIC_RELAXED);
    if (h >= job->n_heads) break;
    attention_head(job->q, job->key_cache, job->value_cache, job->xb,
                   job->att + (size_t)h * (size_t)(job->position + 1), h, job->head_size,
                   job->kv_stride, job->kv_mul, job->position, job->divisor);
  }
  return NULL;
}

int oracle_max_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

static void run_heads(heads_job* job, int n_threads) {
  int nt = n_threads > 0 ? n_threads : oracle_max_threads();
  if (nt > job->n_heads) nt = job->n_heads;
  if (nt < 1) nt = 1;
  job->next = 0;
  pthread_t tids[256];
  if (nt > 256) nt = 256;
  int started = 0;
  for (int i = 1; i < nt; i++) {
    if (pthread_create(&tids[started], NULL, heads_worker, job) == 0) started++;
  }
  heads_worker(job);
  for (int i = 0; i < started; i++) pthread_join(tids[i], NULL);
}

/* One head of InferenceCore.java:105-144.  key_cache/value_cache are the
 * layer's [position][kv_stride] caches (the reference uses kv_stride = kvDim),
 * att is the head's score scratch of >= position+1 floats. */
static void attention_head(const float* q, const float* key_cache, const float* value_cache,
                           float* xb, float* att, int h, int head_size, int64_t kv_stride,
                           int kv_mul, int position, float sqrt_head_size) {
  int q_offset = h * head_size;
  for (int t = 0; t <= position; t++) {
    int64_t key_off = (int64_t)t * kv_stride + (int64_t)(h / kv_mul) * head_size;
    float score = scalar_dot(q + q_offset, key_cache + key_off, head_size);
    score = score / sqrt_head_size;
    att[t] = score;
  }
  softmax_inplace(att, position + 1);
  int xb_offset = h * head_size;
  for (int i = 0; i < head_size; i++) xb[xb_offset + i] = 0.0f; /* fillInPlace */
  for (int t = 0; t <= position; t++) {
    int64_t v_off = (int64_t)t * kv_stride + (int64_t)(h / kv_mul) * head_size;
    float a = att[t];
    saxpy_inplace(xb + xb_offset, value_cache + v_off, head_size, a);
  }
}

/* Decode attention of one token at `position` (rows 0..position), all heads,
 * parallel over heads like Parallel.parallelFor (n_threads <= 0: all cores).
 * The divisor is (float)Math.sqrt(headSize) (InferenceCore.java:65). */
void oracle_decode_f32(const float* q, const float* key_cache, const float* value_cache, float* xb,
                       int n_heads, int head_size, int64_t kv_stride, int kv_mul, int position,
                       int n_threads) {
  float sqrt_head_size = (float)sqrt((double)head_size);
  float* att = (float*)malloc(sizeof(float) * (size_t)n_heads * (size_t)(position + 1));
  heads_job job = {q, key_cache, value_cache, xb, att, n_heads, head_size, kv_mul, position,
                   kv_stride, sqrt_head_size, 0};
  run_heads(&job, n_threads);
  free(att);
}

/* Same with the divisor given explicitly (Qwen3 divides by sqrt(nEmbdHead),
 * InferenceCore.java:324). */
void oracle_decode_f32_div(const float* q, const float* key_cache, const float* value_cache,
                           float* xb, int n_heads, int head_size, int64_t kv_stride, int kv_mul,
                           int position, float divisor, int n_threads) {
  float* att = (float*)malloc(sizeof(float) * (size_t)n_heads * (size_t)(position + 1));
  heads_job job = {q, key_cache, value_cache, xb, att, n_heads, head_size, kv_mul, position,
                   kv_stride, divisor, 0};
  run_heads(&job, n_threads);
  free(att);
}

/* FP16 cache: the reference has no FP16 KV; its FP32 semantics are applied to
 * the exactly decoded FP16 values. */
void oracle_decode_f16(const float* q, const uint16_t* key_cache, const uint16_t* value_cache,
                       float* xb, int n_heads, int head_size, int64_t kv_stride, int kv_mul,
                       int position, int n_threads) {
  int64_t n = (int64_t)position * kv_stride + kv_stride;
  float* kf = (float*)malloc(sizeof(float) * (size_t)n);
  float* vf = (float*)malloc(sizeof(float) * (size_t)n);
  oracle_half_to_float(key_cache, kf, n);
  oracle_half_to_float(value_cache, vf, n);
  oracle_decode_f32(q, kf, vf, xb, n_heads, head_size, kv_stride, kv_mul, position, n_threads);
  free(kf);
  free(vf);
}

/* Prompt ingestion as the reference does it: decode attention for every
 * position p in [0, L) over rows 0..p (InferenceEngine.java:88-99).
 * q/out [L][n_heads*head_size]; k/v [L][n_kv_heads*head_size], FP32 inputs
 * (FP16 prompts are decoded to float first by the caller). */
void oracle_prefill_causal_f32(const float* q, const float* k, const float* v, float* out, int L,
                               int n_heads, int n_kv_heads, int head_size, int n_threads) {
  int64_t q_stride = (int64_t)n_heads * head_size;
  int64_t kv_stride = (int64_t)n_kv_heads * head_size;
  int kv_mul = n_heads / n_kv_heads;
  for (int p = 0; p < L; p++) {
    oracle_decode_f32(q + p * q_stride, k, v, out + p * q_stride, n_heads, head_size, kv_stride,
                      kv_mul, p, n_threads);
  }
}

/* RoPE.precomputeFreqsCis (RoPE.java:6-37), including the Llama-3.1
 * frequency scaling branch.  cr/ci hold context_length*(head_size/2) floats. */
void oracle_rope_freqs(int context_length, int head_size, double theta, int rope_scaling,
                       float scale_factor, float lo_freq_factor, float hi_freq_factor,
                       float old_context_length, float* cr, float* ci) {
  int n = 0;
  for (int pos = 0; pos < context_length; ++pos) {
    for (int i = 0; i < head_size; i += 2) {
      float freq = (float)(1.0 / pow(theta, i / (double)head_size));
      if (rope_scaling) {
        float lo_freq_wavelen = old_context_length / lo_freq_factor;
        float hi_freq_wavelen = old_context_length / hi_freq_factor;
        float wavelen = (float)(2.0 * M_PI / freq);
        if (wavelen < hi_freq_wavelen) {
          /* freq unchanged */
        } else if (wavelen > lo_freq_wavelen) {
          freq = freq / scale_factor;
        } else {
          float smooth = (old_context_length / wavelen - lo_freq_factor) /
                         (hi_freq_factor - lo_freq_factor);
          freq = (1.0f - smooth) * freq / scale_factor + smooth * freq;
        }
      }
      float val = (float)pos * freq;
      cr[n] = (float)cos((double)val);
      ci[n] = (float)sin((double)val);
      n++;
    }
  }
}

/* Interleaved-pair rotation of q (dim floats) and k (kv_dim floats) at
 * `position` (InferenceCore.java:82-94). */
void oracle_rope_interleaved(float* q, float* k, int dim, int kv_dim, int head_size, int position,
                             const float* cr, const float* ci) {
  for (int i = 0; i < dim; i += 2) {
    int head_dim = i % head_size;
    float fcr = cr[position * (head_size / 2) + (head_dim / 2)];
    float fci = ci[position * (head_size / 2) + (head_dim / 2)];
    int rotn = i < kv_dim ? 2 : 1;
    for (int vv = 0; vv < rotn; vv++) {
      float* vec = vv == 0 ? q : k;
      float v0 = vec[i];
      float v1 = vec[i + 1];
      vec[i] = v0 * fcr - v1 * fci;
      vec[i + 1] = v0 * fci + v1 * fcr;
    }
  }
}

/* NeoX half-split rotation, pairs (ic, ic + head_size/2) in every head
 * (Qwen2 InferenceCore.java:210-225; k rotated for heads < n_kv_heads). */
void oracle_rope_neox(float* q, float* k, int n_heads, int n_kv_heads, int head_size,
                      int position, const float* cr, const float* ci) {
  for (int h = 0; h < n_heads; ++h) {
    int rotn = h < n_kv_heads ? 2 : 1;
    int poffset = h * head_size;
    for (int i0 = 0; i0 < head_size; i0 += 2) {
      int ic = i0 / 2;
      float fcr = cr[position * (head_size / 2) + ic];
      float fci = ci[position * (head_size / 2) + ic];
      for (int vi = 0; vi < rotn; vi++) {
        float* vec = vi == 0 ? q : k;
        float v0 = vec[poffset + ic];
        float v1 = vec[poffset + ic + head_size / 2];
        vec[poffset + ic] = v0 * fcr - v1 * fci;
        vec[poffset + ic + head_size / 2] = v0 * fci + v1 * fcr;
      }
    }
  }
}


/* matrixVectorGenericWithResidual (TransformerComputeKernelsLayered.java:715-733)
 * through matrixVectorRowMajorOptimized's HalfFloatArray overload (:850-878):
 * one workgroup of local_size threads per output row; thread t accumulates
 * w[row*n + j] * x[j] for j = t, t + local_size, ... in that order, then the
 * tree reduction localSum[t] += localSum[t + stride] for stride =
 * local_size/2 .. 1, and hb[row] = hb[row] + localSum[0].  The GPU layer
 * plan launches it with local_size 32 (LOCAL_WORK_GROUP_SIZE_ALLOC,
 * tornadovm/layers/AbstractLayer.java:20; LlamaFP16FFNLayers.java:131). */
void oracle_wo_residual_f16(const float* x, float* hb, const uint16_t* w, int n, int d,
                            int local_size) {
  float local_sum[1024];
  if (local_size < 1 || local_size > 1024) return;
  for (int row = 0; row < d; ++row) {
    const uint16_t* wr = w + (int64_t)row * n;
    for (int t = 0; t < local_size; ++t) {
      float partial = 0.0f;
      for (int j = t; j < n; j += local_size) partial += half_to_float(wr[j]) * x[j];
      local_sum[t] = partial;
    }
    for (int stride = local_size / 2; stride > 0; stride >>= 1)
      for (int t = 0; t < stride; ++t) local_sum[t] += local_sum[t + stride];
    hb[row] = hb[row] + local_sum[0];
  }
}

/* IEEE binary32 -> binary16, round to nearest even (NaN -> quiet NaN). */
static uint16_t float_to_half_rne(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t a = x & 0x7fffffffu;
  if (a >= 0x7f800000u) return sign | (a > 0x7f800000u ? 0x7e00u : 0x7c00u);
  if (a >= 0x477ff000u) return sign | 0x7c00u; /* >= 65520 rounds to infinity */
  if (a < 0x38800000u) {                       /* below 2^-14: subnormal half */
    float af;
    memcpy(&af, &a, 4);
    return sign | (uint16_t)nearbyint((double)af * 16777216.0); /* units of 2^-24 */
  }
  uint32_t h = ((((a >> 23) - 127 + 15) & 0x1fu) << 10) | ((a & 0x7fffffu) >> 13);
  const uint32_t rem = a & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h; /* a carry may raise the exponent */
  return sign | (uint16_t)h;
}

void oracle_float_to_half(const float* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = float_to_half_rne(in[i]);
}

/* Q8 KV cache rows as GGML's Q8_0 reference quantiser does a block of 32:
 * amax = max |x|, d = amax / 127, id = d ? 1/d : 0, q = roundf(x * id), d kept
 * as FP16.  Layout: values [rows][kv_stride] int8 (head g at g*hd), scales
 * [rows][n_kv][8] FP16 bits with K blocks at 0.. and V blocks at 4.., the other
 * halves 0. */
static void quantize_head_row(const float* x, int8_t* q, uint16_t* s, int nb) {
  for (int b = 0; b < nb; ++b) {
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) {
      const float ax = fabsf(x[32 * b + j]);
      if (ax > amax) amax = ax;
    }
    const float d = amax / 127.0f;
    /* d below ~1e-38 makes 1/d overflow; such a block's FP16 scale is 0 anyway */
    const float r = d != 0.0f ? 1.0f / d : 0.0f;
    const float id = (d != 0.0f && r < INFINITY) ? r : 0.0f;
    for (int j = 0; j < 32; ++j) q[32 * b + j] = (int8_t)roundf(x[32 * b + j] * id);
    s[b] = float_to_half_rne(d);
  }
}

void oracle_quantize_q8(const float* k, const float* v, int64_t src_stride, int n_rows, int n_kv,
                        int hd, int8_t* kq, int8_t* vq, int64_t kv_stride, uint16_t* scales) {
  const int nb = hd / 32;
  for (int64_t r = 0; r < n_rows; ++r)
    for (int g = 0; g < n_kv; ++g) {
      uint16_t* srow = scales + (r * n_kv + g) * 8;
      memset(srow, 0, 8 * sizeof(uint16_t));
      quantize_head_row(k + r * src_stride + (int64_t)g * hd, kq + r * kv_stride + (int64_t)g * hd,
                        srow, nb);
      quantize_head_row(v + r * src_stride + (int64_t)g * hd, vq + r * kv_stride + (int64_t)g * hd,
                        srow + 4, nb);
    }
}
