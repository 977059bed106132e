// decode_kernel.cuh - split-KV flash-decoding kernel for B200 (sm_100a).
//
// One token per sequence attends to rows [0, n_pos) of its K/V cache
// (layout [row][kv_stride], kv head g at column g*HD), for every q head
// h = g*G + i (GQA group of G = n_heads/n_kv_heads q heads per kv head;
// TransformerComputeKernelsLayered.java:336-458 runs the same math with one
// workgroup per q head).
//
// Structure (one persistent CTA per SM):
//  * The tiles of all (sequence, kv head) segments are dealt to the CTAs in
//    contiguous near-equal ranges (gla_common.cuh), so every SM streams the
//    same number of KV bytes whatever the sequence lengths.
//  * Warp NW is the producer: per tile it issues one bulk TMA copy
//    (cp.async.bulk) per K row and per V row into a ring of `stages` shared
//    memory stages guarded by full/empty mbarriers.  Rows of one kv head are
//    head_dim contiguous elements, so each copy is a 128-512 byte burst and
//    HBM sees long coalesced reads.
//  * Warps 0..NW-1 consume every stage together; each owns a fixed slice of
//    the tile's rows and keeps its own online-softmax state (m, l, o) for all
//    G q heads of the group, so all heads of a group share one K/V tile read
//    and no CTA-wide barrier is needed per tile.
//  * At the end of a segment piece the warps merge their states in shared
//    memory.  A segment held by one CTA is written straight to xb; otherwise
//    each CTA stores its piece to a workspace slot and the last CTA to finish
//    (atomic counter, reset by that CTA) merges the pieces (log-sum-exp).
//
// Consumers: F32Consumer (FP32 cache, CUDA-core FMA: the FP32 cache delivers
// at most G/2 FLOP per byte) and F16Consumer (FP16 cache, mma.sync m16n8k16
// with q and p split into hi+lo halves so products keep ~22 mantissa bits;
// FP32 accumulation).  Scores are kept in the log2 domain (q pre-scaled by
// scale*log2(e)), which is the same softmax.
#pragma once

#include "gla_common.cuh"

namespace gla {

struct DecodeArgs {
  const float* q;              // [B][n_heads][HD]
  const void* k;               // layer base (single sequence) or nullptr
  const void* v;
  const void* const* k_ptrs;   // device [B] layer bases (batched) or nullptr
  const void* const* v_ptrs;
  int64_t kv_stride;           // elements between rows
  const int32_t* n_pos_dev;    // device [B] or nullptr
  int32_t n_pos;               // rows when n_pos_dev == nullptr
  int32_t n_pos_add;           // added to n_pos_dev[b] (position holder: +1)
  int32_t n_pos_cap;           // rows present in the cache; larger n_pos is clamped
                               // and latched as GLA_ERR_INVALID_ARG
  int32_t batch;
  int32_t n_heads;
  int32_t n_kv;
  int32_t group;               // G
  int32_t tile;                // rows per stage
  int32_t stages;
  float q_scale;               // scale * log2(e)
  float* out;                  // xb [B][n_heads][HD] or records [B][n_heads][HD+2]
  int32_t record_mode;
  float* ws_part;              // workspace slots [P + B*n_kv][G][HD+2]
  int32_t* ws_counter;         // [B*n_kv], zero between calls
  int32_t* status;             // device status word
  // shared memory layout (bytes)
  int32_t row_bytes;           // smem bytes per cached row (incl. padding)
  int32_t stage_bytes;         // 2 * tile * row_bytes
  int32_t off_bars;
  int32_t off_seq;
  int32_t off_pbuf;
  int32_t off_merge;
  int32_t off_flags;
};

constexpr float kLn2 = 0.69314718055994530942f;

// ---------------------------------------------------------------------------
// FP32 cache consumer: 16 lanes per row in phase A (q.k), all 32 lanes across
// head_dim in phase B (p.v).
// ---------------------------------------------------------------------------
template <int HD, int GT, int NW>
struct F32Consumer {
  static constexpr int kVecA = (HD % 64 == 0) ? 4 : 2;   // floats per phase-A load
  static constexpr int kChunksA = HD / 16 / kVecA;       // loads per lane per row
  static constexpr int kVB = HD / 32;                    // floats per lane in phase B
  static constexpr int kTileMax = (HD <= 64) ? 64 : 32;
  static constexpr int kMaxPass = kTileMax / NW / 2;
  static constexpr int kMergeG = GT;
  static constexpr int kElemBytes = 4;
  static constexpr int kRowBytes = HD * 4;
  static constexpr int kPbufFloats = 64;  // per warp: <= 8 rows x 8 heads
  static_assert(HD % 32 == 0 || HD == 96, "head_dim");

  float qreg[GT][HD / 16];
  float m[GT], l[GT];
  float o[GT][kVB];

  __device__ __forceinline__ void begin(const DecodeArgs& a, int b, int g, int lane) {
    const int j = lane & 15;
    const float* qb = a.q + ((int64_t)b * a.n_heads + (int64_t)g * a.group) * HD;
#pragma unroll
    for (int h = 0; h < GT; ++h) {
#pragma unroll
      for (int c = 0; c < kChunksA; ++c) {
#pragma unroll
        for (int e = 0; e < kVecA; ++e) {
          float x = 0.f;
          if (h < a.group) x = qb[h * HD + (c * 16 + j) * kVecA + e] * a.q_scale;
          qreg[h][c * kVecA + e] = x;
        }
      }
      m[h] = -INFINITY;
      l[h] = 0.f;
#pragma unroll
      for (int e = 0; e < kVB; ++e) o[h][e] = 0.f;
    }
  }

  __device__ __forceinline__ void consume(const DecodeArgs& a, const char* stage, int rows,
                                          float* pbuf_w, int w, int lane) {
    const float* Ks = reinterpret_cast<const float*>(stage);
    const float* Vs = reinterpret_cast<const float*>(stage + a.tile * kRowBytes);
    const int rpw = a.tile / NW;
    const int npass = rpw >> 1;
    const int half = lane >> 4, j = lane & 15;
    const int row_base = w * rpw;
    float s[kMaxPass][GT];
#pragma unroll
    for (int pp = 0; pp < kMaxPass; ++pp) {
      if (pp < npass) {
        const int row = row_base + 2 * pp + half;
        const float* kr = Ks + row * HD;
        float acc[GT];
#pragma unroll
        for (int h = 0; h < GT; ++h) acc[h] = 0.f;
#pragma unroll
        for (int c = 0; c < kChunksA; ++c) {
          float kv[kVecA];
          if constexpr (kVecA == 4) {
            float4 t = *reinterpret_cast<const float4*>(kr + (c * 16 + j) * 4);
            kv[0] = t.x; kv[1] = t.y; kv[2] = t.z; kv[3] = t.w;
          } else {
            float2 t = *reinterpret_cast<const float2*>(kr + (c * 16 + j) * 2);
            kv[0] = t.x; kv[1] = t.y;
          }
#pragma unroll
          for (int h = 0; h < GT; ++h)
#pragma unroll
            for (int e = 0; e < kVecA; ++e) acc[h] = fmaf(qreg[h][c * kVecA + e], kv[e], acc[h]);
        }
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1)
#pragma unroll
          for (int h = 0; h < GT; ++h) acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], off);
        const bool valid = row < rows;
#pragma unroll
        for (int h = 0; h < GT; ++h) s[pp][h] = valid ? acc[h] : -INFINITY;
      } else {
#pragma unroll
        for (int h = 0; h < GT; ++h) s[pp][h] = -INFINITY;
      }
    }
    // online softmax over this warp's rows of the tile
#pragma unroll
    for (int h = 0; h < GT; ++h) {
      float mt = s[0][h];
#pragma unroll
      for (int pp = 1; pp < kMaxPass; ++pp) mt = fmaxf(mt, s[pp][h]);
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
      const float mn = fmaxf(m[h], mt);
      const bool none = (mn == -INFINITY);
      const float alpha = none ? 1.f : fast_exp2(m[h] - mn);
      float psum = 0.f;
#pragma unroll
      for (int pp = 0; pp < kMaxPass; ++pp) {
        const float p = none ? 0.f : fast_exp2(s[pp][h] - mn);
        s[pp][h] = p;
        psum += p;
      }
      psum += __shfl_xor_sync(0xffffffffu, psum, 16);
      l[h] = l[h] * alpha + psum;
      m[h] = mn;
#pragma unroll
      for (int e = 0; e < kVB; ++e) o[h][e] *= alpha;
    }
    if (j == 0) {
#pragma unroll
      for (int pp = 0; pp < kMaxPass; ++pp) {
        if (pp < npass) {
#pragma unroll
          for (int h = 0; h < GT; ++h) pbuf_w[(2 * pp + half) * 8 + h] = s[pp][h];
        }
      }
    }
    __syncwarp();
    const int nrows = min(rpw, rows - row_base);
    for (int r = 0; r < nrows; ++r) {
      const float* vr = Vs + (row_base + r) * HD + lane * kVB;
      float vv[kVB];
      if constexpr (kVB == 4) {
        float4 t = *reinterpret_cast<const float4*>(vr);
        vv[0] = t.x; vv[1] = t.y; vv[2] = t.z; vv[3] = t.w;
      } else if constexpr (kVB == 2) {
        float2 t = *reinterpret_cast<const float2*>(vr);
        vv[0] = t.x; vv[1] = t.y;
      } else {
#pragma unroll
        for (int e = 0; e < kVB; ++e) vv[e] = vr[e];
      }
      float pr[GT];
      const float* prow = pbuf_w + r * 8;
      if constexpr (GT >= 4) {
#pragma unroll
        for (int h4 = 0; h4 < GT; h4 += 4) {
          float4 t = *reinterpret_cast<const float4*>(prow + h4);
          pr[h4] = t.x; pr[h4 + 1] = t.y; pr[h4 + 2] = t.z; pr[h4 + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int h = 0; h < GT; ++h) pr[h] = prow[h];
      }
#pragma unroll
      for (int h = 0; h < GT; ++h)
#pragma unroll
        for (int e = 0; e < kVB; ++e) o[h][e] = fmaf(pr[h], vv[e], o[h][e]);
    }
    __syncwarp();
  }

  // Writes this warp's (m, l, o) for q heads h < group into merge_w[h][HD+2].
  __device__ __forceinline__ void to_merge(const DecodeArgs& a, float* merge_w, int lane) {
#pragma unroll
    for (int h = 0; h < GT; ++h) {
      if (h < a.group) {
        float* mh = merge_w + h * (HD + 2);
#pragma unroll
        for (int e = 0; e < kVB; ++e) mh[lane * kVB + e] = o[h][e];
        if (lane == 0) {
          mh[HD] = m[h];
          mh[HD + 1] = l[h];
        }
      }
    }
  }
};

// ---------------------------------------------------------------------------
// FP16 cache consumer: each warp owns 16 rows of a tile and computes
// S = Q K^T and O += P V with mma.sync.m16n8k16 (f16 x f16 -> f32).
// A-operand rows 0..7 hold the hi halves of the G <= 8 q heads (or p), rows
// 8..15 the lo halves (x - float(hi)), so row h + row h+8 of the product is
// the full-precision result for head h.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

__device__ __forceinline__ void split_half(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(x - __half2float(hi));
}

__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Zeroes the halves of a B fragment register whose rows (positions p0, p0+1)
// are outside the valid range.
__device__ __forceinline__ uint32_t mask_pair(uint32_t r, int p0, int nvalid) {
  uint32_t keep = (p0 < nvalid ? 0x0000ffffu : 0u) | (p0 + 1 < nvalid ? 0xffff0000u : 0u);
  return r & keep;
}

template <int HD, int NW>
struct F16Consumer {
  static constexpr int kRS = HD + 8;             // smem row stride in halves (16 B pad)
  static constexpr int kRowBytes = kRS * 2;
  static constexpr int kElemBytes = 2;
  static constexpr int kPbufFloats = 0;
  static constexpr int kTileMax = 16 * NW;
  static constexpr int kMergeG = kMaxGroup;
  static constexpr int kKS = HD / 16;            // k-steps of q.k
  static constexpr int kNT = HD / 8;             // n-tiles of p.v
  static_assert(kKS % 2 == 0 && kNT % 2 == 0, "head_dim must be a multiple of 32");

  uint32_t qa[kKS][4];
  float m_run, l_run;
  float oacc[kNT][4];

  __device__ __forceinline__ void begin(const DecodeArgs& a, int b, int g, int lane) {
    const int gid = lane >> 2, tig = lane & 3;
    const float* qh = a.q + ((int64_t)b * a.n_heads + (int64_t)g * a.group + gid) * HD;
    const bool live = gid < a.group;
#pragma unroll
    for (int kk = 0; kk < kKS; ++kk) {
      const int c0 = kk * 16 + 2 * tig, c1 = c0 + 8;
      float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
      if (live) {
        float2 u = *reinterpret_cast<const float2*>(qh + c0);
        float2 w = *reinterpret_cast<const float2*>(qh + c1);
        x0 = u.x * a.q_scale; x1 = u.y * a.q_scale;
        x2 = w.x * a.q_scale; x3 = w.y * a.q_scale;
      }
      __half h0, l0, h1, l1, h2, l2, h3, l3;
      split_half(x0, h0, l0); split_half(x1, h1, l1);
      split_half(x2, h2, l2); split_half(x3, h3, l3);
      qa[kk][0] = pack_half2(h0, h1);
      qa[kk][1] = pack_half2(l0, l1);
      qa[kk][2] = pack_half2(h2, h3);
      qa[kk][3] = pack_half2(l2, l3);
    }
    m_run = -INFINITY;
    l_run = 0.f;
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) oacc[nt][e] = 0.f;
  }

  __device__ __forceinline__ void consume(const DecodeArgs& a, const char* stage, int rows,
                                          float* /*pbuf_w*/, int w, int lane) {
    const int rb = w * 16;
    if (rb >= rows) return;
    const int nvalid = min(16, rows - rb);
    const int tig = lane & 3;
    const uint32_t kbase = smem_u32(stage) + (uint32_t)(rb * kRowBytes);
    const uint32_t vbase = kbase + (uint32_t)(a.tile * kRowBytes);
    float sacc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sacc[nt][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kKS; kk += 2) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint32_t addr =
            kbase + (uint32_t)(((nt * 8 + (lane & 7)) * kRS + kk * 16 + (lane >> 3) * 8) * 2);
        uint32_t r0, r1, r2, r3;
        ldsm_x4(addr, r0, r1, r2, r3);
        mma_16816(sacc[nt], qa[kk], r0, r1);
        mma_16816(sacc[nt], qa[kk + 1], r2, r3);
      }
    }
    float s[2][2];
    float mt = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int pos = nt * 8 + 2 * tig + e;
        const float x = sacc[nt][e] + sacc[nt][2 + e];
        s[nt][e] = pos < nvalid ? x : -INFINITY;
        mt = fmaxf(mt, s[nt][e]);
      }
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    const float mn = fmaxf(m_run, mt);  // finite: row rb is valid
    const float alpha = fast_exp2(m_run - mn);
    float p[2][2];
    float psum = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        p[nt][e] = fast_exp2(s[nt][e] - mn);
        psum += p[nt][e];
      }
    l_run = l_run * alpha + psum;
    m_run = mn;
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) oacc[nt][e] *= alpha;
    uint32_t pa[4];
    {
      __half h00, l00, h01, l01, h10, l10, h11, l11;
      split_half(p[0][0], h00, l00); split_half(p[0][1], h01, l01);
      split_half(p[1][0], h10, l10); split_half(p[1][1], h11, l11);
      pa[0] = pack_half2(h00, h01);
      pa[1] = pack_half2(l00, l01);
      pa[2] = pack_half2(h10, h11);
      pa[3] = pack_half2(l10, l11);
    }
    const bool partial = nvalid < 16;
#pragma unroll
    for (int nt = 0; nt < kNT; nt += 2) {
      const uint32_t addr =
          vbase + (uint32_t)((((lane & 7) + ((lane >> 3) & 1) * 8) * kRS + (nt + (lane >> 4)) * 8) * 2);
      uint32_t r0, r1, r2, r3;
      ldsm_x4_t(addr, r0, r1, r2, r3);
      if (partial) {
        r0 = mask_pair(r0, 2 * tig, nvalid);
        r1 = mask_pair(r1, 8 + 2 * tig, nvalid);
        r2 = mask_pair(r2, 2 * tig, nvalid);
        r3 = mask_pair(r3, 8 + 2 * tig, nvalid);
      }
      mma_16816(oacc[nt], pa, r0, r1);
      mma_16816(oacc[nt + 1], pa, r2, r3);
    }
  }

  __device__ __forceinline__ void to_merge(const DecodeArgs& a, float* merge_w, int lane) {
    const int gid = lane >> 2, tig = lane & 3;
    float lt = l_run;
    lt += __shfl_xor_sync(0xffffffffu, lt, 1);
    lt += __shfl_xor_sync(0xffffffffu, lt, 2);
    if (gid < a.group) {
      float* mh = merge_w + gid * (HD + 2);
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt) {
        mh[nt * 8 + 2 * tig] = oacc[nt][0] + oacc[nt][2];
        mh[nt * 8 + 2 * tig + 1] = oacc[nt][1] + oacc[nt][3];
      }
      if (tig == 0) {
        mh[HD] = m_run;
        mh[HD + 1] = lt;
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Output helpers
// ---------------------------------------------------------------------------
template <int HD>
__device__ __forceinline__ void write_final(const DecodeArgs& a, int b, int hq, int d, float O,
                                            float M, float L) {
  const int64_t row = (int64_t)b * a.n_heads + hq;
  if (a.record_mode) {
    float* rec = a.out + row * (HD + 2);
    rec[d] = L > 0.f ? O / L : 0.f;
    if (d == 0) {
      rec[HD] = L > 0.f ? M * kLn2 : -INFINITY;
      rec[HD + 1] = L;
    }
  } else {
    a.out[row * HD + d] = L > 0.f ? O / L : 0.f;
  }
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int HD, int NW, class Consumer>
__global__ void __launch_bounds__((NW + 1) * 32, 1) decode_kernel(const DecodeArgs a) {
  extern __shared__ __align__(128) char smem[];
  constexpr int kNCT = NW * 32;  // consumer threads
  constexpr int kMG = Consumer::kMergeG;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int B = a.batch, n_kv = a.n_kv, G = a.group;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bars);
  uint64_t* empty = full + a.stages;
  int32_t* seq_start = reinterpret_cast<int32_t*>(smem + a.off_seq);  // [B+1]
  int32_t* ntiles = seq_start + (B + 1);                              // [B]
  int32_t* npos = ntiles + B;                                         // [B]
  float* pbuf = reinterpret_cast<float*>(smem + a.off_pbuf);           // [NW][kPbufFloats]
  float* merge = reinterpret_cast<float*>(smem + a.off_merge);         // [NW][kMG][HD+2]
  volatile int* flags = reinterpret_cast<volatile int*>(smem + a.off_flags);  // [0]=abort [1]=last

  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_mbarrier_init();
  }
  // per-sequence rows and tile prefix (warp 0 scans 32 sequences at a time)
  if (warp == 0) {
    int32_t carry = 0;
    for (int base = 0; base < B; base += 32) {
      const int b = base + lane;
      int32_t np = 0, nt = 0;
      if (b < B) {
        np = a.n_pos_dev ? a.n_pos_dev[b] + a.n_pos_add : a.n_pos;
        np = np < 0 ? 0 : np;
        if (np > a.n_pos_cap) {
          atomicCAS(a.status, 0, GLA_ERR_INVALID_ARG);
          np = a.n_pos_cap;
        }
        nt = ceil_div(np, a.tile);
        npos[b] = np;
        ntiles[b] = nt;
      }
      int32_t incl = nt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        int32_t y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      if (b < B) seq_start[b] = (carry + incl - nt) * n_kv;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) seq_start[B] = carry * n_kv;
  }
  __syncthreads();

  const int32_t W = seq_start[B];
  const Split sp = make_split(W, (int32_t)gridDim.x);
  const int32_t my_lo = split_lo(sp, blockIdx.x);
  const int32_t my_count = split_count(sp, blockIdx.x);

  if (warp == NW) {
    // ---------------- producer ----------------
    if (my_count > 0) {
      const uint64_t pol = l2_evict_first_policy();
      constexpr int esize = Consumer::kElemBytes;
      const uint32_t copy_bytes = HD * esize;
      TileRef tr = locate_tile(seq_start, ntiles, B, n_kv, my_lo);
      int cur_b = -1;
      const char* kb = nullptr;
      const char* vb = nullptr;
      for (int32_t i = 0; i < my_count; ++i) {
        const int st = i % a.stages;
        const uint32_t use = (uint32_t)(i / a.stages);
        if (!mbar_wait(&empty[st], (use & 1u) ^ 1u, flags, a.status)) break;
        if (tr.b != cur_b) {
          cur_b = tr.b;
          kb = static_cast<const char*>(a.k_ptrs ? a.k_ptrs[cur_b] : a.k);
          vb = static_cast<const char*>(a.v_ptrs ? a.v_ptrs[cur_b] : a.v);
          // caller-supplied device pointers: a null or unaligned base would
          // make the bulk copies fault, so refuse it and drain instead
          if (kb == nullptr || vb == nullptr ||
              ((reinterpret_cast<uintptr_t>(kb) | reinterpret_cast<uintptr_t>(vb)) & 15u)) {
            atomicCAS(a.status, 0, GLA_ERR_ALIGNMENT);
            flags[0] = 1;
            break;
          }
        }
        const int row0 = tr.j * a.tile;
        const int rows = min(a.tile, npos[tr.b] - row0);
        if (lane == 0) mbar_arrive_expect_tx(&full[st], (uint32_t)rows * copy_bytes * 2u);
        __syncwarp();
        char* ks = smem + (size_t)st * a.stage_bytes;
        char* vs = ks + (size_t)a.tile * a.row_bytes;
        for (int r = lane; r < rows; r += 32) {
          const int64_t off = ((int64_t)(row0 + r) * a.kv_stride + (int64_t)tr.g * HD) * esize;
          bulk_g2s(ks + (size_t)r * a.row_bytes, kb + off, copy_bytes, &full[st], pol);
          bulk_g2s(vs + (size_t)r * a.row_bytes, vb + off, copy_bytes, &full[st], pol);
        }
        next_tile(tr, ntiles, B, n_kv);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  // segments with no rows (n_pos <= 0) produce zeros / empty records
  for (int s = blockIdx.x; s < B * n_kv; s += gridDim.x) {
    const int b = s / n_kv, g = s - b * n_kv;
    if (ntiles[b] == 0)
      for (int idx = tid; idx < G * HD; idx += kNCT)
        write_final<HD>(a, b, g * G + idx / HD, idx % HD, 0.f, 0.f, 0.f);
  }
  if (my_count == 0) return;

  Consumer cons;
  float* pbuf_w = pbuf + warp * Consumer::kPbufFloats;
  float* merge_w = merge + warp * kMG * (HD + 2);
  TileRef tr = locate_tile(seq_start, ntiles, B, n_kv, my_lo);
  int cur_b = -1, cur_g = -1;

  auto finish_piece = [&](int b, int g) {
    cons.to_merge(a, merge_w, lane);
    consumer_sync(kNCT);
    const int s = b * n_kv + g;
    int32_t c0;
    const int32_t npieces = segment_pieces(sp, seq_start, ntiles, b, g, &c0);
    const int slot_floats = G * (HD + 2);
    for (int idx = tid; idx < G * HD; idx += kNCT) {
      const int h = idx / HD, d = idx - h * HD;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < NW; ++w) M = fmaxf(M, merge[(w * kMG + h) * (HD + 2) + HD]);
      float O = 0.f, L = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const float* mh = merge + (w * kMG + h) * (HD + 2);
          const float sc = fast_exp2(mh[HD] - M);
          O += sc * mh[d];
          L += sc * mh[HD + 1];
        }
      }
      if (npieces == 1) {
        write_final<HD>(a, b, g * G + h, d, O, M, L);
      } else {
        float* slot = a.ws_part + (int64_t)(blockIdx.x + s) * slot_floats + h * (HD + 2);
        slot[d] = O;
        if (d == 0) {
          slot[HD] = M;
          slot[HD + 1] = L;
        }
      }
    }
    if (npieces > 1) {
      __threadfence();
      consumer_sync(kNCT);
      if (tid == 0) {
        const int old = atomicAdd(&a.ws_counter[s], 1);
        flags[1] = (old == npieces - 1) ? 1 : 0;
      }
      consumer_sync(kNCT);
      if (flags[1]) {
        __threadfence();
        for (int idx = tid; idx < G * HD; idx += kNCT) {
          const int h = idx / HD, d = idx - h * HD;
          float M = -INFINITY;
          for (int c = c0; c < c0 + npieces; ++c)
            M = fmaxf(M, ld_cg(a.ws_part + (int64_t)(c + s) * slot_floats + h * (HD + 2) + HD));
          float O = 0.f, L = 0.f;
          if (M != -INFINITY) {
            for (int c = c0; c < c0 + npieces; ++c) {
              const float* sl = a.ws_part + (int64_t)(c + s) * slot_floats + h * (HD + 2);
              const float sc = fast_exp2(ld_cg(sl + HD) - M);
              O += sc * ld_cg(sl + d);
              L += sc * ld_cg(sl + HD + 1);
            }
          }
          write_final<HD>(a, b, g * G + h, d, O, M, L);
        }
        if (tid == 0) a.ws_counter[s] = 0;
      }
    }
    consumer_sync(kNCT);
  };

  for (int32_t i = 0; i < my_count; ++i) {
    if (tr.b != cur_b || tr.g != cur_g) {
      if (cur_b >= 0) finish_piece(cur_b, cur_g);
      cur_b = tr.b;
      cur_g = tr.g;
      cons.begin(a, cur_b, cur_g, lane);
    }
    const int st = i % a.stages;
    const uint32_t use = (uint32_t)(i / a.stages);
    const int rows = min(a.tile, npos[tr.b] - tr.j * a.tile);
    mbar_wait(&full[st], use & 1u, flags, a.status);
    cons.consume(a, smem + (size_t)st * a.stage_bytes, rows, pbuf_w, warp, lane);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    next_tile(tr, ntiles, B, n_kv);
  }
  finish_piece(cur_b, cur_g);
}

}  // namespace gla
