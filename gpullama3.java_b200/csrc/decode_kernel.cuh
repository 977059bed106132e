// decode_kernel.cuh - split-KV flash-decoding kernel for B200 (sm_100a).
//
// One token per sequence attends to rows [0, n_pos) of its K/V cache
// (layout [row][kv_stride], kv head g at column g*HD), for every q head
// h = g*G + i (GQA group of G = n_heads/n_kv_heads q heads per kv head;
// TransformerComputeKernelsLayered.java:336-458 runs the same math with one
// workgroup per q head).
//
// Structure (one persistent CTA per SM):
//  * The 64-row tiles of all (sequence, kv head) segments are dealt to the
//    CTAs (gla_common.cuh, Deal): one sequence gives each kv head its own
//    group of CTAs; batches are dealt in contiguous near-equal ranges, so
//    every SM streams the same number of KV bytes whatever the lengths.
//  * Warp NW is the producer.  It fills a ring of `stages` shared-memory
//    stages guarded by full/empty mbarriers, one K tile and one V tile
//    (`tile` rows of one kv head) per stage:
//      LOADER 0 (single sequence): tiled TMA, one cp.async.bulk.tensor.2d per
//        tensor and column block through a 2D tensor map [rows][kv_stride];
//        tiles land 128B/64B-swizzled so shared-memory reads are
//        conflict-free; rows past the cache end are zero-filled by the TMA
//        unit.  The first ring pass of cache history may be fetched before
//        the dependency wait (early prefetch, see the kernel).
//      LOADER 1 (batched, per-sequence pointers read on the device): 16-byte
//        cp.async into the same swizzled layout, completion via
//        cp.async.mbarrier.arrive.
//  * Warps 0..NW-1 consume every stage together; each owns a fixed slice of
//    the tile's rows and keeps its own online-softmax state (m, l, o) for all
//    G q heads of the group, so all heads of a group share one K/V tile read
//    and no CTA-wide barrier is needed per tile.
//  * At the end of a segment piece the warps merge their states in shared
//    memory.  A segment held by one CTA is written straight to xb; otherwise
//    each CTA stores its piece to a workspace slot as 64-bit words tagged
//    with the call's epoch and counts itself on the segment's counter; the
//    last min(G, pieces) CTAs to count (round-robin deal; only the last in
//    the contiguous deal) merge one q head each (log-sum-exp), and the last
//    one resets the counter.
//    Sharded sequences (record mode 2) then exchange per-rank records over
//    peer memory and merge them in the same kernel (publish_merge).
//
// Consumers: F32Consumer (FP32 cache, CUDA-core FMA: the FP32 cache delivers
// at most G/2 FLOP per byte) and F16Consumer (FP16 cache, mma.sync m16n8k16
// with q and p split into hi+lo halves so products keep ~22 mantissa bits;
// FP32 accumulation).  Scores are kept in the log2 domain (q pre-scaled by
// scale*log2(e)), which is the same softmax.
#pragma once

#include "gla_common.cuh"
#include "gla_rope.cuh"
#include "gla_xch.h"

namespace gla {

// Q8 cache scales: one row of 8 halves per (key, kv head): the K block scales
// (one per 32 values) at [0, HD/32), the V block scales at [4, 4 + HD/32).
constexpr int kQ8ScaleHalves = 8;
constexpr int kQ8ScaleRowBytes = 16;

struct DecodeArgs {
  CUtensorMap tmap_k;          // LOADER 0: [rows][kv_stride] box (col_block, tile rows)
  CUtensorMap tmap_v;
  CUtensorMap tmap_s;          // Q8 cache: scales [rows][n_kv * 8] halves, box (8, tile rows)
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
  int32_t early_kv;            // LOADER 0: prefetch history tiles before the preceding
                               // grid completes: 1 host n_pos, 2 also n_pos_dev (see kernel)
  int32_t batch;
  int32_t n_heads;
  int32_t n_kv;
  int32_t group;               // G
  int32_t tile;                // rows per stage and per work unit
  int32_t stages;
  float q_scale;               // scale * log2(e)
  float* out;                  // xb [B][n_heads][HD] or records [B][n_heads][HD+2]
  int32_t record_mode;         // 0 xb, 1 records, 2 records merged across ranks (peer
                               // exchange, one sequence; see gla_xch.h)
  const uint64_t* xch_bases;   // mode 2: device [world], every rank's exchange buffer as
                               // mapped in this process
  char* xch_local;             // mode 2: this rank's exchange buffer
  float* xch_out;              // mode 2: merged xb [n_heads][HD]
  int32_t xch_world;
  int32_t xch_rank;
  // fused RoPE + append (rope != 0: one sequence, FP32 cache, tensor-map
  // loader): the new token's key row is rotated and written, with its value
  // row, at row n_pos - 1 of the caches before that row's tile is loaded; q
  // is rotated on its way into shared memory
  const float* rope_k;         // [n_kv * HD] new key, unrotated
  const float* rope_v;         // [n_kv * HD] new value
  double rope_theta;
  int32_t rope;
  int32_t rope_style;
  uint64_t* ws_part;           // piece slots [P + B*n_kv][G][HD+4] tagged words (o, m, l, pad)
  int32_t* ws_counter;         // [B*n_kv] piece counters, zero between calls
  unsigned long long* ws_epoch;  // call epoch << 32 | CTAs that took a ticket this call
  int32_t* status;             // device status word
  uint64_t* trace;             // optional [grid][kTraceWords] phase stamps (null: off)
  const void* scales;          // Q8 cache: [rows][n_kv][8] halves (row patches)
  // shared memory layout (bytes)
  int32_t stage_bytes;         // 2 * tile * head_dim * element size
  int32_t off_bars;
  int32_t off_seq;
  int32_t off_pbuf;
  int32_t off_q;               // the group's q vectors [kMaxGroup][HD]
  int32_t off_merge;
  int32_t off_flags;
  int32_t off_rope;            // float2 [HD/2]: (cos, sin) of the new position
};

// Floats per head in a workspace piece slot: o[HD], m, l, 2 pad (16-byte rows).
template <int HD>
constexpr int slot_head_floats() { return HD + 4; }
// Floats per head in a warp's merge buffer: the same 16-byte-row layout.
template <int HD>
constexpr int merge_head_floats() { return HD + 4; }

constexpr float kLn2 = 0.69314718055994530942f;

// ---------------------------------------------------------------------------
// Tile layout in shared memory (both loaders write it, both consumers read
// it): each tensor tile is split into column blocks of kCW elements; block cb
// holds [tile][kCW] rows of kRowB bytes with the TMA swizzle applied: the
// 16-byte chunk c of row r sits at chunk c ^ (r & 7) for 128-byte rows
// (SWIZZLE_128B) and c ^ ((r >> 1) & 3) for 64-byte rows (SWIZZLE_64B).
// Reading 8 consecutive rows at one logical chunk (ldmatrix, or one row per
// lane) therefore touches 8 different bank groups.
// ---------------------------------------------------------------------------
template <int ESIZE, int HD>
struct TileLayout {
  // FP32: 32-element blocks; FP16: 64 (32 for head_dim 96); int8: the whole
  // head row (64 or 128 bytes)
  static constexpr int kCW = (ESIZE == 4) ? 32 : (ESIZE == 2) ? ((HD % 64 == 0) ? 64 : 32) : HD;
  static constexpr int kRowB = kCW * ESIZE;  // 128 or 64
  static constexpr int kBlocks = HD / kCW;
  static_assert(HD % kCW == 0, "head_dim must be a multiple of the column block");
  static_assert(kRowB == 128 || kRowB == 64, "tile rows are 64 or 128 bytes");
  // byte offset of the 16-byte chunk holding (row, col); col % (16/ESIZE) == 0
  __device__ __forceinline__ static int chunk_off(int tile, int row, int col) {
    const int cb = col / kCW;
    const int c = ((col % kCW) * ESIZE) >> 4;
    const int sw = (kRowB == 128) ? (row & 7) : ((row >> 1) & 3);
    return cb * tile * kRowB + row * kRowB + ((c ^ sw) << 4);
  }
};

// ---------------------------------------------------------------------------
// FP32 cache consumer (CUDA-core FMA; an FP32 cache carries at most G/2 FLOP
// per byte).  8 warps, each owning 8 rows of a tile (two warps per scheduler
// hide each other's latency).  Latency bounds it, and a consumer squeezed
// below the 168 registers that 9 warps allow serialises its loads, so the
// layout keeps q small in registers and every load batch independent.
//   phase A (q.k): lane = (row rl of kRL, part of kLP = 32/kRL): the lane
//     streams kEC = head_dim/(4 kLP) float4 chunks of its row against the
//     same chunks of the G q vectors (registers while they take <= 64 of
//     them, else shared memory); hd >= 96 uses 4 rows x 8 parts, two passes
//     over the warp's 8 rows, hd 64 uses 8 rows x 4 parts.  Shuffles over
//     the parts join the dot products.
//   online softmax: one 8-row max per head per tile, branch-free so the G
//     heads' shuffle chains interleave (a lazy, vote-guarded rescale measured
//     slower: the branches serialise the heads).
//   phase B (p.v): lane = one float4 column chunk (two rows per pass when a
//     row has 16 chunks); all 8 rows unrolled, p read back as one float4 per
//     row and 4 heads; rows past the tile's end contribute zero (their V is
//     not trusted: it may be stale cache memory).
// ---------------------------------------------------------------------------
template <int HD, int GT>
struct F32Consumer {
  using TL = TileLayout<4, HD>;
  static constexpr int kElemBytes = 4;
  static constexpr bool kQ8 = false;
  static constexpr int kCtasPerSm = 1;  // 8 consumer warps: one CTA fills the schedulers
  static constexpr int kNW = 8;
  static constexpr int kRows = 8;               // rows per warp
  static constexpr int kTileMax = kRows * kNW;  // 64: the only tile height plans use
  static constexpr int kMergeG = GT;
  static constexpr int kPbufFloats = kRows * 8;  // per warp: 8 rows x 8 heads
  static constexpr int kC4 = HD / 4;             // float4 chunks per row
  // phase A: lane = (row rl of kRL, part of kLP)
  static constexpr int kLP = HD >= 96 ? 8 : 4;   // lanes per row
  static constexpr int kRL = 32 / kLP;           // rows per pass
  static constexpr int kPA = kRows / kRL;        // passes
  static constexpr int kEC = kC4 / kLP;          // chunks per lane and row
  // phase B: lane = (row rp of kBR, lane lr of kBL in the row), kBC chunks
  // lr + j * kBL (interleaved: a quarter warp reads 8 distinct chunks of one
  // row, conflict-free under the 128-byte swizzle)
  // (one chunk, one row per pass, when the o accumulators would not fit)
  static constexpr int kBC = HD == 96 ? (GT <= 3 ? 3 : 1) : (HD == 64 || GT <= 4 ? 2 : 1);
  static constexpr int kBL = kC4 / kBC;          // lanes per row
  static constexpr int kBR = 32 / kBL;           // rows per pass (lanes >= kBR * kBL idle)
  static constexpr int kPB = kRows / kBR;        // passes
  static constexpr int kPH = (GT + 3) / 4;       // float4s of p per row
  static constexpr bool kQReg = GT * kEC * 4 <= 64;
  static_assert(kC4 % kLP == 0, "head_dim must be a multiple of 16 (32 from 96 up)");
  static_assert(kC4 % kBC == 0 && kBL <= 32 && kRows % kBR == 0 &&
                    (kBR == 1 || kBR * kBL == 32), "phase B lane map");

  float m[GT], l[GT];  // m: warp-uniform; l: per-lane part (part-0 lanes own rows)
  float4 o[GT][kBC];   // phase B chunks of each head (sums over this lane's rows)
  float4 qr[kQReg ? GT : 1][kQReg ? kEC : 1];

  __device__ __forceinline__ void begin(const DecodeArgs&, const float* qs, int lane) {
#pragma unroll
    for (int h = 0; h < GT; ++h) {
      m[h] = -INFINITY;
      l[h] = 0.f;
#pragma unroll
      for (int j = 0; j < kBC; ++j) o[h][j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if constexpr (kQReg) {
      const int part = lane / kRL;
#pragma unroll
      for (int h = 0; h < GT; ++h)
#pragma unroll
        for (int i = 0; i < kEC; ++i)
          qr[h][i] = *reinterpret_cast<const float4*>(qs + h * HD + (part * kEC + i) * 4);
    }
  }

  template <bool kFull>
  __device__ __forceinline__ void phase_b(const char* Vs, const float* pbuf_w, int rb, int nvalid,
                                          int lane) {
    const bool on = kBR * kBL == 32 || lane < kBL;
    const int rp = on ? lane / kBL : 0, lr = on ? lane - rp * kBL : 0;
#pragma unroll
    for (int pb = 0; pb < kPB; ++pb) {
      const int r = pb * kBR + rp;
      float4 vv[kBC];
#pragma unroll
      for (int j = 0; j < kBC; ++j) {
        const float4 t = *reinterpret_cast<const float4*>(
            Vs + TL::chunk_off(kTileMax, rb + r, (lr + j * kBL) * 4));
        vv[j] = ((kFull || r < nvalid) && on) ? t : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      const float4* pr = reinterpret_cast<const float4*>(pbuf_w + r * 8);
#pragma unroll
      for (int u = 0; u < kPH; ++u) {
        const float4 pu = pr[u];
        const float pw[4] = {pu.x, pu.y, pu.z, pu.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = 4 * u + e;
          if (h < GT) {
#pragma unroll
            for (int j = 0; j < kBC; ++j) {
              o[h][j].x = fmaf(pw[e], vv[j].x, o[h][j].x);
              o[h][j].y = fmaf(pw[e], vv[j].y, o[h][j].y);
              o[h][j].z = fmaf(pw[e], vv[j].z, o[h][j].z);
              o[h][j].w = fmaf(pw[e], vv[j].w, o[h][j].w);
            }
          }
        }
      }
    }
  }

  __device__ __forceinline__ void consume(const DecodeArgs& a, const char* stage, int rows,
                                          float* pbuf_w, const float* qs, int w, int lane) {
    const int rb = w * kRows;
    if (rb >= rows) return;
    const int rl = lane % kRL, part = lane / kRL;
    const char* Ks = stage;
    const char* Vs = stage + kTileMax * HD * 4;
    float acc[kPA][GT];
#pragma unroll
    for (int pa = 0; pa < kPA; ++pa)
#pragma unroll
      for (int h = 0; h < GT; ++h) acc[pa][h] = 0.f;
#pragma unroll
    for (int i = 0; i < kEC; ++i) {
      const int c = part * kEC + i;
      float4 k4[kPA];
#pragma unroll
      for (int pa = 0; pa < kPA; ++pa)
        k4[pa] = *reinterpret_cast<const float4*>(
            Ks + TL::chunk_off(kTileMax, rb + pa * kRL + rl, c * 4));
#pragma unroll
      for (int h = 0; h < GT; ++h) {
        float4 q4;
        if constexpr (kQReg) q4 = qr[h][i];
        else q4 = *reinterpret_cast<const float4*>(qs + h * HD + c * 4);
#pragma unroll
        for (int pa = 0; pa < kPA; ++pa) {
          float& ac = acc[pa][h];
          ac = fmaf(q4.x, k4[pa].x, ac);
          ac = fmaf(q4.y, k4[pa].y, ac);
          ac = fmaf(q4.z, k4[pa].z, ac);
          ac = fmaf(q4.w, k4[pa].w, ac);
        }
      }
    }
    float p[kPA][kPH * 4];
#pragma unroll
    for (int h = 0; h < GT; ++h) {
      float sv[kPA];
      float mt = -INFINITY;
#pragma unroll
      for (int pa = 0; pa < kPA; ++pa) {
        float sc = acc[pa][h];
#pragma unroll
        for (int off = kRL; off < 32; off <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
        sv[pa] = (rb + pa * kRL + rl < rows) ? sc : -INFINITY;
        mt = fmaxf(mt, sv[pa]);
      }
#pragma unroll
      for (int off = 1; off < kRL; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float mn = fmaxf(m[h], mt);  // finite: row rb is valid
      const float alpha = fast_exp2(m[h] - mn);
      float ps = 0.f;
#pragma unroll
      for (int pa = 0; pa < kPA; ++pa) {
        p[pa][h] = fast_exp2(sv[pa] - mn);
        ps += p[pa][h];
      }
      l[h] = l[h] * alpha + (part == 0 ? ps : 0.f);
      m[h] = mn;
#pragma unroll
      for (int j = 0; j < kBC; ++j) {
        o[h][j].x *= alpha;
        o[h][j].y *= alpha;
        o[h][j].z *= alpha;
        o[h][j].w *= alpha;
      }
    }
    if (part == 0) {
#pragma unroll
      for (int pa = 0; pa < kPA; ++pa) {
#pragma unroll
        for (int h = GT; h < kPH * 4; ++h) p[pa][h] = 0.f;
        float4* pr = reinterpret_cast<float4*>(pbuf_w + (pa * kRL + rl) * 8);
#pragma unroll
        for (int u = 0; u < kPH; ++u)
          pr[u] = make_float4(p[pa][4 * u], p[pa][4 * u + 1], p[pa][4 * u + 2], p[pa][4 * u + 3]);
      }
    }
    __syncwarp();
    const int nvalid = rows - rb;
    if (nvalid >= kRows) phase_b<true>(Vs, pbuf_w, rb, nvalid, lane);
    else phase_b<false>(Vs, pbuf_w, rb, nvalid, lane);
    __syncwarp();
  }

  // Writes this warp's (o, m, l) for q heads h < group into
  // merge_w[h][merge_head_floats]: o at [0, HD), (m, l) at HD.
  __device__ __forceinline__ void to_merge(const DecodeArgs& a, float* merge_w, int lane) {
    const int rp = lane / kBL, lr = lane - rp * kBL;  // idle lanes (rp >= kBR) write nothing
#pragma unroll
    for (int h = 0; h < GT; ++h) {
      float lt = l[h];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, off);
#pragma unroll
      for (int j = 0; j < kBC; ++j) {
        float4 ov = o[h][j];
#pragma unroll
        for (int off = kBL; kBR > 1 && off < 32; off <<= 1) {  // join the rows of a pass
          ov.x += __shfl_xor_sync(0xffffffffu, ov.x, off);
          ov.y += __shfl_xor_sync(0xffffffffu, ov.y, off);
          ov.z += __shfl_xor_sync(0xffffffffu, ov.z, off);
          ov.w += __shfl_xor_sync(0xffffffffu, ov.w, off);
        }
        if (h < a.group && rp == 0)
          *reinterpret_cast<float4*>(merge_w + h * merge_head_floats<HD>() + (lr + j * kBL) * 4) = ov;
      }
      if (h < a.group && lane == 0)
        *reinterpret_cast<float2*>(merge_w + h * merge_head_floats<HD>() + HD) = make_float2(m[h], lt);
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

template <int HD>
struct F16Consumer {
  using TL = TileLayout<2, HD>;
  static constexpr int kElemBytes = 2;
  static constexpr bool kQ8 = false;
  // with the cp.async loader (batches) two CTAs an SM: the producer warp's
  // per-chunk copies limit one CTA (C3: 86 % of HBM against 70 %); the TMA
  // loader keeps one CTA with the deeper ring (C4: 77 % against 70 %)
  static constexpr int kCtasPerSm = 2;
  static constexpr int kNW = 4;
  static constexpr int kPbufFloats = 0;
  static constexpr int kTileMax = 16 * kNW;
  static constexpr int kMergeG = kMaxGroup;
  static constexpr int kKS = HD / 16;            // k-steps of q.k
  static constexpr int kNT = HD / 8;             // n-tiles of p.v
  static_assert(kKS % 2 == 0 && kNT % 2 == 0, "head_dim must be a multiple of 32");

  uint32_t qa[kKS][4];
  float m_run, l_run;
  float oacc[kNT][4];

  __device__ __forceinline__ static uint32_t chunk(uint32_t base, int tile, int row, int col) {
    return base + (uint32_t)TL::chunk_off(tile, row, col);
  }

  // qs: the group's pre-scaled q vectors [kMaxGroup][HD] in shared memory
  // (rows >= group are zero).
  __device__ __forceinline__ void begin(const DecodeArgs&, const float* qs, int lane) {
    const int gid = lane >> 2, tig = lane & 3;
    const float* qh = qs + gid * HD;
#pragma unroll
    for (int kk = 0; kk < kKS; ++kk) {
      const int c0 = kk * 16 + 2 * tig, c1 = c0 + 8;
      const float2 u = *reinterpret_cast<const float2*>(qh + c0);
      const float2 w = *reinterpret_cast<const float2*>(qh + c1);
      const float x0 = u.x, x1 = u.y, x2 = w.x, x3 = w.y;
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
                                          float* /*pbuf_w*/, const float* /*qs*/, int w,
                                          int lane) {
    const int rb = w * 16;
    if (rb >= rows) return;
    const int nvalid = min(16, rows - rb);
    const int tig = lane & 3;
    const uint32_t kbase = smem_u32(stage);
    const uint32_t vbase = kbase + (uint32_t)(a.tile * HD * 2);
    float sacc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sacc[nt][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kKS; kk += 2) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint32_t addr = chunk(kbase, a.tile, rb + nt * 8 + (lane & 7), kk * 16 + (lane >> 3) * 8);
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
          chunk(vbase, a.tile, rb + (lane & 7) + ((lane >> 3) & 1) * 8, (nt + (lane >> 4)) * 8);
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
      float* mh = merge_w + gid * merge_head_floats<HD>();
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
        *reinterpret_cast<float2*>(mh + nt * 8 + 2 * tig) =
            make_float2(oacc[nt][0] + oacc[nt][2], oacc[nt][1] + oacc[nt][3]);
      if (tig == 0) *reinterpret_cast<float2*>(mh + HD) = make_float2(m_run, lt);
    }
  }
};

// ---------------------------------------------------------------------------
// Q8 cache consumer: int8 K/V values with one FP16 scale per 32 values of a
// head row (Q8_0-style blocks; the scales of a key sit side by side, see
// kQ8ScaleHalves).  The hi/lo MMA scheme is F16Consumer's.  int8 values
// become FP16 exactly (|v| <= 128: the byte,
// offset by 128, is placed in the mantissa of 1024.0 and 1152 subtracted);
// the scales are applied in FP32: each 32-column block of q.k is multiplied
// by its key's K scale, and p is multiplied by its key's V scale of an output
// block before the hi/lo split.  ldmatrix reads int8 pairs as 16-bit elements:
//   q.k: the head_dim columns are permuted inside every 16-column step
//     (k index 2t+e <-> column 4t+e, 8+2t+e <-> 4t+2+e, for q and K alike,
//     which leaves the dot product unchanged), so the four bytes a lane gets
//     from a plain ldmatrix are its two B registers;
//   p.v: a transposed ldmatrix gives a lane keys (2t, 2t+1) x columns
//     (2j, 2j+1): bytes 0 and 2 are its B register for column 2j, bytes 1
//     and 3 for column 2j+1, so a 16-column group is two n-tiles (even and
//     odd columns) and a lane's outputs land on 4 consecutive columns.
// Keys past n_pos: scores -inf and p exactly 0 (their scale bytes may be
// anything), int8 values are finite.
// ---------------------------------------------------------------------------
// Two bytes of u (chosen by sel, a prmt selector placing them in the low
// bytes of the halves) as an exact half2; u holds signed int8 values offset
// by 128 (r ^ 0x80808080).
__device__ __forceinline__ uint32_t i8pair_to_h2(uint32_t u, uint32_t sel) {
  uint32_t h;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(h) : "r"(u), "r"(0x64646464u), "r"(sel));
  const __half2 x = __hsub2(*reinterpret_cast<const __half2*>(&h), __half2half2(__ushort_as_half(0x6480)));
  return *reinterpret_cast<const uint32_t*>(&x);
}
constexpr uint32_t kSelB01 = 0x4140u, kSelB23 = 0x4342u, kSelB02 = 0x4240u, kSelB13 = 0x4341u;

__device__ __forceinline__ void mma_1688(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// (x0, x1) as hi and lo half2 pairs: hi = half(x), lo = half(x - float(hi)).
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 hf = __half22float2(h);
  const __half2 l = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// 8 consumer warps, each owning 8 keys of a 64-row tile (two warps a
// scheduler: the per-warp chain is latency-bound).  q.k: m16n8k16, one
// ldmatrix.x4 covers the warp's 8 keys x 64 columns; p.v: m16n8k8 over the 8
// keys, one transposed ldmatrix.x4 covers 8 keys x 64 columns (8 n-tiles).
// O is rescaled only when a head's running max moved in this tile.
template <int HD>
struct Q8Consumer {
  using TL = TileLayout<1, HD>;
  static constexpr int kElemBytes = 1;
  static constexpr bool kQ8 = true;
  static constexpr int kCtasPerSm = 1;  // TMA loader only
  static constexpr int kNW = 8;
  static constexpr int kKeys = 8;       // keys of a tile per warp
  static constexpr int kPbufFloats = 0;
  static constexpr int kTileMax = kKeys * kNW;
  static constexpr int kMergeG = kMaxGroup;
  static constexpr int kKS = HD / 16;  // k-steps of q.k
  static constexpr int kNB = HD / 32;  // scale blocks of a head row
  static constexpr int kNT = HD / 8;   // n-tiles of p.v
  static_assert(HD == 64 || HD == 128, "Q8 cache: head_dim 64 or 128");

  uint32_t qa[kKS][4];
  float m_run, l_run;
  float oacc[kNT][4];

  __device__ __forceinline__ static uint32_t chunk(uint32_t base, int tile, int row, int col) {
    return base + (uint32_t)TL::chunk_off(tile, row, col);
  }

  __device__ __forceinline__ void begin(const DecodeArgs&, const float* qs, int lane) {
    const int gid = lane >> 2, tig = lane & 3;
    const float* qh = qs + gid * HD;
#pragma unroll
    for (int kk = 0; kk < kKS; ++kk) {
      // permuted columns: k (2t, 2t+1) <- 4t, 4t+1; k (2t+8, 2t+9) <- 4t+2, 4t+3
      const float4 u = *reinterpret_cast<const float4*>(qh + kk * 16 + 4 * tig);
      split2(u.x, u.y, qa[kk][0], qa[kk][1]);
      split2(u.z, u.w, qa[kk][2], qa[kk][3]);
    }
    m_run = -INFINITY;
    l_run = 0.f;
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) oacc[nt][e] = 0.f;
  }

  __device__ __forceinline__ void consume(const DecodeArgs& a, const char* stage, int rows,
                                          float* /*pbuf_w*/, const float* /*qs*/, int w,
                                          int lane) {
    const int rb = w * kKeys;
    if (rb >= rows) return;
    const int nvalid = min(kKeys, rows - rb);
    const int tig = lane & 3, mi = lane >> 3;
    const uint32_t kbase = smem_u32(stage);
    const uint32_t vbase = kbase + (uint32_t)(a.tile * HD);
    const char* sbase = stage + (size_t)2 * a.tile * HD;
    // the block scales of the lane's keys rb + 2*tig + e: halves 0..3 K, 4..7 V
    uint4 sc[2];
#pragma unroll
    for (int e = 0; e < 2; ++e)
      sc[e] = *reinterpret_cast<const uint4*>(sbase + (rb + 2 * tig + e) * kQ8ScaleRowBytes);
    auto scale_of = [&](int e, int idx) {
      const uint32_t word = (idx >> 1) == 0 ? sc[e].x : (idx >> 1) == 1 ? sc[e].y
                            : (idx >> 1) == 2 ? sc[e].z : sc[e].w;
      return __half2float(
          __ushort_as_half((unsigned short)((idx & 1) ? (word >> 16) : (word & 0xffffu))));
    };
    // ---- scores: per 32-column block, q.k times the key's K scale
    float s[2] = {0.f, 0.f};
#pragma unroll
    for (int q4 = 0; q4 < kKS / 4; ++q4) {
      uint32_t r[4];  // matrix j: the warp's 8 keys x k-step 4*q4 + j
      ldsm_x4(chunk(kbase, a.tile, rb + (lane & 7), (4 * q4 + mi) * 16), r[0], r[1], r[2], r[3]);
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] ^= 0x80808080u;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const int b = 2 * q4 + hb;
        float tmp[4] = {0.f, 0.f, 0.f, 0.f};
        mma_16816(tmp, qa[2 * b], i8pair_to_h2(r[2 * hb], kSelB01),
                  i8pair_to_h2(r[2 * hb], kSelB23));
        mma_16816(tmp, qa[2 * b + 1], i8pair_to_h2(r[2 * hb + 1], kSelB01),
                  i8pair_to_h2(r[2 * hb + 1], kSelB23));
#pragma unroll
        for (int e = 0; e < 2; ++e) s[e] = fmaf(tmp[e] + tmp[2 + e], scale_of(e, b), s[e]);
      }
    }
    // ---- online softmax over the warp's 8 keys
    float mt = -INFINITY;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      s[e] = 2 * tig + e < nvalid ? s[e] : -INFINITY;
      mt = fmaxf(mt, s[e]);
    }
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    const float mn = fmaxf(m_run, mt);  // finite: key rb is valid
    const float alpha = fast_exp2(m_run - mn);
    float p[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) p[e] = fast_exp2(s[e] - mn);
    l_run = l_run * alpha + (p[0] + p[1]);
    if (__any_sync(0xffffffffu, mn != m_run)) {
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) oacc[nt][e] *= alpha;
    }
    m_run = mn;
    // ---- p.v: per output block, p times the key's V scale (0 past n_pos)
#pragma unroll
    for (int q4 = 0; q4 < HD / 64; ++q4) {
      uint32_t r[4];  // matrix j: the warp's 8 keys x columns 64*q4 + 16*j .. +15
      ldsm_x4_t(chunk(vbase, a.tile, rb + (lane & 7), 64 * q4 + 16 * mi), r[0], r[1], r[2], r[3]);
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] ^= 0x80808080u;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const int b = 2 * q4 + hb;
        float pv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) pv[e] = 2 * tig + e < nvalid ? p[e] * scale_of(e, 4 + b) : 0.f;
        uint32_t ahi, alo;
        split2(pv[0], pv[1], ahi, alo);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = 2 * hb + jj;
          const int c = 4 * q4 + j;  // 16-column group: n-tiles 2c (even), 2c+1 (odd)
          mma_1688(oacc[2 * c], ahi, alo, i8pair_to_h2(r[j], kSelB02));
          mma_1688(oacc[2 * c + 1], ahi, alo, i8pair_to_h2(r[j], kSelB13));
        }
      }
    }
  }

  __device__ __forceinline__ void to_merge(const DecodeArgs& a, float* merge_w, int lane) {
    const int gid = lane >> 2, tig = lane & 3;
    float lt = l_run;
    lt += __shfl_xor_sync(0xffffffffu, lt, 1);
    lt += __shfl_xor_sync(0xffffffffu, lt, 2);
    if (gid < a.group) {
      float* mh = merge_w + gid * merge_head_floats<HD>();
      // n-tiles 2c (even columns) and 2c+1 (odd) of 16-column group c: this
      // lane's columns 16c + 4*tig .. +3
#pragma unroll
      for (int c = 0; c < HD / 16; ++c) {
        const float(&ev)[4] = oacc[2 * c];
        const float(&od)[4] = oacc[2 * c + 1];
        *reinterpret_cast<float4*>(mh + 16 * c + 4 * tig) =
            make_float4(ev[0] + ev[2], od[0] + od[2], ev[1] + ev[3], od[1] + od[3]);
      }
      if (tig == 0) *reinterpret_cast<float2*>(mh + HD) = make_float2(m_run, lt);
    }
  }
};

// ---------------------------------------------------------------------------
// Output helpers
// ---------------------------------------------------------------------------
// Exchange-buffer record row: o[HD], m, l, 2 pad (16-byte rows).
template <int HD>
constexpr int xch_row_floats() { return HD + 4; }

// An exchange word: the value's bits and the call's epoch, stored and loaded
// as one 64-bit single-copy-atomic access.
__device__ __forceinline__ uint64_t xch_word(float v, uint32_t ep) {
  return (uint64_t)__float_as_uint(v) | ((uint64_t)ep << 32);
}

// record_mode 2 writes this rank's record straight into slot [ep & 1][own
// rank] of every rank's exchange buffer (peer stores over NVLink), each word
// tagged with the call's epoch `ep`.
template <int HD, bool XCH = false>
__device__ __forceinline__ void write_final(const DecodeArgs& a, int b, int hq, int d, float O,
                                            float M, float L, uint32_t ep = 0) {
  const int64_t row = (int64_t)b * a.n_heads + hq;
  if constexpr (XCH) {
    const float o = L > 0.f ? O / L : 0.f;
    const float m = L > 0.f ? M * kLn2 : -INFINITY;
    for (int r = 0; r < a.xch_world; ++r) {
      uint64_t* rec =
          reinterpret_cast<uint64_t*>(a.xch_bases[r] + xch_rec_offset((int)(ep & 1u), a.xch_rank)) +
          row * xch_row_floats<HD>();
      st_relaxed_sys_u64(rec + d, xch_word(o, ep));
      if (d == 0) {
        st_relaxed_sys_u64(rec + HD, xch_word(m, ep));
        st_relaxed_sys_u64(rec + HD + 1, xch_word(L, ep));
      }
    }
  } else if (a.record_mode) {
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

template <int HD, bool XCH = false>
__device__ __forceinline__ void write_final4(const DecodeArgs& a, int b, int hq, int d, float4 O,
                                             float M, float L, uint32_t ep = 0) {
  if constexpr (XCH) {
    const float m = L > 0.f ? M * kLn2 : -INFINITY;
    const int64_t row = (int64_t)b * a.n_heads + hq;
    const uint64_t w0 = xch_word(L > 0.f ? O.x / L : 0.f, ep), w1 = xch_word(L > 0.f ? O.y / L : 0.f, ep);
    const uint64_t w2 = xch_word(L > 0.f ? O.z / L : 0.f, ep), w3 = xch_word(L > 0.f ? O.w / L : 0.f, ep);
    for (int r = 0; r < a.xch_world; ++r) {
      uint64_t* rec =
          reinterpret_cast<uint64_t*>(a.xch_bases[r] + xch_rec_offset((int)(ep & 1u), a.xch_rank)) +
          row * xch_row_floats<HD>();
      st_relaxed_sys_u64x2(rec + d, w0, w1);  // rows are 32-byte aligned, d % 4 == 0
      st_relaxed_sys_u64x2(rec + d + 2, w2, w3);
      if (d == 0) st_relaxed_sys_u64x2(rec + HD, xch_word(m, ep), xch_word(L, ep));
    }
  } else if (a.record_mode) {
    write_final<HD>(a, b, hq, d, O.x, M, L);
    write_final<HD>(a, b, hq, d + 1, O.y, M, L);
    write_final<HD>(a, b, hq, d + 2, O.z, M, L);
    write_final<HD>(a, b, hq, d + 3, O.w, M, L);
  } else {
    const int64_t row = (int64_t)b * a.n_heads + hq;
    float4 r;
    r.x = L > 0.f ? O.x / L : 0.f;
    r.y = L > 0.f ? O.y / L : 0.f;
    r.z = L > 0.f ? O.z / L : 0.f;
    r.w = L > 0.f ? O.w / L : 0.f;
    *reinterpret_cast<float4*>(a.out + row * HD + d) = r;
  }
}

// ---------------------------------------------------------------------------
// Phase trace (DecodeArgs::trace, off when null): %globaltimer stamps per CTA,
// kTraceWords words a CTA, overwritten by every launch.
// ---------------------------------------------------------------------------
constexpr int kTraceWords = 16;
enum TraceSlot : int {
  kTrEntry = 0,      // kernel entry
  kTrWait = 1,       // dependency wait returned
  kTrQ = 2,          // q of the first piece in shared memory
  kTrFirstTile = 3,  // first tile ready for the consumers
  kTrLastTile = 4,   // last tile consumed
  kTrCounted = 5,    // piece stored and counted (or final, one-piece segment)
  kTrMerged = 6,     // merger: segment merged and written
  kTrPublished = 7,  // merger, sharded: every rank's records merged into xb
  kTrProdFirst = 8,  // producer: early copies forwarded, first copy after the wait issued
  kTrProdLast = 9,   // producer: last copy issued
  kTrInfo = 10,      // tiles | early tiles << 16 | merger << 24 | smid << 32
  kTrExit = 11,      // consumers done
  kTrGather = 12,    // merger: first chunk of pieces copied into shared memory
  kTrFolded = 13,    // merger: every piece folded (before the result is written)
  kTrMergeCycles = 14,  // merger, first head: SM cycles of copy | weights | sums | rest (16 bits each)
  kTrMergeTries = 15,   // merger, first head: copy rounds
};

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int HD, class Consumer, int LOADER, bool XCH>
__global__ void __launch_bounds__((Consumer::kNW + 1) * 32,
                                  (LOADER == 1 && !XCH) ? Consumer::kCtasPerSm : 1)
    decode_kernel(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(1024) char smem_raw[];
  // swizzled TMA tiles need 1024-byte aligned stages (the host adds the slack)
  char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr int NW = Consumer::kNW;
  constexpr int kNCT = NW * 32;  // consumer threads
  constexpr int kMG = Consumer::kMergeG;
  constexpr int esize = Consumer::kElemBytes;
  using TL = TileLayout<esize, HD>;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int B = a.batch, n_kv = a.n_kv, G = a.group;
  const int unit_rows = a.tile;  // work units are whole tiles
  const int32_t P = (int32_t)gridDim.x;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bars);
  uint64_t* empty = full + a.stages;
  uint64_t* land = empty + a.stages;  // early copies (issued before the dependency wait)
  uint64_t* ep_bar = land + a.stages;  // the call epoch is in flags[4]
  int32_t* seq_start = reinterpret_cast<int32_t*>(smem + a.off_seq);  // [B+1] (units)
  int32_t* nunits = seq_start + (B + 1);                              // [B]
  int32_t* npos = nunits + B;                                         // [B]
  float* qs = reinterpret_cast<float*>(smem + a.off_q);                // [kMaxGroup][HD]
  float* pbuf = reinterpret_cast<float*>(smem + a.off_pbuf);           // [NW][kPbufFloats]
  float* merge = reinterpret_cast<float*>(smem + a.off_merge);         // [NW][kMG][HD+4]
  // [0] abort  [1] this CTA merges  [2] exchange epoch  [3] position hint
  // [4] call epoch  [5] early copies issued  [6] first tile stamped
  volatile int* flags = reinterpret_cast<volatile int*>(smem + a.off_flags);
  float2* rope_cs = reinterpret_cast<float2*>(smem + a.off_rope);      // [HD/2] (fused RoPE)
  // phase stamps (a.trace lives in the parameter bank: no register stays live)
  // Only the tensor-map loader's launches are traced: in the two-CTA
  // batched kernel (cp.async loader, 168 registers) the trace code alone made
  // the compiler spill.
  constexpr bool kTraced = LOADER == 0;
  auto stamp = [&](int slot) {
    if (kTraced && a.trace) a.trace[(size_t)blockIdx.x * kTraceWords + slot] = global_timer_ns();
  };

  // The deal's mode does not depend on the lengths (see make_deal).  The
  // tensor-map loader serves one sequence with n_kv <= P only (the host plans
  // other single-sequence calls on the cp.async loader): always round robin.
  if (LOADER == 0 && (B != 1 || n_kv > P)) {
    if (threadIdx.x == 0) atomicCAS(a.status, 0, GLA_ERR_NOT_SUPPORTED);
    return;
  }
  const bool mode1 = LOADER == 0 || (B == 1 && n_kv <= P);
  // Early KV prefetch (programmatic dependent launch): the producer starts
  // streaming this CTA's first tiles while the preceding kernel on the stream
  // drains.  Which tiles a CTA owns depends on the length only through their
  // count (round robin), so the count comes from a hint: the host n_pos, or
  // (level 2) the device position read before the wait, which may be stale.
  // Every early copy lands on its own barrier land[k]; after the wait the
  // producer drops the copies the true length does not need, rewrites in
  // shared memory the two newest rows [n_pos - 2, n_pos) of the tiles it
  // keeps (the rows a preceding kernel may still have been writing: a KV
  // append at n_pos - 1, the previous token's fused append at n_pos - 2),
  // and hands each kept stage to the consumers.  Everything else a preceding
  // kernel writes (q, the positions, the workspace) is read after the wait.
  const bool early = LOADER == 0 && a.early_kv >= 1 &&
                     (a.n_pos_dev == nullptr || (a.early_kv >= 2 && mode1));

  if (tid == 0) {
    stamp(kTrEntry);
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], LOADER == 0 ? 1 : 32);
      mbar_init(&empty[s], NW);
      mbar_init(&land[s], 1);
    }
    mbar_init(ep_bar, 1);
    flags[0] = 0;
    flags[1] = 0;
    flags[2] = 0;
    flags[4] = 0;
    flags[6] = 0;
    int32_t hint = 0;
    if (early) {
      hint = a.n_pos_dev ? ld_relaxed_gpu_s32(a.n_pos_dev) + a.n_pos_add : a.n_pos;
      hint = hint < 0 ? 0 : (hint > a.n_pos_cap ? a.n_pos_cap : hint);
    }
    flags[3] = hint;
    flags[5] = 0;
    fence_mbarrier_init();
  }
  if (LOADER == 0 && warp == NW && lane == 0) {
    prefetch_tmap(&a.tmap_k);
    prefetch_tmap(&a.tmap_v);
  }
  __syncthreads();
  const int32_t hint = flags[3];

  // per-sequence rows and unit prefix (warp 0 scans 32 sequences at a time)
  auto scan_sequences = [&]() {
    if (warp == 0) {
      int32_t carry = 0;
      for (int base = 0; base < B; base += 32) {
        const int b = base + lane;
        int32_t np = 0, nu = 0;
        if (b < B) {
          np = a.n_pos_dev ? a.n_pos_dev[b] + a.n_pos_add : a.n_pos;
          np = np < 0 ? 0 : np;
          if (np > a.n_pos_cap) {
            atomicCAS(a.status, 0, GLA_ERR_INVALID_ARG);
            np = a.n_pos_cap;
          }
          nu = ceil_div(np, unit_rows);
          npos[b] = np;
          nunits[b] = nu;
        }
        int32_t incl = nu;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          int32_t y = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += y;
        }
        if (b < B) seq_start[b] = (carry + incl - nu) * n_kv;
        carry += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) seq_start[B] = carry * n_kv;
    }
  };
  // Fused RoPE: (cos, sin) of every pair at position `pos`, once per CTA.
  auto rope_table = [&](int pos) {
    for (int i = tid; i < HD / 2; i += blockDim.x) {
      float c, sn;
      rope_cos_sin(pos, i, HD, a.rope_theta, &c, &sn);
      rope_cs[i] = make_float2(c, sn);
    }
  };
  // Fused RoPE, newest row staged in shared memory (stage st, row r of the
  // tile): the producer warp writes kv head g's rotated key row and value row
  // to the caches (for later calls) and over the stale row of the staged tile
  // (128B-swizzled FP32 layout), after the stage's copy has landed.
  auto append_row_stage = [&](int g, int st, int r) {
    if constexpr (Consumer::kElemBytes != 4) return;  // fused RoPE writes FP32 caches only
    const int pos = npos[0] - 1;
    float* kc = const_cast<float*>(static_cast<const float*>(a.k)) + (int64_t)pos * a.kv_stride +
                (int64_t)g * HD;
    float* vc = const_cast<float*>(static_cast<const float*>(a.v)) + (int64_t)pos * a.kv_stride +
                (int64_t)g * HD;
    const float* kn = a.rope_k + (int64_t)g * HD;
    const float* vn = a.rope_v + (int64_t)g * HD;
    char* ks = smem + (size_t)st * a.stage_bytes;
    char* vs = ks + (size_t)a.tile * HD * esize;
    auto at = [&](char* base, int col) {
      return reinterpret_cast<float*>(base + TL::chunk_off(a.tile, r, col & ~3) + (col & 3) * 4);
    };
    for (int ic = lane; ic < HD / 2; ic += 32) {
      int i0, i1;
      rope_pair(a.rope_style, ic, HD, &i0, &i1);
      const float2 cs = rope_cs[ic];
      float o0, o1;
      rope_rotate(kn[i0], kn[i1], cs.x, cs.y, &o0, &o1);
      const float v0 = vn[i0], v1 = vn[i1];
      kc[i0] = o0;
      kc[i1] = o1;
      vc[i0] = v0;
      vc[i1] = v1;
      *at(ks, i0) = o0;
      *at(ks, i1) = o1;
      *at(vs, i0) = v0;
      *at(vs, i1) = v1;
    }
  };
  // Fused RoPE + append, producer warp, before a copy issued after the wait
  // reads row n_pos - 1: kv head g's rotated key row and its value row are
  // written there, then a proxy fence orders those generic stores before the
  // tensor copy that reads the row back.
  auto append_row = [&](int g) {
    if constexpr (Consumer::kElemBytes != 4) return;  // fused RoPE writes FP32 caches only
    const int pos = npos[0] - 1;
    float* kc = const_cast<float*>(static_cast<const float*>(a.k)) + (int64_t)pos * a.kv_stride +
                (int64_t)g * HD;
    float* vc = const_cast<float*>(static_cast<const float*>(a.v)) + (int64_t)pos * a.kv_stride +
                (int64_t)g * HD;
    const float* kn = a.rope_k + (int64_t)g * HD;
    const float* vn = a.rope_v + (int64_t)g * HD;
    for (int ic = lane; ic < HD / 2; ic += 32) {
      int i0, i1;
      rope_pair(a.rope_style, ic, HD, &i0, &i1);
      const float2 cs = rope_cs[ic];
      float o0, o1;
      rope_rotate(kn[i0], kn[i1], cs.x, cs.y, &o0, &o1);
      kc[i0] = o0;
      kc[i1] = o1;
      vc[i0] = vn[i0];
      vc[i1] = vn[i1];
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncwarp();
  };
  // Producer warp, after the wait: cache row `row` of kv head g (K, V and, for
  // a Q8 cache, the scale row) re-read from global memory into row r of the
  // tile staged in stage st.
  auto copy_row_to_stage = [&](int st, int g, int row, int r) {
    if constexpr (LOADER == 0) {
      char* ks = smem + (size_t)st * a.stage_bytes;
      char* vs = ks + (size_t)a.tile * HD * esize;
      const int64_t off = ((int64_t)row * a.kv_stride + (int64_t)g * HD) * esize;
      const char* kg = static_cast<const char*>(a.k) + off;
      const char* vg = static_cast<const char*>(a.v) + off;
      constexpr int kCpr = HD * esize / 16;  // 16-byte chunks per row
      uint4 x[(2 * kCpr + 31) / 32];
#pragma unroll
      for (int u = 0; u < (2 * kCpr + 31) / 32; ++u) {
        const int c = lane + 32 * u;
        if (c < 2 * kCpr) {
          const int cc = c < kCpr ? c : c - kCpr;
          x[u] = __ldcg(reinterpret_cast<const uint4*>((c < kCpr ? kg : vg) + cc * 16));
        }
      }
#pragma unroll
      for (int u = 0; u < (2 * kCpr + 31) / 32; ++u) {
        const int c = lane + 32 * u;
        if (c < 2 * kCpr) {
          const int cc = c < kCpr ? c : c - kCpr;
          *reinterpret_cast<uint4*>((c < kCpr ? ks : vs) + TL::chunk_off(a.tile, r, cc * (16 / esize))) =
              x[u];
        }
      }
      if constexpr (Consumer::kQ8) {
        if (lane == 0) {
          const char* sg = static_cast<const char*>(a.scales) +
                           ((int64_t)row * n_kv + g) * kQ8ScaleRowBytes;
          *reinterpret_cast<uint4*>(ks + (size_t)2 * a.tile * HD + r * kQ8ScaleRowBytes) =
              __ldcg(reinterpret_cast<const uint4*>(sg));
        }
      }
    }
  };
  // TMA loads of one tile (LOADER 0): whole boxes of `tile` rows; rows past
  // the tensor map's extent are zero-filled, so the byte count is the boxes'
  // size.  Rows past n_pos inside the extent are loaded and masked later.
  auto tma_tile = [&](int st, const Tile& t, uint64_t pol, uint64_t* bar) {
    char* ks = smem + (size_t)st * a.stage_bytes;
    char* vs = ks + (size_t)a.tile * HD * esize;
    mbar_arrive_expect_tx(bar, (uint32_t)(2 * a.tile * HD * esize +
                                          (Consumer::kQ8 ? a.tile * kQ8ScaleRowBytes : 0)));
#pragma unroll
    for (int cb = 0; cb < TL::kBlocks; ++cb) {
      const int x = t.g * HD + cb * TL::kCW;
      const size_t off = (size_t)cb * a.tile * TL::kRowB;
      tma_load_2d(ks + off, &a.tmap_k, x, t.row0, bar, pol);
      tma_load_2d(vs + off, &a.tmap_v, x, t.row0, bar, pol);
    }
    // Q8 cache: the K and V block scales of kv head g, one 16-byte row a key
    if constexpr (Consumer::kQ8)
      tma_load_2d(ks + (size_t)2 * a.tile * HD, &a.tmap_s, t.g * kQ8ScaleHalves, t.row0,
                  bar, pol);
  };

  // ---------------- early copies (before the dependency wait) ----------------
  int32_t n_early = 0;  // producer warp: the ring's first pass, copied early
  if (early) {
    if (a.rope) rope_table(hint - 1);  // recomputed after the wait if the position moved
    if (warp == NW) {
      const uint64_t pol = l2_evict_first_policy();
      const int32_t nu_h = ceil_div(hint, unit_rows);
      int32_t ss[2] = {0, n_kv * nu_h}, nus[1] = {nu_h};
      CtaTiles ct = cta_tiles_of(make_deal(ss[1], P, 1, n_kv, nu_h), blockIdx.x, ss, nus, 1);
      Tile t;
      int32_t seg = -1;
      while (n_early < a.stages && ct.next(nus, 1, n_kv, 1, unit_rows, t)) {
        if (lane == 0) {
          // warm L2 with the inputs read right after the wait (the group's
          // q vectors; fused RoPE: the new key and value rows of kv head g)
          if (t.g != seg) {
            seg = t.g;
            prefetch_l2_bulk(a.q + (int64_t)t.g * G * HD, (uint32_t)(G * HD * sizeof(float)));
            if (a.rope) {
              prefetch_l2_bulk(a.rope_k + (int64_t)t.g * HD, (uint32_t)(HD * sizeof(float)));
              prefetch_l2_bulk(a.rope_v + (int64_t)t.g * HD, (uint32_t)(HD * sizeof(float)));
            }
          }
          tma_tile(n_early, t, pol, &land[n_early]);
        }
        ++n_early;
      }
      if (lane == 0) flags[5] = n_early;
    }
  }
  // Nothing below may read memory a preceding kernel writes (n_pos, q, the
  // newest cache rows, the workspace) before that kernel has completed.
  pdl_wait();
  pdl_launch_dependents();
  if (tid == 0) stamp(kTrWait);
  scan_sequences();
  __syncthreads();
  if (a.rope && (!early || npos[0] != hint)) {
    rope_table(npos[0] - 1);
    __syncthreads();
  }

  const int32_t W = seq_start[B];
  const Deal deal = make_deal(W, P, B, n_kv, nunits[0]);
  auto cta_tiles = [&]() { return cta_tiles_of(deal, blockIdx.x, seq_start, nunits, B); };

  if (warp == NW) {
    // ---------------- producer ----------------
    // The call's epoch (tags of the piece words): every CTA takes a ticket
    // from the workspace's epoch word (epoch << 32 | CTAs of this call so
    // far); the last CTA to take one moves the word to the next epoch.  All
    // CTAs of a call see the same epoch, every call a larger one.  Lane 31
    // takes it and settles it after the copies are issued, when the result
    // has long arrived; the consumers read it behind ep_bar.
    unsigned long long ticket = 0;
    if (lane == 31) ticket = atomicAdd(a.ws_epoch, 1ull);
    auto settle_ticket = [&]() {
      if (lane == 31) {
        const uint32_t call_ep = (uint32_t)(ticket >> 32) + 1u;
        flags[4] = (int)call_ep;
        if ((uint32_t)ticket == (uint32_t)P - 1u)
          atomicExch(a.ws_epoch, (unsigned long long)call_ep << 32);
        mbar_arrive(ep_bar);
      }
    };
    // contiguous deal: a CTA may finish a piece (and need the epoch) while
    // this warp still waits for ring slots of its next piece, so settle now
    if (deal.mode == 0) settle_ticket();
    const uint64_t pol = l2_evict_first_policy();
    CtaTiles ct = cta_tiles();
    Tile t;
    // the early copies: keep (rewrite the newest rows, hand to the
    // consumers) or drop; every one is waited for, so no copy is still in
    // flight when the CTA exits
    for (int32_t k = 0; k < n_early; ++k) {
      const bool keep = ct.next(nunits, B, n_kv, 1, unit_rows, t);
      bool landed = true;
      if (lane == 0) landed = mbar_wait(&land[k], 0, flags, a.status);
      landed = __shfl_sync(0xffffffffu, landed, 0);
      if (!keep) continue;
      if (landed) {
        const int np = npos[t.b];
        const int r_hi = imin(t.row0 + unit_rows, np);
        for (int r = (t.row0 > np - 2 ? t.row0 : np - 2); r < r_hi; ++r) {
          if (a.rope && r == np - 1) append_row_stage(t.g, k, r - t.row0);
          else copy_row_to_stage(k, t.g, r, r - t.row0);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[k]);  // the stage's only arrival this pass
    }
    if (lane == 0) stamp(kTrProdFirst);
    int cur_b = -1;
    const char* kb = nullptr;
    const char* vb = nullptr;
    int st = n_early % a.stages;
    uint32_t phase = n_early < a.stages ? 1u : 0u;  // empty-barrier parity of the ring pass
    for (; ct.next(nunits, B, n_kv, 1, unit_rows, t);) {
      if (!mbar_wait(&empty[st], phase, flags, a.status)) break;
      if constexpr (LOADER == 0) {
        if (a.rope && t.row0 + t.units * unit_rows >= npos[t.b]) append_row(t.g);
        if (lane == 0) tma_tile(st, t, pol, &full[st]);
        __syncwarp();
      } else {
        if (t.b != cur_b) {
          cur_b = t.b;
          kb = static_cast<const char*>(a.k_ptrs ? a.k_ptrs[cur_b] : a.k);
          vb = static_cast<const char*>(a.v_ptrs ? a.v_ptrs[cur_b] : a.v);
          // caller-supplied device pointers: a null or unaligned base would
          // make the copies fault, so refuse it and drain instead
          if (kb == nullptr || vb == nullptr ||
              ((reinterpret_cast<uintptr_t>(kb) | reinterpret_cast<uintptr_t>(vb)) & 15u)) {
            atomicCAS(a.status, 0, GLA_ERR_ALIGNMENT);
            flags[0] = 1;
            break;
          }
        }
        char* ks = smem + (size_t)st * a.stage_bytes;
        char* vs = ks + (size_t)a.tile * HD * esize;
        const int rows = imin(t.units * unit_rows, npos[t.b] - t.row0);
        constexpr int kCpr = HD * esize / 16;  // 16-byte chunks per row
        for (int idx = lane; idx < rows * kCpr; idx += 32) {
          const int r = idx / kCpr, c = idx - r * kCpr;
          const int64_t off =
              ((int64_t)(t.row0 + r) * a.kv_stride + (int64_t)t.g * HD) * esize + c * 16;
          const int soff = TL::chunk_off(a.tile, r, c * (16 / esize));
          cp_async_16(ks + soff, kb + off, pol);
          cp_async_16(vs + soff, vb + off, pol);
        }
        cp_async_arrive_noinc(&full[st]);
      }
      if (++st == a.stages) {
        st = 0;
        phase ^= 1u;
      }
    }
    if (lane == 0) stamp(kTrProdLast);
    // round robin: the one piece ends after its last tile was issued
    if (deal.mode == 1) settle_ticket();
    return;
  }

  // ---------------- consumers ----------------
  // Peer exchange (record_mode 2, one sequence).  The CTA that holds kv head
  // g's final records reads g's epoch first (epoch_read) and write_final
  // stores the records, each word tagged with the epoch, straight into slot
  // [epoch & 1][own rank] of every rank's exchange buffer.  publish_merge
  // advances g's epoch and merges the world records of g into xb as they
  // arrive: every thread polls its words until all carry the call's epoch
  // (bounded: a rank that never writes latches GLA_ERR_TIMEOUT), then
  // M = max m_r, w_r = l_r e^(m_r - M), xb = sum w_r o_r / sum w_r.  Only the
  // publishing CTA reads or advances g's epoch, after the dependency wait,
  // so the previous call's advance is visible.
  auto epoch_read = [&](int g) {
    if (XCH && tid == 0)
      flags[2] = (int)(*reinterpret_cast<volatile uint32_t*>(a.xch_local + xch_epoch_offset(g)) + 1u);
  };
  // Merger r of nm (see finish_piece) publishes q heads r, r + nm, ... of
  // kv head g; merger 0 (the last to count) advances g's epoch.
  auto publish_merge = [&](int g, int r, int nm) {
    if constexpr (!XCH) return;
    const uint32_t ep = (uint32_t)flags[2];
    const int par = (int)(ep & 1u), W = a.xch_world;
    if (tid == 0 && r == 0)
      *reinterpret_cast<volatile uint32_t*>(a.xch_local + xch_epoch_offset(g)) = ep;
    constexpr int kXR = xch_row_floats<HD>();
    constexpr int kD4 = HD / 4;
    // ranks polled together (bounds the registers; the FP32 kernels have fewer)
    constexpr int kRG = Consumer::kElemBytes == 2 ? 4 : 2;
    const int n_heads_mine = (G - r + nm - 1) / nm;
    for (int it = tid; it < n_heads_mine * kD4; it += kNCT) {
      const int hq = g * G + r + (it / kD4) * nm, d = (it % kD4) * 4;
      float M = -INFINITY, L = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r0 = 0; r0 < W; r0 += kRG) {
        uint64_t wv[kRG][6];  // per rank: o[d..d+3], m, l
        unsigned long long t0 = 0;
        for (;;) {
          bool all = true;
#pragma unroll
          for (int u = 0; u < kRG; ++u) {
            if (r0 + u < W) {
              const uint64_t* rec =
                  reinterpret_cast<const uint64_t*>(a.xch_local + xch_rec_offset(par, r0 + u)) +
                  (int64_t)hq * kXR;
              ld_relaxed_sys_u64x2(rec + d, wv[u][0], wv[u][1]);
              ld_relaxed_sys_u64x2(rec + d + 2, wv[u][2], wv[u][3]);
              ld_relaxed_sys_u64x2(rec + HD, wv[u][4], wv[u][5]);
#pragma unroll
              for (int e = 0; e < 6; ++e) all = all && (uint32_t)(wv[u][e] >> 32) == ep;
            }
          }
          if (all || flags[0]) break;
          if (t0 == 0) {
            t0 = global_timer_ns();
          } else if (global_timer_ns() - t0 > kWaitTimeoutNs) {
            flags[0] = 1;
            atomicCAS(a.status, 0, GLA_ERR_TIMEOUT);
            break;
          }
        }
        // fold the group in with a running log-sum-exp
#pragma unroll
        for (int u = 0; u < kRG; ++u) {
          const float l = r0 + u < W ? __uint_as_float((uint32_t)wv[u][5]) : 0.f;
          if (l > 0.f) {
            const float m = __uint_as_float((uint32_t)wv[u][4]);
            const float Mn = fmaxf(M, m);
            const float sc = M == -INFINITY ? 0.f : __expf(M - Mn);
            const float w = l * __expf(m - Mn);
            acc.x = acc.x * sc + w * __uint_as_float((uint32_t)wv[u][0]);
            acc.y = acc.y * sc + w * __uint_as_float((uint32_t)wv[u][1]);
            acc.z = acc.z * sc + w * __uint_as_float((uint32_t)wv[u][2]);
            acc.w = acc.w * sc + w * __uint_as_float((uint32_t)wv[u][3]);
            L = L * sc + w;
            M = Mn;
          }
        }
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      *reinterpret_cast<float4*>(a.xch_out + (int64_t)hq * HD + d) =
          make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    }
    consumer_sync(kNCT);
  };

  // segments with no rows (n_pos <= 0) produce zeros / empty records
  for (int s = blockIdx.x; s < B * n_kv; s += gridDim.x) {
    const int b = s / n_kv, g = s - b * n_kv;
    if (nunits[b] == 0) {
      epoch_read(g);
      consumer_sync(kNCT);
      for (int idx = tid; idx < G * HD; idx += kNCT)
        write_final<HD, XCH>(a, b, g * G + idx / HD, idx % HD, 0.f, 0.f, 0.f, (uint32_t)flags[2]);
      if constexpr (XCH) publish_merge(g, 0, 1);
    }
  }
  const CtaTiles ct = cta_tiles();
  const int my_tiles = ct.count;
  if (my_tiles == 0) return;

  Consumer cons;
  float* pbuf_w = pbuf + warp * Consumer::kPbufFloats;
  constexpr int kMH = merge_head_floats<HD>();
  float* merge_w = merge + warp * kMG * kMH;
  constexpr int kSH = slot_head_floats<HD>();  // words per head in a piece slot
  constexpr int kMergeBytes = NW * kMG * kMH * (int)sizeof(float);  // the warp merge buffer

  // The group's q vectors, pre-scaled by scale*log2(e), rows >= G zeroed.
  auto load_q = [&](int b, int g) {
    const float* qb = a.q + ((int64_t)b * a.n_heads + (int64_t)g * G) * HD;
    if (a.rope) {  // fused RoPE: rotate on the way in (the caller's q stays as it was)
      for (int p = tid; p < kMaxGroup * (HD / 2); p += kNCT) {
        const int h = p / (HD / 2), ic = p - h * (HD / 2);
        int i0, i1;
        rope_pair(a.rope_style, ic, HD, &i0, &i1);
        float o0 = 0.f, o1 = 0.f;
        if (h < G) {
          const float2 cs = rope_cs[ic];
          rope_rotate(qb[h * HD + i0], qb[h * HD + i1], cs.x, cs.y, &o0, &o1);
        }
        qs[h * HD + i0] = o0 * a.q_scale;
        qs[h * HD + i1] = o1 * a.q_scale;
      }
    } else {
      // all of a thread's loads first: one memory round trip on the critical
      // path of every piece, not one per element
      constexpr int kPer = (kMaxGroup * HD + kNCT - 1) / kNCT;
      float v[kPer];
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int i = tid + u * kNCT;
        v[u] = i < G * HD ? __ldg(qb + i) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int i = tid + u * kNCT;
        if (i < kMaxGroup * HD) qs[i] = v[u] * a.q_scale;
      }
    }
    consumer_sync(kNCT);
  };

  // ---- split-KV merge ------------------------------------------------------
  // Every piece word is 64 bits: (float bits, call epoch << 32), stored with
  // one single-copy-atomic access, so the merger recognises the current
  // call's words by their epoch and needs no fence between a piece's stores
  // and the segment counter (a relaxed add).  Epochs grow with every call on
  // the workspace, whatever its shape, so a slot word left by any earlier
  // call never carries the current epoch.
  auto tag = [](float v, uint32_t ep) -> uint64_t {
    return (uint64_t)__float_as_uint(v) | ((uint64_t)ep << 32);
  };
  auto fresh = [](uint64_t w, uint32_t ep) { return (uint32_t)(w >> 32) == ep; };
  constexpr int kD4 = HD / 4;  // float4 column chunks of a head row
  // A piece word polled from global memory until it carries epoch ep
  // (bounded: a piece that never arrives latches GLA_ERR_TIMEOUT).
  auto poll_word = [&](const uint64_t* p, uint32_t ep) -> uint64_t {
    unsigned long long t0 = 0;
    for (;;) {
      uint64_t w0, w1;
      ld_relaxed_gpu_u64x2(
          reinterpret_cast<const uint64_t*>(reinterpret_cast<uintptr_t>(p) & ~(uintptr_t)15), w0,
          w1);
      const uint64_t w = (reinterpret_cast<uintptr_t>(p) & 8) ? w1 : w0;
      if (fresh(w, ep) || flags[0]) return w;
      if (t0 == 0) {
        t0 = global_timer_ns();
      } else if (global_timer_ns() - t0 > kWaitTimeoutNs) {
        flags[0] = 1;
        atomicCAS(a.status, 0, GLA_ERR_TIMEOUT);
        return w;
      }
    }
  };
  auto lo_f = [](uint64_t w) { return __uint_as_float((uint32_t)w); };

  // Split-KV merge of segment s.  The last nm = min(G, npieces) CTAs to
  // count are its mergers: merger r (r = 0 the very last) merges q heads r,
  // r + nm, ... so the merge runs on nm SMs at once.  For each of its heads a
  // merger copies that head's row (o, m, l) of every piece into shared memory
  // `buf` (the drained ring, or the warp merge buffer when the ring still
  // holds this CTA's next piece; chunks of whole pieces when they do not
  // fit).  Every warp then turns the pieces' (m, l) into weights e = 2^(m - M)
  // (M the running maximum) and the sum of e l - the same values in every
  // warp, so no barrier sits between weights and sums - and every thread adds
  // e o over its share of the pieces for a pair of columns.  The epochs are
  // checked on the words as they are used; if any word was stale (a piece
  // whose CTA had not stored yet), the chunk is copied again and redone
  // (bounded).
  auto merge_heads = [&](int b, int g, int s, int c0, int npieces, uint32_t ep, int r, int nm,
                         char* buf, int cap_bytes) {
    constexpr int kRowW = HD + 4;       // words of a head row: o[HD], m, l, 2 pad
    constexpr int kRowB = kRowW * 8;
    constexpr int kC16 = kRowB / 16;    // 16-byte chunks of a row
    constexpr int kHalf = HD / 2;       // column pairs
    constexpr int kTPI = kNCT / kHalf;  // threads per column pair (piece split)
    // pieces a lane holds in the weights (a chunk has at most 32 kPL pieces;
    // fewer registers in the two-CTA kernels, whose segments have few pieces)
    constexpr int kPL = LOADER == 0 ? 6 : 2;
    const int piece_words = G * kSH;
    const uint64_t* src0 = a.ws_part + (int64_t)(c0 + s) * piece_words;
    // buf: rows [cap][kRowW] words, then each warp's weights [NW][cap]; the
    // [kTPI][HD] partial sums reuse the rows once the pieces are folded
    // (kTPI * HD * 4 <= 2 KB)
    const int cap = imin(imin(npieces, 32 * kPL), cap_bytes / (kRowB + NW * 4));
    char* rows = buf;
    float* Ew = reinterpret_cast<float*>(buf + (size_t)cap * kRowB) + warp * cap;
    float* part = reinterpret_cast<float*>(buf);
    // early copies that the true length did not need may still be landing in
    // the ring: the producer drains them, and so does the merger before it
    // overwrites the ring
    if (tid == 0 && buf == smem)
      for (int k = my_tiles; k < flags[5]; ++k) mbar_wait(&land[k], 0, flags, a.status);
    const int q = tid % kHalf, j = tid / kHalf;  // column pair, piece share
    const bool active = j < kTPI;
    long long ck[5] = {clock64(), 0, 0, 0, 0};
    int tries = 0;
    for (int h = r; h < G; h += nm) {
      float2 acc = make_float2(0.f, 0.f);
      float Mrun = -INFINITY, Lrun = 0.f;
      for (int p0 = 0; p0 < npieces; p0 += cap) {
        const int n = imin(cap, npieces - p0);
        unsigned long long t0 = 0;
        for (;;) {  // until every word of the chunk carried the epoch
          for (int i = tid; i < n * kC16; i += kNCT) {
            const int p = i / kC16, c = i - p * kC16;
            cp_async_16_plain(rows + (size_t)p * kRowB + c * 16,
                              reinterpret_cast<const char*>(
                                  src0 + ((int64_t)(p0 + p) * G + h) * kSH) + c * 16);
          }
          cp_async_commit_wait_all();
          consumer_sync(kNCT);
          ++tries;
          if (tries == 1) ck[1] = clock64();
          if (p0 == 0 && h == r && tid == 0) stamp(kTrGather);
          // weights, computed by every warp: lane holds pieces lane + 32 k
          bool stale = false;
          float mk[kPL], lk[kPL];
          float mx = -INFINITY;
#pragma unroll
          for (int k = 0; k < kPL; ++k) {
            const int p = lane + 32 * k;
            mk[k] = -INFINITY;
            lk[k] = 0.f;
            if (p < n) {
              const ulonglong2 w = lds_u64x2(smem_u32(rows + (size_t)p * kRowB + HD * 8));
              stale = stale || !fresh(w.x, ep) || !fresh(w.y, ep);
              mk[k] = lo_f(w.x);
              lk[k] = lo_f(w.y);
              mx = fmaxf(mx, mk[k]);
            }
          }
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
          const float Mn = fmaxf(Mrun, mx);
          float ls = 0.f;
#pragma unroll
          for (int k = 0; k < kPL; ++k) {
            const int p = lane + 32 * k;
            if (p < n) {
              const float e = (mk[k] == -INFINITY) ? 0.f : fast_exp2(mk[k] - Mn);
              Ew[p] = e;
              ls = fmaf(e, lk[k], ls);
            }
          }
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
          const float so = (Mrun == -INFINITY) ? 0.f : fast_exp2(Mrun - Mn);
          __syncwarp();
          if (tries == 1) ck[2] = clock64();
          float2 r2 = make_float2(acc.x * so, acc.y * so);
          if (active) {
            const uint32_t col = smem_u32(rows) + (uint32_t)q * 16u;
            const uint32_t eb = smem_u32(Ew);
            int p = j;
            for (; p + 3 * kTPI < n; p += 4 * kTPI) {
              ulonglong2 w[4];
              float e[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) w[u] = lds_u64x2(col + (uint32_t)(p + u * kTPI) * kRowB);
#pragma unroll
              for (int u = 0; u < 4; ++u) e[u] = lds_f32(eb + (uint32_t)(p + u * kTPI) * 4u);
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                stale = stale || !fresh(w[u].x, ep) || !fresh(w[u].y, ep);
                r2.x = fmaf(e[u], lo_f(w[u].x), r2.x);
                r2.y = fmaf(e[u], lo_f(w[u].y), r2.y);
              }
            }
            for (; p < n; p += kTPI) {
              const ulonglong2 w = lds_u64x2(col + (uint32_t)p * kRowB);
              const float e = lds_f32(eb + (uint32_t)p * 4u);
              stale = stale || !fresh(w.x, ep) || !fresh(w.y, ep);
              r2.x = fmaf(e, lo_f(w.x), r2.x);
              r2.y = fmaf(e, lo_f(w.y), r2.y);
            }
          }
          if (tries == 1) ck[3] = clock64();
          // the chunk is read before it is copied again or the next one lands
          const bool any_stale = consumer_sync_or(kNCT, stale);
          if (!any_stale || flags[0]) {
            acc = r2;
            Lrun = Lrun * so + ls;
            Mrun = Mn;
            break;
          }
          if (tid == 0) {
            if (t0 == 0) t0 = global_timer_ns();
            else if (global_timer_ns() - t0 > kWaitTimeoutNs) {
              flags[0] = 1;
              atomicCAS(a.status, 0, GLA_ERR_TIMEOUT);
            }
          }
        }
      }
      if (h == r) {
        ck[4] = clock64();
        if (kTraced && a.trace && tid == 0) {
          auto d16 = [](long long x) { return (uint64_t)(x > 65535 ? 65535 : x); };
          a.trace[(size_t)blockIdx.x * kTraceWords + kTrMergeCycles] =
              d16(ck[1] - ck[0]) | (d16(ck[2] - ck[1]) << 16) | (d16(ck[3] - ck[2]) << 32) |
              (d16(ck[4] - ck[3]) << 48);
          a.trace[(size_t)blockIdx.x * kTraceWords + kTrMergeTries] = (uint64_t)tries;
        }
      }
      // join the kTPI shares of every column pair and write the head
      if (active) *reinterpret_cast<float2*>(part + j * HD + 2 * q) = acc;
      consumer_sync(kNCT);
      if (tid == 0) stamp(kTrFolded);
      if (tid < kHalf) {
        float2 t = make_float2(0.f, 0.f);
#pragma unroll
        for (int u = 0; u < kTPI; ++u) {
          const float2 v = *reinterpret_cast<const float2*>(part + u * HD + 2 * tid);
          t.x += v.x;
          t.y += v.y;
        }
        write_final<HD, XCH>(a, b, g * G + h, 2 * tid, t.x, Mrun, Lrun, (uint32_t)flags[2]);
        write_final<HD, XCH>(a, b, g * G + h, 2 * tid + 1, t.y, Mrun, Lrun, (uint32_t)flags[2]);
      }
      consumer_sync(kNCT);
    }
  };

  // ring_free: no tiles of a later piece of this CTA are in flight or staged.
  auto finish_piece = [&](int b, int g, bool ring_free, bool first) {
    cons.to_merge(a, merge_w, lane);
    if (first && tid == 0) mbar_wait(ep_bar, 0, flags, a.status);  // flags[4]: the call epoch
    consumer_sync(kNCT);
    const int s = b * n_kv + g;
    int32_t c0;
    const int32_t npieces = deal.pieces(seq_start, nunits, b, g, &c0);
    const uint32_t ep = (uint32_t)flags[4];
    // one thread per (head, 4 columns): the warps' (m, l) pairs, then their
    // o chunks, as float2 / float4 shared loads
    for (int idx = tid; idx < G * kD4; idx += kNCT) {
      const int h = idx / kD4, d = (idx - h * kD4) * 4;
      float2 ml[NW];
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        ml[w] = *reinterpret_cast<const float2*>(merge + (w * kMG + h) * kMH + HD);
        M = fmaxf(M, ml[w].x);
      }
      float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
      float L = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const float4 ow = *reinterpret_cast<const float4*>(merge + (w * kMG + h) * kMH + d);
          const float sc = fast_exp2(ml[w].x - M);
          O.x += sc * ow.x; O.y += sc * ow.y; O.z += sc * ow.z; O.w += sc * ow.w;
          L += sc * ml[w].y;
        }
      }
      if (npieces == 1) {
        write_final4<HD, XCH>(a, b, g * G + h, d, O, M, L, (uint32_t)flags[2]);
      } else {
        uint64_t* slot = a.ws_part + ((int64_t)(blockIdx.x + s) * G + h) * kSH;
        st_relaxed_gpu_u64x2(slot + d, tag(O.x, ep), tag(O.y, ep));
        st_relaxed_gpu_u64x2(slot + d + 2, tag(O.z, ep), tag(O.w, ep));
        if (d == 0) st_relaxed_gpu_u64x2(slot + HD, tag(M, ep), tag(L, ep));
      }
    }
    bool merged_here = npieces == 1;  // this CTA writes final records of the segment
    int mr = 0, mn = 1;                 // merger index and mergers of the segment
    if (npieces > 1) {
      consumer_sync(kNCT);
      if (tid == 0) flags[1] = atomic_add_relaxed_gpu(&a.ws_counter[s], 1);
      consumer_sync(kNCT);
      // round robin: the last G to count merge (each CTA holds one piece, so
      // a merger that waits for a later piece holds up no other segment);
      // contiguous deal: only the last, which never waits for a piece (an
      // earlier merger would wait for CTAs still busy with earlier segments)
      mn = deal.mode == 1 ? imin(G, npieces) : 1;
      mr = npieces - 1 - flags[1];  // 0: the last to count
      merged_here = mr < mn;
      if (tid == 0) stamp(kTrCounted);
      if (merged_here) {
        if (ring_free) merge_heads(b, g, s, c0, npieces, ep, mr, mn, smem, a.stages * a.stage_bytes);
        else merge_heads(b, g, s, c0, npieces, ep, mr, mn, reinterpret_cast<char*>(merge), kMergeBytes);
        // every CTA has counted: the last one resets the counter
        if (mr == 0 && tid == 0) st_relaxed_gpu_s32(&a.ws_counter[s], 0);
      }
    } else if (tid == 0) {
      stamp(kTrCounted);
    }
    consumer_sync(kNCT);
    if (merged_here && tid == 0) stamp(kTrMerged);
    if constexpr (XCH) {
      if (merged_here) publish_merge(g, mr, mn);
    }
    if (merged_here && tid == 0) stamp(kTrPublished);
    return merged_here;
  };

  // Piece by piece, tile by tile: the inner loop carries only the ring
  // position and the row cursor, so the consumer keeps its registers.
  int st = 0;
  uint32_t phase = 0;
  auto run_piece = [&](const Piece& pc, int row0, int row_step, bool ring_free,
                       bool first_piece) {
    // kv head pc.g's exchange epoch (read by every CTA holding a piece of it,
    // advanced only by its publisher), loaded alongside q
    epoch_read(pc.g);
    load_q(pc.b, pc.g);
    if (first_piece && tid == 0) stamp(kTrQ);
    cons.begin(a, qs, lane);
    const int np = npos[pc.b];
    const int row_end = row0 + pc.n * row_step;
    for (; row0 < row_end; row0 += row_step) {
      const int rows = imin(unit_rows, np - row0);
      mbar_wait(&full[st], phase, flags, a.status);
      if (kTraced && a.trace && tid == 0 && flags[6] == 0) {
        stamp(kTrFirstTile);
        flags[6] = 1;
      }
      cons.consume(a, smem + (size_t)st * a.stage_bytes, rows, pbuf_w, qs, warp, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (++st == a.stages) {
        st = 0;
        phase ^= 1u;
      }
    }
    if (tid == 0) stamp(kTrLastTile);
    return finish_piece(pc.b, pc.g, ring_free, first_piece);
  };
  bool merger = false;
  if (LOADER == 0 || deal.mode == 1) {  // one piece: kv head g's tiles j, j + S, ...
    Piece pc;
    pc.b = 0;
    pc.g = ct.g;
    pc.u0 = 0;
    pc.n = ct.count;
    merger = run_piece(pc, ct.j * unit_rows, ct.S * unit_rows, true, true);
  } else if constexpr (LOADER == 1) {  // contiguous deal: piece by piece
    TileWalk wk = ct.wk;
    Piece pc;
    bool first = true;
    while (wk.next_piece(nunits, B, n_kv, pc)) {
      merger = run_piece(pc, pc.u0 * unit_rows, unit_rows, wk.p >= wk.end, first) || merger;
      first = false;
    }
  }
  if (kTraced && a.trace && tid == 0) {
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    a.trace[(size_t)blockIdx.x * kTraceWords + kTrInfo] =
        (uint64_t)(uint32_t)my_tiles | ((uint64_t)(flags[5] & 0xff) << 16) |
        ((uint64_t)(merger ? 1 : 0) << 24) | ((uint64_t)smid << 32);
    stamp(kTrExit);
  }
}

}  // namespace gla
