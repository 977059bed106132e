// gla_common.cuh - device helpers shared by the libgpullama_attn kernels:
// mbarrier pipeline primitives with bounded waits, bulk (TMA) copies, and the
// split-KV work partition used identically by kernels and host code.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>

#include "gpullama_attn.h"

#define GLA_HD __host__ __device__ __forceinline__

namespace gla {

// Longest time one bounded device wait may spin before the kernel latches
// GLA_ERR_TIMEOUT into the status word and drains without waiting further.
constexpr unsigned long long kWaitTimeoutNs = 1000000000ull;  // 1 s

// Maximum q heads per KV head (kvMul) handled by one decode CTA.
constexpr int kMaxGroup = 8;

// Maximum batch of the batched decode entry points.
constexpr int kMaxBatch = 1024;

// ---------------------------------------------------------------------------
// Split-KV work partition.
//
// The decode work of a call is the list of units of `unit_rows` rows (the
// decode kernels use whole tiles) ordered by (sequence b, kv head g, unit u):
// segment s = b*n_kv + g holds nunits(b) = ceil(n_pos[b]/unit_rows) units.
// The W units are dealt to P CTAs in contiguous, near-equal ranges (the first
// W%P CTAs get one extra unit), so every CTA streams the same number of KV
// bytes (+- one unit) whatever the sequence lengths.  A CTA walks its range
// in tiles of up to `tile_units` units that never cross a segment boundary.  The intersection of a CTA
// range with a segment is a "piece"; the piece of (CTA c, segment s) owns
// partial slot c + s, which is unique because walking the unit list each new
// piece increments c, s, or both.
// ---------------------------------------------------------------------------
struct Split {
  int32_t q;  // W / P
  int32_t r;  // W % P
};

GLA_HD Split make_split(int32_t W, int32_t P) { return Split{W / P, W % P}; }

GLA_HD int32_t split_lo(Split sp, int32_t c) { return c * sp.q + (c < sp.r ? c : sp.r); }

GLA_HD int32_t split_count(Split sp, int32_t c) { return sp.q + (c < sp.r ? 1 : 0); }

// CTA that owns unit t.
GLA_HD int32_t split_owner(Split sp, int32_t t) {
  int32_t big = sp.r * (sp.q + 1);
  if (t < big) return t / (sp.q + 1);
  return sp.r + (t - big) / sp.q;
}

GLA_HD int32_t ceil_div(int32_t a, int32_t b) { return (a + b - 1) / b; }
GLA_HD int32_t imin(int32_t a, int32_t b) { return a < b ? a : b; }

// One tile of a CTA's walk.
struct Tile {
  int32_t b;      // sequence
  int32_t g;      // kv head
  int32_t row0;   // first row inside the segment
  int32_t units;  // 16-row units (rows may end earlier at the segment's last row)
};

// The units [u0, u0 + n) of segment (b, g) that one CTA holds.
struct Piece {
  int32_t b, g, u0, n;
};

// Walker over a CTA's unit range [p, end) given the per-sequence unit prefix
// seq_start[b] = n_kv * sum_{b'<b} nunits(b') (length n_seq + 1).
struct TileWalk {
  int32_t p, end;
  int32_t b, g, nu;
  int32_t seg_lo, seg_hi;

  GLA_HD void init(const int32_t* seq_start, const int32_t* nunits, int32_t n_seq, int32_t lo,
                   int32_t hi) {
    p = lo;
    end = hi;
    b = g = nu = seg_lo = seg_hi = 0;
    if (lo >= hi) return;
    int32_t l = 0, h = n_seq - 1;
    while (l < h) {  // last b with seq_start[b] <= lo (sequences with no units are skipped)
      const int32_t mid = (l + h + 1) >> 1;
      if (seq_start[mid] <= lo) l = mid; else h = mid - 1;
    }
    while (l < n_seq - 1 && seq_start[l + 1] <= lo) ++l;
    b = l;
    nu = nunits[b];
    g = (lo - seq_start[b]) / nu;
    seg_lo = seq_start[b] + g * nu;
    seg_hi = seg_lo + nu;
  }

  // Next tile of at most tile_units units of unit_rows rows; false when the
  // range is done.
  GLA_HD bool next(const int32_t* nunits, int32_t n_seq, int32_t n_kv, int32_t tile_units,
                   int32_t unit_rows, Tile& t) {
    if (p >= end) return false;
    const int32_t n = imin(tile_units, imin(seg_hi - p, end - p));
    t.b = b;
    t.g = g;
    t.row0 = (p - seg_lo) * unit_rows;
    t.units = n;
    advance(nunits, n_seq, n_kv, n);
    return true;
  }

  // Next piece: the rest of the range inside the current segment.
  GLA_HD bool next_piece(const int32_t* nunits, int32_t n_seq, int32_t n_kv, Piece& pc) {
    if (p >= end) return false;
    const int32_t n = imin(seg_hi - p, end - p);
    pc.b = b;
    pc.g = g;
    pc.u0 = p - seg_lo;
    pc.n = n;
    advance(nunits, n_seq, n_kv, n);
    return true;
  }

  GLA_HD void advance(const int32_t* nunits, int32_t n_seq, int32_t n_kv, int32_t n) {
    p += n;
    if (p == seg_hi && p < end) {  // step to the next segment
      if (++g == n_kv) {
        g = 0;
        do {
          ++b;
        } while (b < n_seq && nunits[b] == 0);
        nu = b < n_seq ? nunits[b] : 1;
      }
      seg_lo = p;
      seg_hi = p + nu;
    }
  }
};

// Number of CTAs holding a piece of segment (b, g); *first_cta the first.
GLA_HD int32_t segment_pieces(Split sp, const int32_t* seq_start, const int32_t* nunits, int32_t b,
                              int32_t g, int32_t* first_cta) {
  const int32_t t0 = seq_start[b] + g * nunits[b];
  const int32_t t1 = t0 + nunits[b] - 1;
  const int32_t c0 = split_owner(sp, t0);
  *first_cta = c0;
  return split_owner(sp, t1) - c0 + 1;
}

// How the W units of a call are dealt to P CTAs.
//  contiguous (mode 0): Split(W, P) over the (b, g, u) order; a CTA range may
//    straddle segments and then holds several pieces.
//  round robin per segment (mode 1; one sequence, n_kv <= P): kv head g gets
//    the S_g CTAs of group g of Split(P, n_kv); CTA j of the group takes the
//    units j, j + S_g, j + 2 S_g, ... of segment g.  No CTA holds more than
//    one piece (a piece boundary inside a CTA's range stalls its consumers
//    for a partial write and counter round trip, and a late CTA becomes its
//    segment's merger), the shares differ by at most one unit, and which
//    units a CTA owns does not depend on the segment's length: the first
//    units of a CTA can be fetched before the length (a position the
//    preceding kernel may still be writing) is known.
// Either way the pieces of a segment are consecutive CTAs, and piece
// (CTA c, segment s) owns partial slot c + s.
struct Deal {
  int32_t mode;
  Split sp;    // mode 0: Split(W, P); mode 1: Split(P, n_kv)
  int32_t nu;  // mode 1: units per segment

  // mode 0: the unit range [lo, lo + cnt) of CTA c in the (b, g, u) order.
  GLA_HD void range(int32_t c, int32_t* lo, int32_t* cnt) const {
    *lo = split_lo(sp, c);
    *cnt = split_count(sp, c);
  }

  // mode 1: CTA c's kv head g, its index j in the group and the group size.
  GLA_HD void group_of(int32_t c, int32_t* g, int32_t* j, int32_t* S) const {
    *g = split_owner(sp, c);
    *j = c - split_lo(sp, *g);
    *S = split_count(sp, *g);
  }

  GLA_HD int32_t pieces(const int32_t* seq_start, const int32_t* nunits, int32_t b, int32_t g,
                        int32_t* first_cta) const {
    if (mode == 0) return segment_pieces(sp, seq_start, nunits, b, g, first_cta);
    *first_cta = split_lo(sp, g);
    return imin(split_count(sp, g), nu);
  }
};

// mode 1: units of a segment of nu units that CTA j of a group of S owns.
GLA_HD int32_t rr_count(int32_t nu, int32_t j, int32_t S) {
  return j < nu ? (nu - 1 - j) / S + 1 : 0;
}

// W = total units, P = CTAs, nu0 = units of sequence 0.  The mode does not
// depend on the lengths, so a kernel picks the same mode before and after it
// knows them.
GLA_HD Deal make_deal(int32_t W, int32_t P, int32_t n_seq, int32_t n_kv, int32_t nu0) {
  Deal d;
  if (n_seq == 1 && n_kv <= P) {
    d.mode = 1;
    d.sp = make_split(P, n_kv);
    d.nu = nu0;
  } else {
    d.mode = 0;
    d.sp = make_split(W, P);
    d.nu = 0;
  }
  return d;
}

// The tiles of one CTA in walk (ring) order: mode 1 round robin over one
// kv head's units (j, j + S, j + 2S, ..., one unit a tile), mode 0 the
// contiguous unit range walked by TileWalk.
struct CtaTiles {
  int32_t mode, g, j, S, k, count;
  TileWalk wk;

  GLA_HD bool next(const int32_t* nunits, int32_t n_seq, int32_t n_kv, int32_t tile_units,
                   int32_t unit_rows, Tile& t) {
    if (mode == 1) {
      if (k >= count) return false;
      t.b = 0;
      t.g = g;
      t.row0 = (j + k * S) * unit_rows;
      t.units = 1;
      ++k;
      return true;
    }
    return wk.next(nunits, n_seq, n_kv, tile_units, unit_rows, t);
  }
};

// CTA c's tiles under `deal` (seq_start / nunits as for TileWalk).
GLA_HD CtaTiles cta_tiles_of(const Deal& deal, int32_t c, const int32_t* seq_start,
                             const int32_t* nunits, int32_t n_seq) {
  CtaTiles ct;
  ct.mode = deal.mode;
  ct.k = 0;
  ct.g = ct.j = ct.count = 0;
  ct.S = 1;
  if (deal.mode == 1) {
    deal.group_of(c, &ct.g, &ct.j, &ct.S);
    ct.count = rr_count(nunits[0], ct.j, ct.S);
  } else {
    int32_t lo, cnt;
    deal.range(c, &lo, &cnt);
    ct.wk.init(seq_start, nunits, n_seq, lo, lo + cnt);
    ct.count = cnt;
  }
  return ct;
}

#ifdef __CUDACC__

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `bar` with the given parity.  Bounded: after
// kWaitTimeoutNs it latches GLA_ERR_TIMEOUT in *status, raises the CTA's
// abort flag and returns false; once the flag is up every later wait returns
// at once, so a failed CTA drains through its remaining barriers and exits.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1;
      atomicCAS(status, 0, GLA_ERR_TIMEOUT);
      return false;
    }
  }
}

// Bulk (non-tensor) TMA copy global -> shared, completing `bytes` of
// transaction count on `bar`.  src/dst 16-byte aligned, bytes % 16 == 0.
// Evict-first L2 hint: the KV stream is read once per call.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// L2 prefetch of `bytes` (a multiple of 16) from a 16-byte aligned address: a
// hint only (L2 is the coherence point), safe while another kernel writes it.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Tiled TMA load of a 2D box at (x, y) of `tmap` (a __grid_constant__ kernel
// parameter) into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tmap, int32_t x,
                                            int32_t y, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 16-byte cp.async (L2 only) global -> shared with an L2 cache hint.
__device__ __forceinline__ void cp_async_16(void* dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)),
               "l"(src), "l"(policy)
               : "memory");
}

// Arrives on `bar` once all earlier cp.async of this thread have landed
// (the arrival is pre-counted in the barrier's expected count).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Named barrier 1 over the consumer threads that also ORs a predicate across
// them: true if any thread passed true.
__device__ __forceinline__ bool consumer_sync_or(int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(nthreads)
      : "memory");
  return r != 0;
}

// Named barrier over the `nthreads` consumer threads (id 1; id 0 is
// __syncthreads).
__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }

__device__ __forceinline__ float2 ld_cg2(const float* p) {
  return __ldcg(reinterpret_cast<const float2*>(p));
}

__device__ __forceinline__ float4 ld_cg4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}

// Relaxed add at GPU scope: the piece counter of a segment.  No ordering is
// needed because every piece word carries the call's epoch (tagged words).
__device__ __forceinline__ int atomic_add_relaxed_gpu(int32_t* p, int v) {
  int old;
  asm volatile("atom.relaxed.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
               : "memory");
  return old;
}

// GPU-scope relaxed accesses of tagged 64-bit words (value bits | epoch << 32);
// an aligned 64-bit access is single-copy atomic, so a word that carries the
// expected epoch carries that call's value.
__device__ __forceinline__ void st_relaxed_gpu_u64x2(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b)
               : "memory");
}
__device__ __forceinline__ void ld_relaxed_gpu_u64x2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p)
               : "memory");
}
__device__ __forceinline__ int32_t ld_relaxed_gpu_s32(const int32_t* p) {
  int32_t v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_gpu_s32(int32_t* p, int32_t v) {
  asm volatile("st.relaxed.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 16-byte cp.async (L2 only) global -> shared without a cache hint: the
// piece words of the split-KV merge, read by the generic proxy like the
// stores that wrote them.
__device__ __forceinline__ void cp_async_16_plain(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
// Shared-memory loads by 32-bit shared address (volatile: kept in order with
// the barriers around them; no memory clobber, so loads of one group issue
// back to back).
__device__ __forceinline__ ulonglong2 lds_u64x2(uint32_t addr) {
  ulonglong2 v;
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// System-scope 64-bit accesses for the peer exchange (another GPU's kernel
// writes or reads the word over NVLink); aligned 64-bit accesses are
// single-copy atomic.
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Two words per access (16-byte aligned): each 64-bit element is still a
// single-copy-atomic access of its own.
__device__ __forceinline__ void st_relaxed_sys_u64x2(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b)
               : "memory");
}
__device__ __forceinline__ void ld_relaxed_sys_u64x2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p)
               : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Programmatic dependent launch: wait for the preceding grid's memory, and
// let the next grid start its prologue early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

// ---- packed FP32 pairs (sm_100 f32x2 instructions) -----------------------
// A pair is a b64 register: element 0 in the low half, element 1 in the high
// half, the same order as two consecutive floats in memory.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

#endif  // __CUDACC__

// Raises the kernel's dynamic shared memory limit to the device's opt-in
// maximum once per (kernel, device): the attribute is per function and
// context, and setting it on every launch cost ~1 us of host time.
template <class Kern>
void ensure_smem_attr(Kern kern, size_t bytes, std::atomic<uint64_t>& done) {
  // done: bit d set once device d has the attribute (devices < 64)
  if (bytes <= 48 * 1024) return;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return;
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           std::max<int>(optin, (int)bytes)) == cudaSuccess && bit)
    done.fetch_or(bit, std::memory_order_acq_rel);
}

}  // namespace gla
