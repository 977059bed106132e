// gla_common.cuh - device helpers shared by the libgpullama_attn kernels:
// mbarrier pipeline primitives with bounded waits, bulk (TMA) copies, and the
// split-KV work partition used identically by kernels and host code.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

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
// The decode work of a call is the list of tiles ordered by
// (sequence b, kv head g, tile j): segment s = b*n_kv + g holds
// ntiles(b) = ceil(n_pos[b]/tile) tiles.  The W tiles are dealt to P CTAs in
// contiguous, near-equal ranges (the first W%P CTAs get one extra), so every
// CTA streams the same number of KV bytes (+-1 tile) whatever the sequence
// lengths.  The intersection of a CTA range with a segment is a "piece"; the
// piece of (CTA c, segment s) owns partial slot c + s, which is unique because
// walking the tile list each new piece increments c, s, or both.
// ---------------------------------------------------------------------------
struct Split {
  int32_t q;  // W / P
  int32_t r;  // W % P
};

GLA_HD Split make_split(int32_t W, int32_t P) { return Split{W / P, W % P}; }

GLA_HD int32_t split_lo(Split sp, int32_t c) { return c * sp.q + (c < sp.r ? c : sp.r); }

GLA_HD int32_t split_count(Split sp, int32_t c) { return sp.q + (c < sp.r ? 1 : 0); }

// CTA that owns tile t.
GLA_HD int32_t split_owner(Split sp, int32_t t) {
  int32_t big = sp.r * (sp.q + 1);
  if (t < big) return t / (sp.q + 1);
  return sp.r + (t - big) / sp.q;
}

GLA_HD int32_t ceil_div(int32_t a, int32_t b) { return (a + b - 1) / b; }

// Position of a tile inside the work list.
struct TileRef {
  int32_t b;    // sequence
  int32_t g;    // kv head
  int32_t j;    // tile index inside the segment
  int32_t nt;   // tiles of this sequence's segments
};

// Locates global tile t given the per-sequence tile prefix
// seq_start[b] = n_kv * sum_{b'<b} ntiles(b') (length n_seq + 1).
GLA_HD TileRef locate_tile(const int32_t* seq_start, const int32_t* ntiles, int32_t n_seq,
                           int32_t n_kv, int32_t t) {
  int32_t lo = 0, hi = n_seq - 1;
  while (lo < hi) {  // last b with seq_start[b] <= t (sequences with 0 tiles are skipped)
    int32_t mid = (lo + hi + 1) >> 1;
    if (seq_start[mid] <= t) lo = mid; else hi = mid - 1;
  }
  while (lo < n_seq - 1 && seq_start[lo + 1] <= t) ++lo;
  TileRef r;
  r.b = lo;
  r.nt = ntiles[lo];
  int32_t off = t - seq_start[lo];
  r.g = off / r.nt;
  r.j = off - r.g * r.nt;
  (void)n_kv;
  return r;
}

// Advances a TileRef to the next tile of the work list.
GLA_HD void next_tile(TileRef& r, const int32_t* ntiles, int32_t n_seq, int32_t n_kv) {
  if (++r.j < r.nt) return;
  r.j = 0;
  if (++r.g < n_kv) return;
  r.g = 0;
  do {
    ++r.b;
  } while (r.b < n_seq && ntiles[r.b] == 0);
  if (r.b < n_seq) r.nt = ntiles[r.b];
}

// Number of CTAs holding a piece of segment (b, g).
GLA_HD int32_t segment_pieces(Split sp, const int32_t* seq_start, const int32_t* ntiles,
                              int32_t b, int32_t g, int32_t* first_cta) {
  int32_t t0 = seq_start[b] + g * ntiles[b];
  int32_t t1 = t0 + ntiles[b] - 1;
  int32_t c0 = split_owner(sp, t0);
  *first_cta = c0;
  return split_owner(sp, t1) - c0 + 1;
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

// Named barrier over the `nthreads` consumer threads (id 1; id 0 is
// __syncthreads).
__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }

__device__ __forceinline__ float4 ld_cg4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}

// Release/acquire add at GPU scope (one thread, after a CTA barrier: the
// release covers every write the CTA made before the barrier).
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int32_t* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
               : "memory");
  return old;
}

// Programmatic dependent launch: wait for the preceding grid's memory, and
// let the next grid start its prologue early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

#endif  // __CUDACC__

}  // namespace gla
