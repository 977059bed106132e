// gla_xch.h - layout of the peer exchange buffer of KV-sequence-sharded
// decode (one per rank, mapped into every other rank with CUDA IPC).
//
// Each rank publishes its shard's per-head records (o normalised, m in
// natural-log units, l, 2 pad: [n_heads][head_dim + 4] floats, 16-byte rows)
// into slot [parity][own rank] of EVERY rank's buffer
// with plain peer stores, then raises flag [parity][own rank][kv head] on
// every rank.  A rank merges kv head g once the flags of all ranks for g
// carry the call's epoch.  Two parities: a rank can run at most one call
// ahead of another (it waits for everybody's records of the current call),
// so a slot is never overwritten while it is read.
//
//   records  [2][kXchMaxWorld][kXchRecFloats]   float
//   flags    [2][kXchMaxWorld][kXchMaxSeg]      uint32 (epoch of the write)
//   epochs   [kXchMaxSeg] uint32: calls completed for kv head g on this rank,
//            read and advanced only by the CTA that publishes g (one per call)
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __CUDACC__
#define GLA_XCH_HD __host__ __device__ __forceinline__
#else
#define GLA_XCH_HD inline
#endif

namespace gla {

constexpr int kXchMaxWorld = 8;
constexpr int kXchRecFloats = 128 * (128 + 4);  // up to 128 heads of head_dim 128
constexpr int kXchMaxSeg = 128;                 // kv heads of one call

GLA_XCH_HD size_t xch_rec_offset(int parity, int src) {  // bytes
  return ((size_t)parity * kXchMaxWorld + src) * kXchRecFloats * sizeof(float);
}
GLA_XCH_HD size_t xch_flags_base() {
  return (size_t)2 * kXchMaxWorld * kXchRecFloats * sizeof(float);
}
GLA_XCH_HD size_t xch_flag_offset(int parity, int src, int seg) {
  return xch_flags_base() + (((size_t)parity * kXchMaxWorld + src) * kXchMaxSeg + seg) * 4;
}
GLA_XCH_HD size_t xch_epoch_offset(int seg) {
  return xch_flags_base() + (size_t)2 * kXchMaxWorld * kXchMaxSeg * 4 + (size_t)seg * 4;
}
GLA_XCH_HD size_t xch_bytes() { return xch_epoch_offset(kXchMaxSeg); }

}  // namespace gla
