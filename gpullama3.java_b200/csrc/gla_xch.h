// gla_xch.h - layout of the peer exchange buffer of KV-sequence-sharded
// decode (one per rank, mapped into every other rank with CUDA IPC).
//
// Each rank publishes its shard's per-head records (o normalised, m in
// natural-log units, l: [n_heads][head_dim + 4] words, 2 pad words) into slot
// [parity][own rank] of EVERY rank's buffer with plain peer stores.  Every
// record word is 64 bits, (float bits, epoch of the call) written by one
// single-copy-atomic store, so a reader polls the words themselves until
// they carry the call's epoch: no flag, no fence (the low-latency protocol
// of packing data and flag into one atomic word).  Two parities: a rank can
// run at most one call ahead of another (it needs everybody's records of the
// current call to finish it), so a slot is never overwritten while it is
// read.
//
//   records  [2][kXchMaxWorld][kXchRecWords]   uint64
//   epochs   [kXchMaxSeg] uint32: calls completed for kv head g on this rank,
//            read by every CTA holding a piece of g and advanced once a call
//            by g's merger 0 (the last of g's mergers to count; each merger
//            publishes its own q heads of g)
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
constexpr int kXchRecWords = 128 * (128 + 4);  // up to 128 heads of head_dim 128
constexpr int kXchMaxSeg = 128;                // kv heads of one call

GLA_XCH_HD size_t xch_rec_offset(int parity, int src) {  // bytes
  return ((size_t)parity * kXchMaxWorld + src) * kXchRecWords * sizeof(uint64_t);
}
GLA_XCH_HD size_t xch_epoch_offset(int seg) {
  return (size_t)2 * kXchMaxWorld * kXchRecWords * sizeof(uint64_t) + (size_t)seg * 4;
}
GLA_XCH_HD size_t xch_bytes() { return xch_epoch_offset(kXchMaxSeg); }

}  // namespace gla
