// decode.cu - launch planning and template instantiation of the split-KV
// decode kernel (decode_kernel.cuh).
#include <algorithm>
#include <cmath>
#include <mutex>

#include "decode_kernel.cuh"
#include "gla_internal.h"

namespace gla {

namespace {

constexpr int kNWf32 = 8;  // consumer warps, FP32 cache
constexpr int kNWf16 = 4;  // consumer warps, FP16 cache
constexpr int kMaxStages = 8;

size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

int tile_max_for(int dtype, int hd) {
  if (dtype == GLA_DTYPE_F16) return 16 * kNWf16;
  return hd <= 64 ? 64 : 32;
}

int row_bytes_for(int dtype, int hd) { return dtype == GLA_DTYPE_F16 ? (hd + 8) * 2 : hd * 4; }

int group_cap_for(int dtype, int group) {
  if (dtype == GLA_DTYPE_F16) return kMaxGroup;
  return group <= 1 ? 1 : group <= 2 ? 2 : group <= 4 ? 4 : 8;
}

// Shared memory layout for a given tile/stage count.
struct Layout {
  int32_t off_bars, off_seq, off_pbuf, off_merge, off_flags;
  size_t total;
};

Layout layout_for(int dtype, int hd, int group, int tile, int stages, int batch) {
  const int nw = dtype == GLA_DTYPE_F16 ? kNWf16 : kNWf32;
  Layout L;
  size_t off = (size_t)stages * 2 * tile * row_bytes_for(dtype, hd);
  L.off_bars = (int32_t)align16(off);
  off = L.off_bars + (size_t)stages * 2 * sizeof(uint64_t);
  L.off_seq = (int32_t)align16(off);
  off = L.off_seq + (size_t)(3 * batch + 1) * sizeof(int32_t);
  L.off_pbuf = (int32_t)align16(off);
  off = L.off_pbuf + (dtype == GLA_DTYPE_F16 ? 0 : (size_t)nw * 64 * sizeof(float));
  L.off_merge = (int32_t)align16(off);
  off = L.off_merge + (size_t)nw * group_cap_for(dtype, group) * (hd + 2) * sizeof(float);
  L.off_flags = (int32_t)align16(off);
  L.total = L.off_flags + 16;
  return L;
}

template <class Kern>
void ensure_smem_attr(Kern kern, size_t bytes) {
  // cudaFuncSetAttribute is per device; setting it on every launch is cheap
  // compared with a failed launch, but skip it below the default 48 KB.
  if (bytes > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <int HD, int NW, class C>
cudaError_t launch_impl(const DecodeArgs& a, const DecodePlan& p, cudaStream_t st) {
  auto kern = decode_kernel<HD, NW, C>;
  ensure_smem_attr(kern, p.smem);
  kern<<<p.grid, p.threads, p.smem, st>>>(a);
  return cudaGetLastError();
}

template <int HD>
cudaError_t launch_f32(const DecodeArgs& a, const DecodePlan& p, cudaStream_t st) {
  const int gc = group_cap_for(GLA_DTYPE_F32, a.group);
  switch (gc) {
    case 1: return launch_impl<HD, kNWf32, F32Consumer<HD, 1, kNWf32>>(a, p, st);
    case 2: return launch_impl<HD, kNWf32, F32Consumer<HD, 2, kNWf32>>(a, p, st);
    case 4: return launch_impl<HD, kNWf32, F32Consumer<HD, 4, kNWf32>>(a, p, st);
    default: return launch_impl<HD, kNWf32, F32Consumer<HD, 8, kNWf32>>(a, p, st);
  }
}

}  // namespace

int plan_decode(const DecodeRequest& r, const DeviceInfo& dev, DecodePlan* p, std::string* err) {
  const int hd = r.head_dim;
  if (!(hd == 64 || hd == 96 || hd == 128)) {
    *err = "head_dim must be 64, 96 or 128";
    return GLA_ERR_NOT_SUPPORTED;
  }
  const int group = r.n_heads / r.n_kv;
  if (group > kMaxGroup) {
    *err = "n_heads / n_kv_heads must be <= 8";
    return GLA_ERR_NOT_SUPPORTED;
  }
  if (r.batch < 1 || r.batch > kMaxBatch) {
    *err = "batch must be in [1, 1024]";
    return GLA_ERR_NOT_SUPPORTED;
  }
  // Tile: largest tile that still gives every SM at least two tiles.
  const int64_t rows = std::max<int64_t>(1, r.max_n_pos);
  int tile = tile_max_for(r.dtype, hd);
  auto tiles_at = [&](int t) { return (int64_t)r.batch * r.n_kv * ((rows + t - 1) / t); };
  while (tile > 16 && tiles_at(tile) < 2 * (int64_t)dev.sms) tile >>= 1;
  const int64_t W = tiles_at(tile);
  if (W > (int64_t)1 << 30) {
    *err = "decode work too large for one call";
    return GLA_ERR_NOT_SUPPORTED;
  }
  // Every CTA participates when n_pos is only known on the device.
  int grid = dev.sms;
  if (r.n_pos_dev == nullptr) grid = (int)std::min<int64_t>(dev.sms, W);
  grid = std::max(grid, 1);
  // Stages: as many as fit (the ring is the only large smem consumer).
  int stages = kMaxStages;
  Layout L = layout_for(r.dtype, hd, group, tile, stages, r.batch);
  while (stages > 2 && L.total > (size_t)dev.smem_optin) {
    --stages;
    L = layout_for(r.dtype, hd, group, tile, stages, r.batch);
  }
  if (L.total > (size_t)dev.smem_optin) {
    *err = "shared memory layout does not fit";
    return GLA_ERR_NOT_SUPPORTED;
  }
  p->tile = tile;
  p->stages = stages;
  p->grid = grid;
  p->threads = ((r.dtype == GLA_DTYPE_F16 ? kNWf16 : kNWf32) + 1) * 32;
  p->smem = L.total;
  p->part_floats = (size_t)(grid + r.batch * r.n_kv) * group * (hd + 2);
  p->counters = (size_t)r.batch * r.n_kv;
  return GLA_OK;
}

int launch_decode(const DecodeRequest& r, const DecodePlan& p, float* ws_part, int32_t* ws_counter,
                  int32_t* status, cudaStream_t stream, std::string* err) {
  const int hd = r.head_dim;
  const int group = r.n_heads / r.n_kv;
  Layout L = layout_for(r.dtype, hd, group, p.tile, p.stages, r.batch);
  DecodeArgs a{};
  a.q = r.q;
  a.k = r.k;
  a.v = r.v;
  a.k_ptrs = r.k_ptrs;
  a.v_ptrs = r.v_ptrs;
  a.kv_stride = r.kv_stride;
  a.n_pos_dev = r.n_pos_dev;
  a.n_pos = r.n_pos;
  a.n_pos_add = r.n_pos_add;
  a.n_pos_cap = r.n_pos_cap;
  a.batch = r.batch;
  a.n_heads = r.n_heads;
  a.n_kv = r.n_kv;
  a.group = group;
  a.tile = p.tile;
  a.stages = p.stages;
  a.q_scale = r.scale * 1.4426950408889634f;
  a.out = r.out;
  a.record_mode = r.record_mode;
  a.ws_part = ws_part;
  a.ws_counter = ws_counter;
  a.status = status;
  a.row_bytes = row_bytes_for(r.dtype, hd);
  a.stage_bytes = 2 * p.tile * a.row_bytes;
  a.off_bars = L.off_bars;
  a.off_seq = L.off_seq;
  a.off_pbuf = L.off_pbuf;
  a.off_merge = L.off_merge;
  a.off_flags = L.off_flags;
  cudaError_t rc;
  if (r.dtype == GLA_DTYPE_F32) {
    switch (hd) {
      case 64: rc = launch_f32<64>(a, p, stream); break;
      case 96: rc = launch_f32<96>(a, p, stream); break;
      default: rc = launch_f32<128>(a, p, stream); break;
    }
  } else {
    switch (hd) {
      case 64: rc = launch_impl<64, kNWf16, F16Consumer<64, kNWf16>>(a, p, stream); break;
      case 96: rc = launch_impl<96, kNWf16, F16Consumer<96, kNWf16>>(a, p, stream); break;
      default: rc = launch_impl<128, kNWf16, F16Consumer<128, kNWf16>>(a, p, stream); break;
    }
  }
  if (rc != cudaSuccess) {
    *err = std::string("decode launch failed: ") + cudaGetErrorString(rc);
    return GLA_ERR_CUDA;
  }
  return GLA_OK;
}

}  // namespace gla
