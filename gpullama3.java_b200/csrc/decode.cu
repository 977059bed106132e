// decode.cu - launch planning and template instantiation of the split-KV
// decode kernel (decode_kernel.cuh).
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cmath>
#include <mutex>

#include "decode_kernel.cuh"
#include "gla_internal.h"

namespace gla {

namespace {

constexpr int kTileMax = 64;
static_assert(kTraceWords == kTraceWordsPerCta, "trace layout shared with the context");
static_assert(F32Consumer<128, 1>::kTileMax == kTileMax && F16Consumer<128>::kTileMax == kTileMax &&
                  Q8Consumer<128>::kTileMax == kTileMax,
              "consumers address stages with a compile-time tile height");

// consumer warps: F32Consumer (8), F16Consumer (4), Q8Consumer (8)
int nw_for(int dtype) { return dtype == GLA_DTYPE_F16 ? 4 : 8; }
constexpr int kMaxStages = 8;

size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

// LOADER 0 (tiled TMA) for one sequence whose base pointer the host knows
// and whose kv heads each get their own CTA group (n_kv <= SMs); LOADER 1
// (cp.async) when the per-sequence bases live in device memory, and for one
// sequence with more kv heads than SMs (contiguous deal, base pointer a.k).
int loader_for(const DecodeRequest& r, int sms) {
  return (r.k_ptrs || (r.batch == 1 && r.n_kv > sms)) ? 1 : 0;
}

int esize_for(int dtype) { return dtype == GLA_DTYPE_F32 ? 4 : dtype == GLA_DTYPE_F16 ? 2 : 1; }

// One stage: a K and a V tile, and for a Q8 cache the tile's scale rows.
size_t stage_bytes_for(int dtype, int hd, int tile) {
  return (size_t)2 * tile * hd * esize_for(dtype) +
         (dtype == GLA_DTYPE_Q8 ? (size_t)tile * kQ8ScaleRowBytes : 0);
}

int group_cap_for(int dtype, int group) {
  if (dtype != GLA_DTYPE_F32) return kMaxGroup;
  return group <= 4 ? group : 8;
}

// Shared memory layout for a given tile/stage count.
struct Layout {
  int32_t off_bars, off_seq, off_q, off_pbuf, off_merge, off_flags, off_rope;
  size_t total;
};

Layout layout_for(int dtype, int hd, int group, int tile, int stages, int batch, int grid) {
  Layout L;
  size_t off = (size_t)stages * stage_bytes_for(dtype, hd, tile);
  L.off_bars = (int32_t)align16(off);
  off = L.off_bars + (size_t)(stages * 3 + 1) * sizeof(uint64_t);  // full, empty, land, epoch
  L.off_seq = (int32_t)align16(off);
  off = L.off_seq + (size_t)(3 * batch + 1) * sizeof(int32_t);
  L.off_q = (int32_t)align16(off);
  off = L.off_q + (size_t)kMaxGroup * hd * sizeof(float);
  L.off_pbuf = (int32_t)align16(off);
  const int nw = nw_for(dtype);
  off = L.off_pbuf +
        (dtype != GLA_DTYPE_F32 ? 0 : (size_t)nw * F32Consumer<128, 1>::kPbufFloats * sizeof(float));
  L.off_merge = (int32_t)align16(off);
  off = L.off_merge + (size_t)nw * group_cap_for(dtype, group) * (hd + 4) * sizeof(float);
  L.off_flags = (int32_t)align16(off);
  L.off_rope = (int32_t)align16(L.off_flags + 32);
  (void)grid;
  L.total = L.off_rope + (size_t)(hd / 2) * 8 + 1024;  // + slack to 1024-align the stage ring
  return L;
}

template <int HD, class C, int LOADER, bool XCH>
cudaError_t launch_impl(const DecodeArgs& a, const DecodePlan& p, cudaStream_t st) {
  auto kern = decode_kernel<HD, C, LOADER, XCH>;
  static std::atomic<uint64_t> smem_set{0};  // one per kernel instantiation
  ensure_smem_attr(kern, p.smem, smem_set);
  // programmatic dependent launch: this grid's CTAs may start (prologue
  // only; the kernel waits on griddepcontrol before touching memory) while
  // the previous kernel on the stream drains
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(p.threads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int HD, int LOADER, bool XCH>
cudaError_t launch_f32(const DecodeArgs& a, const DecodePlan& p, cudaStream_t st) {
  switch (group_cap_for(GLA_DTYPE_F32, a.group)) {
    case 1: return launch_impl<HD, F32Consumer<HD, 1>, LOADER, XCH>(a, p, st);
    case 2: return launch_impl<HD, F32Consumer<HD, 2>, LOADER, XCH>(a, p, st);
    case 3: return launch_impl<HD, F32Consumer<HD, 3>, LOADER, XCH>(a, p, st);
    case 4: return launch_impl<HD, F32Consumer<HD, 4>, LOADER, XCH>(a, p, st);
    default: return launch_impl<HD, F32Consumer<HD, 8>, LOADER, XCH>(a, p, st);
  }
}

template <int LOADER, bool XCH>
cudaError_t launch_any(int dtype, int hd, const DecodeArgs& a, const DecodePlan& p,
                       cudaStream_t st) {
  if (dtype == GLA_DTYPE_F32) {
    switch (hd) {
      case 64: return launch_f32<64, LOADER, XCH>(a, p, st);
      case 96: return launch_f32<96, LOADER, XCH>(a, p, st);
      default: return launch_f32<128, LOADER, XCH>(a, p, st);
    }
  }
  if (dtype == GLA_DTYPE_Q8) {  // one sequence, tensor-map loader only (checked by the plan)
    if constexpr (LOADER == 0 && !XCH) {
      return hd == 64 ? launch_impl<64, Q8Consumer<64>, 0, false>(a, p, st)
                      : launch_impl<128, Q8Consumer<128>, 0, false>(a, p, st);
    }
    return cudaErrorInvalidValue;
  }
  switch (hd) {
    case 64: return launch_impl<64, F16Consumer<64>, LOADER, XCH>(a, p, st);
    case 96: return launch_impl<96, F16Consumer<96>, LOADER, XCH>(a, p, st);
    default: return launch_impl<128, F16Consumer<128>, LOADER, XCH>(a, p, st);
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2D map over a cache [rows][kv_stride] with boxes of one column block x tile
// rows, swizzled like TileLayout (128B for 128-byte block rows, 64B for 64).
bool encode_kv_map(CUtensorMap* map, const void* base, int dtype, int hd, int64_t kv_stride,
                   int64_t rows, int tile, std::string* err) {
  auto fn = encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  const int esize = esize_for(dtype);
  const int cw = dtype == GLA_DTYPE_F32 ? 32 : dtype == GLA_DTYPE_Q8 ? hd : (hd % 64 == 0 ? 64 : 32);
  const CUtensorMapSwizzle swz =
      cw * esize == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  cuuint64_t dims[2] = {(cuuint64_t)kv_stride, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(kv_stride * esize)};
  cuuint32_t box[2] = {(cuuint32_t)cw, (cuuint32_t)tile};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype == GLA_DTYPE_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                      : dtype == GLA_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                  2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
    return false;
  }
  return true;
}

// Q8 scales [rows][n_kv * 8] halves, boxes of one kv head's 8 halves x tile rows.
bool encode_scale_map(CUtensorMap* map, const void* base, int n_kv, int64_t rows, int tile,
                      std::string* err) {
  auto fn = encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  cuuint64_t dims[2] = {(cuuint64_t)n_kv * kQ8ScaleHalves, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)n_kv * kQ8ScaleRowBytes};
  cuuint32_t box[2] = {(cuuint32_t)kQ8ScaleHalves, (cuuint32_t)tile};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled (scales) failed (" + std::to_string((int)r) + ")";
    return false;
  }
  return true;
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
  if (r.dtype == GLA_DTYPE_Q8 &&
      (!(hd == 64 || hd == 128) || r.k_ptrs || r.record_mode == 2 || r.rope || !r.scales)) {
    *err = "Q8 cache: one sequence, head_dim 64 or 128";
    return GLA_ERR_NOT_SUPPORTED;
  }
  // the tensor-map loader (fused RoPE, Q8 caches, the peer exchange) gives
  // every kv head its own CTA group
  if ((r.rope || r.dtype == GLA_DTYPE_Q8 || r.record_mode == 2) && r.n_kv > dev.sms) {
    *err = "fused RoPE, Q8 caches and the peer exchange need n_kv_heads <= the SM count";
    return GLA_ERR_NOT_SUPPORTED;
  }
  // Work is streamed and dealt to CTAs in whole tiles of kTileMax rows.
  // (16-row units, balanced to +-16 rows per CTA, measured slower on B200
  // for every decode shape tried, 512 to 128K rows: the extra pieces and
  // ragged boxes cost more than the imbalance of one tile.)
  const int64_t rows = std::max<int64_t>(1, r.max_n_pos);
  const int tile = kTileMax;
  const int64_t W = (int64_t)r.batch * r.n_kv * ((rows + tile - 1) / tile);
  if (W > (int64_t)1 << 30) {
    *err = "decode work too large for one call";
    return GLA_ERR_NOT_SUPPORTED;
  }
  // The FP16 consumer with the cp.async loader (batches) runs two CTAs an SM
  // (F16Consumer::kCtasPerSm), each with half an SM's shared memory.
  const int per_sm = (r.dtype == GLA_DTYPE_F16 && loader_for(r, dev.sms) == 1 && r.record_mode != 2 &&
                      dev.smem_per_sm > 0)
                         ? 2
                         : 1;
  const size_t smem_cap =
      per_sm == 1 ? (size_t)dev.smem_optin
                  : std::min<size_t>(dev.smem_optin, (size_t)dev.smem_per_sm / 2 - 1024);
  // Every CTA participates when n_pos is only known on the device.
  int grid = dev.sms * per_sm;
  if (r.n_pos_dev == nullptr) grid = (int)std::min<int64_t>(grid, W);
  grid = std::max(grid, 1);
  // the tensor-map loader's round-robin deal gives every kv head a CTA group
  if (loader_for(r, dev.sms) == 0) grid = std::max(grid, r.n_kv);
  // Stages: as many as fit (the ring is the only large smem consumer).
  int stages = kMaxStages;
  Layout L = layout_for(r.dtype, hd, group, tile, stages, r.batch, grid);
  while (stages > 2 && L.total > smem_cap) {
    --stages;
    L = layout_for(r.dtype, hd, group, tile, stages, r.batch, grid);
  }
  if (L.total > smem_cap) {
    *err = "shared memory layout does not fit";
    return GLA_ERR_NOT_SUPPORTED;
  }
  p->loader = loader_for(r, dev.sms);
  p->tile = tile;
  p->stages = stages;
  p->grid = grid;
  p->threads = (nw_for(r.dtype) + 1) * 32;
  p->smem = L.total;
  p->part_words = (size_t)(grid + r.batch * r.n_kv) * group * (hd + 4);
  p->counters = (size_t)r.batch * r.n_kv;
  return GLA_OK;
}

int launch_decode(const DecodeRequest& r, const DecodePlan& p, const DecodeWorkspace& ws,
                  cudaStream_t stream, std::string* err) {
  const int hd = r.head_dim;
  const int group = r.n_heads / r.n_kv;
  const int loader = p.loader;
  Layout L = layout_for(r.dtype, hd, group, p.tile, p.stages, r.batch, p.grid);
  DecodeArgs a{};
  if (loader == 0) {
    if (!encode_kv_map(&a.tmap_k, r.k, r.dtype, hd, r.kv_stride, r.n_pos_cap, p.tile, err) ||
        !encode_kv_map(&a.tmap_v, r.v, r.dtype, hd, r.kv_stride, r.n_pos_cap, p.tile, err))
      return GLA_ERR_INVALID_ARG;
    if (r.dtype == GLA_DTYPE_Q8 &&
        !encode_scale_map(&a.tmap_s, r.scales, r.n_kv, r.n_pos_cap, p.tile, err))
      return GLA_ERR_INVALID_ARG;
  }
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
  a.early_kv = r.early_kv;
  a.batch = r.batch;
  a.n_heads = r.n_heads;
  a.n_kv = r.n_kv;
  a.group = group;
  a.tile = p.tile;
  a.stages = p.stages;
  a.q_scale = r.scale * 1.4426950408889634f;
  a.out = r.out;
  a.record_mode = r.record_mode;
  a.xch_bases = r.xch_bases;
  a.xch_local = r.xch_local;
  a.xch_out = r.xch_out;
  a.xch_world = r.xch_world;
  a.xch_rank = r.xch_rank;
  a.ws_part = ws.part;
  a.ws_counter = ws.counter;
  a.ws_epoch = ws.epoch;
  a.status = ws.status;
  a.trace = ws.trace;
  a.scales = r.scales;
  a.stage_bytes = (int32_t)stage_bytes_for(r.dtype, hd, p.tile);
  a.off_bars = L.off_bars;
  a.off_seq = L.off_seq;
  a.off_pbuf = L.off_pbuf;
  a.off_q = L.off_q;
  a.off_merge = L.off_merge;
  a.off_flags = L.off_flags;
  a.off_rope = L.off_rope;
  a.rope = r.rope;
  a.rope_style = r.rope_style;
  a.rope_theta = r.rope_theta;
  a.rope_k = r.rope_k;
  a.rope_v = r.rope_v;
  // the peer exchange (record mode 2: one sequence, tensor-map loader) is a
  // separate instantiation, so the other kernels carry none of its registers
  cudaError_t rc = r.record_mode == 2 && loader == 0 ? launch_any<0, true>(r.dtype, hd, a, p, stream)
                   : loader == 0                     ? launch_any<0, false>(r.dtype, hd, a, p, stream)
                                                     : launch_any<1, false>(r.dtype, hd, a, p, stream);
  if (rc != cudaSuccess) {
    *err = std::string("decode launch failed: ") + cudaGetErrorString(rc);
    return GLA_ERR_CUDA;
  }
  return GLA_OK;
}

}  // namespace gla
