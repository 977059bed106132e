// prefill.cu - causal prefill attention on tcgen05 tensor cores with TMEM
// accumulators (sm_100a).
//
// out[p][h] = softmax_{t <= p}(scale * q[p][h] . k[t][g]) . v[t][g], g = h / kvMul,
// for a whole prompt at once: what the reference computes one position at a
// time while it ingests a prompt (InferenceEngine.java:88-99, one
// InferenceCore.forwardJava attention block per position).
//
// One CTA per (head, block of NT 128-row query tiles), heaviest blocks first
// (NT = 2 for head_dim 64/96, 1 for 128); 4 NT + 2 warps:
//   warp 4NT   producer: TMA loads of the NT Q tiles once, then K and V
//              blocks of 128 keys into two separate rings (SWIZZLE_64B,
//              32-half column blocks): K_j is released as soon as every S of
//              block j is computed, V_j after the P V products, so the next
//              K tiles stream in while softmax runs.
//   warp 4NT+1 MMA issuer (one thread): per query tile t, S_t = Q_t K_j^T
//              into TMEM columns [256t, 256t+128), then O_t += P_t V_j into
//              columns [256t+128, 256t+128+hd); the tiles alternate, so one
//              tile's MMAs run while the other tile's softmax works;
//              tcgen05.commit signals mbarriers.
//   warps 4t..4t+3, softmax of query tile t: thread r owns query row r,
//              reads its 128 scores with tcgen05.ld in two 64-column passes,
//              keeps the row max/sum in registers (no shuffles), writes P
//              (FP16) to a swizzled shared-memory buffer for the second MMA,
//              and rescales O in TMEM only when the row max grows by more
//              than 2^8 (otherwise p <= 2^8 stays exact in FP16 and the final
//              division by l absorbs the stale max).
// FP32 softmax and accumulation; FP16 inputs; FP32 output.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>

#include "gla_common.cuh"
#include "gla_internal.h"

namespace gla {

namespace {

constexpr int kBM = 128;       // query rows per CTA
constexpr int kBN = 128;       // keys per block
constexpr float kRescaleLog2 = 8.0f;
// Pairs of every 4 (per 8 keys) whose exponentials use the FMA-pipe
// polynomial instead of MUFU.  Measured on B200 (config 5, before the
// softmax ping-pong): 0 of 4 655 TFLOP/s, 1 of 4 678, 2 of 4 622, 3 of 4
// 568 - the polynomial costs about as many issue slots as it frees on MUFU.
constexpr int kPolyPairs = 0;

struct PrefillArgs {
  CUtensorMap tq;  // [L][n_heads*hd]           box (32, 128), SWIZZLE_64B
  CUtensorMap tk;  // [q_off+L][n_kv*hd], rows kv_stride apart; box (32, 128)
  CUtensorMap tv;
  float* out;      // [L][n_heads*hd] FP32
  int32_t L;       // query rows
  int32_t q_off;   // position of query row 0: row i attends keys 0..q_off+i
  int32_t n_heads;
  int32_t kv_mul;
  int32_t n_qblocks;
  float scale_log2;
  int32_t* status;
};

// ---- tcgen05 / TMEM wrappers ----------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// The issuing helpers below are executed by a whole converged warp: the
// operands are computed by every lane, so they stay warp-uniform (the tensor
// core takes them from uniform registers), and `elect.sync` picks the one
// lane that issues.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 lanes x 32 columns of 32-bit: thread i of the warp gets lane (warp%4)*32+i.
// The wait sits in the same asm statement so no use of the registers can be
// scheduled before the load has landed.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// A whole 128-column row (thread = lane) in one load + wait.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float (&v)[128]) {
  uint32_t r[128];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}

// Half a row (64 columns) in one load + wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}


// 2^x for a pair on the FMA pipe (takes load off the MUFU unit, which the
// softmax otherwise saturates).  Cody-Waite split x = n + f with n the
// nearest integer (the 1.5*2^23 shifter leaves n in the low mantissa bits)
// and f in [-1/2, 1/2]; 2^f from a degree-4 polynomial fitted to 2^f at
// Chebyshev nodes by iteratively reweighted least squares (max relative
// error 2.7e-6 in FP32, below FP16 rounding of P); n is added to the
// exponent field as an integer.  Inputs are clamped to >= -126, so a masked
// score (-inf) gives ~1e-38 instead of 0, which FP16 P rounds to 0.
constexpr float kE2C0 = 0x1.ffffe8p-1f, kE2C1 = 0x1.62e0dcp-1f, kE2C2 = 0x1.ec06dap-3f,
                kE2C3 = 0x1.ca1440p-5f, kE2C4 = 0x1.3997d4p-7f;
__device__ __forceinline__ void exp2_poly_pair(float x0, float x1, float& y0, float& y1) {
  const float kShift = 12582912.0f;  // 1.5 * 2^23
  const uint64_t X = pk2(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t T = add2(X, pk2(kShift, kShift));
  const uint64_t N = add2(T, pk2(-kShift, -kShift));
  const uint64_t F = fma2(N, pk2(-1.f, -1.f), X);
  uint64_t P = fma2(pk2(kE2C4, kE2C4), F, pk2(kE2C3, kE2C3));
  P = fma2(P, F, pk2(kE2C2, kE2C2));
  P = fma2(P, F, pk2(kE2C1, kE2C1));
  P = fma2(P, F, pk2(kE2C0, kE2C0));
  float p0, p1, t0, t1;
  upk2(P, p0, p1);
  upk2(T, t0, t1);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

// 2^x on the MUFU unit (flush-to-zero: subnormal probabilities become 0).
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, SWIZZLE_64B (layout type 4), version 1.
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t saddr, uint32_t lbo_bytes,
                                                   uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (Blackwell)
  d |= (uint64_t)4 << 61;  // SWIZZLE_64B
  return d;
}

// Instruction descriptor for kind::f16: F16 x F16 -> F32, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool b_mn_major) {
  return (1u << 4)                          // D format F32
         | (0u << 7) | (0u << 10)           // A, B format F16
         | (0u << 15)                       // A K-major
         | ((b_mn_major ? 1u : 0u) << 16)   // B major
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// Byte offset, inside a [blocks][rows][32 halves] SWIZZLE_64B tile, of the
// 16-byte chunk `c` (0..3) of `row` in column block `cb`.
__device__ __forceinline__ uint32_t sw64_off(int rows, int cb, int row, int c) {
  return (uint32_t)(cb * rows * 64 + row * 64 + ((c ^ ((row >> 1) & 3)) << 4));
}

// Packed FP16 pairs into 32 TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// D (TMEM) [+]= A (TMEM, FP16 pairs per 32-bit column) x B (shared memory);
// issued like tc_mma_f16 by one elected lane of a converged warp.
__device__ __forceinline__ void tc_mma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Named barriers (ids 1 and 2) over the two softmax warpgroups (256 threads).
__device__ __forceinline__ void named_sync(int id) {
  asm volatile("bar.sync %0, 256;" ::"r"(id) : "memory");
}
__device__ __forceinline__ void named_arrive(int id) {
  asm volatile("bar.arrive %0, 256;" ::"r"(id) : "memory");
}

// Register split of the warpgroups (setmaxnreg): the block launches with
// kLaunchRegs a thread; the producer/MMA warpgroup gives back to kLowRegs,
// the two softmax warpgroups take kHighRegs (2 * 128 * kHighRegs + 128 *
// kLowRegs <= 384 * kLaunchRegs, the registers the block was launched with).
// 72/208 is the split at which neither side spills for any head size (at
// 40 registers the MMA issue loop spilled to local memory).
constexpr int kLaunchRegs = 168, kLowRegs = 72, kHighRegs = 208;
static_assert(2 * 128 * kHighRegs + 128 * kLowRegs <= 384 * kLaunchRegs, "register split");
__device__ __forceinline__ void regs_low() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kLowRegs));
}
__device__ __forceinline__ void regs_high() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kHighRegs));
}

template <int HD, int NT>
struct PrefillSmem {
  static_assert(NT == 2, "two query tiles per CTA: two softmax warpgroups");
  static constexpr int kCB = HD / 32;                  // 32-half column blocks
  static constexpr int kQBytes = kBM * HD * 2;         // one Q tile
  static constexpr int kKVBytes = kBN * HD * 2;        // one K or V block
  // ring depths: as deep as 227 KB allow (HD 96: 48 + 4 * 24 + 3 * 24 KB)
  static constexpr int kKS = HD <= 96 ? 4 : 2;         // K ring depth
  static constexpr int kVS = HD <= 64 ? 4 : HD <= 96 ? 3 : 2;  // V ring depth
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + NT * kQBytes;
  static constexpr int kOffV = kOffK + kKS * kKVBytes;
  static constexpr int kOffBar = kOffV + kVS * kKVBytes;
  // barriers: q_full, k_full[KS], k_empty[KS], v_full[VS], v_empty[VS],
  // per tile s_full and p_full; mma_done
  static constexpr int kNumBars = 1 + 2 * kKS + 2 * kVS + 2 * NT + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 32;
  static constexpr int kThreads = (NT + 1) * 128;  // softmax warpgroups + producer/MMA warpgroup
};

// NT = 2 query tiles of 128 rows per CTA share every K/V block.  Tile t owns
// TMEM columns [256t, 256t + 256): S (128 columns; P, as FP16 pairs, is
// written over its first 64 once the scores are read) and O (next HD
// columns).  Per 128-key block j of tile t the MMA warp issues, once the
// softmax has written P_t(j): O_t += P_t(j) V_j (A from TMEM), then
// S_t(j+1) = Q_t K_{j+1}^T over the same columns (the tensor core runs them
// in order, so P is read before it is overwritten), and one commit that
// hands S_t(j+1) - and the finished P V - to the softmax.  While one tile's
// softmax works, the tensor core runs the other tile's products.
// Warps: 0-3 softmax of tile 0, 4-7 of tile 1, 8 Q and K loads, 9 MMA
// issue, 10 V loads, 11 idle (setmaxnreg works on whole warpgroups).
template <int HD, int NT>
__global__ void __launch_bounds__(PrefillSmem<HD, NT>::kThreads, 1)
    prefill_kernel(const __grid_constant__ PrefillArgs a) {
  using SM = PrefillSmem<HD, NT>;

  constexpr int KS = SM::kKS, VS = SM::kVS;
  extern __shared__ __align__(1024) char smem_raw[];
  char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // heaviest (longest causal range) query blocks first
  const int qb = a.n_qblocks - 1 - (int)(blockIdx.x / a.n_heads);
  const int h = (int)(blockIdx.x % a.n_heads);
  const int g = h / a.kv_mul;
  // key blocks of query tile qt: through the block holding the position of
  // its last row below L (rows past L are computed but never stored)
  auto tile_blocks = [&](int qt) { return (a.q_off + imin(qt * kBM + kBM, a.L) - 1) / kBN + 1; };
  const int nb_last = tile_blocks(qb * NT + NT - 1);  // key blocks of the last tile

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::kOffBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + VS;
  uint64_t* s_full = v_empty + VS;
  uint64_t* p_full = s_full + NT;
  uint64_t* mma_done = p_full + NT;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SM::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + SM::kOffMisc + 8);

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < NT; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 4 * NT + 1) {
    tmem_alloc(tmem_slot, 256 * NT);  // tile t: S [256t, 256t+128), O [256t+128, +HD)
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 4 * NT) {
    regs_low();
    if (warp == 4 * NT || warp == 4 * NT + 2) {
      // ------------------------------------------------- producers: K and V
      // one thread each, so that neither ring waits behind the other's
      // free slot (K_j is freed once S(j) is done, V_j once P(j) V_j is)
      if (lane == 0) {
        const bool is_k = warp == 4 * NT;
        const uint64_t pol = l2_evict_first_policy();
        if (is_k) {
          mbar_arrive_expect_tx(q_full, NT * SM::kQBytes);
#pragma unroll
          for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int cb = 0; cb < SM::kCB; ++cb)
              tma_load_2d(smem + SM::kOffQ + t * SM::kQBytes + cb * kBM * 64, &a.tq,
                          h * HD + cb * 32, (qb * NT + t) * kBM, q_full, pol);
        }
        const int S = is_k ? KS : VS;
        uint64_t* full = is_k ? k_full : v_full;
        uint64_t* empty = is_k ? k_empty : v_empty;
        char* ring = smem + (is_k ? SM::kOffK : SM::kOffV);
        const CUtensorMap* map = is_k ? &a.tk : &a.tv;
        for (int j = 0; j < nb_last; ++j) {
          const int st = j % S;
          if (!mbar_wait(&empty[st], (uint32_t)(((j / S) & 1) ^ 1), abort_flag, a.status)) break;
          char* dst = ring + st * SM::kKVBytes;
          mbar_arrive_expect_tx(&full[st], SM::kKVBytes);
#pragma unroll
          for (int cb = 0; cb < SM::kCB; ++cb)
            tma_load_2d(dst + cb * kBN * 64, map, g * HD + cb * 32, j * kBN, &full[st], pol);
        }
      }
    } else if (warp == 4 * NT + 1) {
      // ----------------------------------------------------------- MMA issuer
      // the whole warp runs the loop (uniform operands); one lane issues
      {
        constexpr uint32_t kIdS = idesc_f16(kBM, kBN, false);
        constexpr uint32_t kIdO = idesc_f16(kBM, HD, true);
        // every lane waits; the warp goes on together (all lanes agree on ok)
        auto wwait = [&](uint64_t* bar, uint32_t parity) {
          return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, a.status));
        };
        bool ok = wwait(q_full, 0);
        auto issue_s = [&](int t, int j) {  // S_t(j) = Q_t K_j^T
          const uint32_t sq = smem_u32(smem + SM::kOffQ + t * SM::kQBytes);
          const uint32_t sk = smem_u32(smem + SM::kOffK + (j % KS) * SM::kKVBytes);
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint32_t off = (k >> 1) * kBM * 64 + (k & 1) * 32;
            const uint64_t ad = smem_desc_sw64(sq + off, 16, 512);
            const uint64_t bd = smem_desc_sw64(sk + (k >> 1) * kBN * 64 + (k & 1) * 32, 16, 512);
            tc_mma_f16(tmem + 256 * t, ad, bd, kIdS, k > 0 ? 1u : 0u);
          }
        };
        auto issue_pv = [&](int t, int j) {  // O_t += P_t(j) V_j, P from TMEM
          const uint32_t sv = smem_u32(smem + SM::kOffV + (j % VS) * SM::kKVBytes);
#pragma unroll
          for (int k = 0; k < kBN / 16; ++k) {
            // A = P: 16 keys = 8 columns of FP16 pairs; B = V (MN-major: hd
            // contiguous): 16 keys = two 8-row atoms of 512 B, LBO = stride
            // between 32-half column blocks of hd
            const uint64_t bd = smem_desc_sw64(sv + k * 1024, kBN * 64, 512);
            tc_mma_f16_ta(tmem + 256 * t + 128, tmem + 256 * t + 8 * k, bd, kIdO,
                          (j > 0 || k > 0) ? 1u : 0u);
          }
        };
        ok = ok && wwait(&k_full[0], 0);
        tc_fence_after();
        for (int t = 0; t < NT; ++t) {
          issue_s(t, 0);
          tc_commit(&s_full[t]);
        }
        tc_commit(&k_empty[0]);
        for (int j = 0; j < nb_last; ++j) {
          ok = ok && wwait(&v_full[j % VS], (uint32_t)((j / VS) & 1));
          const bool next_k = j + 1 < nb_last;
          if (next_k)
            ok = ok && wwait(&k_full[(j + 1) % KS], (uint32_t)(((j + 1) / KS) & 1));
          for (int t = 0; t < NT; ++t) {
            const int nb_t = tile_blocks(qb * NT + t);
            if (j >= nb_t) continue;
            ok = ok && wwait(&p_full[t], (uint32_t)(j & 1));
            tc_fence_after();
            issue_pv(t, j);
            if (j + 1 < nb_t) issue_s(t, j + 1);
            tc_commit(&s_full[t]);  // S_t(j+1) (or, last block, the final P V) done
          }
          tc_commit(&v_empty[j % VS]);
          if (next_k) tc_commit(&k_empty[(j + 1) % KS]);
        }
        // every MMA of this CTA has finished before TMEM is released (also on
        // the drain path after a timed-out wait)
        tc_commit(mma_done);
        volatile int no_abort = 0;
        mbar_wait(mma_done, 0, &no_abort, a.status);
        __syncwarp();
        (void)ok;
      }
    }
  } else {
    // ------------------------------------------------------------- softmax
    regs_high();
    const int t = warp >> 2;                  // query tile of this warpgroup
    const int r = tid & 127;                  // row inside the tile (== TMEM lane)
    const int qt = qb * NT + t;               // global 128-row block of the tile
    const int qi = qt * kBM + r;              // query row
    const int qpos = a.q_off + qi;            // its position: keys 0..qpos
    const int nb = tile_blocks(qt);           // causal key blocks of this tile
    const uint32_t lane_sel = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + 256 * t + lane_sel;
    const uint32_t tO = tS + 128;
    float m_ref = -INFINITY, l = 0.f;
    const float sl2 = a.scale_log2;
    // The exp2 unit bounds the exponentials, so the two tiles take turns
    // (ping-pong): in every block tile 0 runs its exponentials, then tile 1.
    // Each tile loads its scores and takes the row max while the other one
    // holds the turn.  Tile 0 waits (barrier 1) for tile 1's block j-1, tile
    // 1 (barrier 2) for tile 0's block j, while the other tile has that block.
    const int nb_o = tile_blocks(qb * NT + (NT - 1 - t));  // the other tile's blocks
    for (int j = 0; j < nb; ++j) {
      mbar_wait(&s_full[t], (uint32_t)(j & 1), abort_flag, a.status);
      tc_fence_after();
      // the whole row of scores in one load; the causal mask touches only
      // blocks holding a key past the tile's first position
      float s[128];
      tmem_ld128(tS, s);
      if (j * kBN + kBN - 1 > a.q_off + qt * kBM) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (j * kBN + c > qpos) s[c] = -INFINITY;
      }
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 128; c += 8) {
        m4[0] = max3(m4[0], s[c], s[c + 1]);
        m4[1] = max3(m4[1], s[c + 2], s[c + 3]);
        m4[2] = max3(m4[2], s[c + 4], s[c + 5]);
        m4[3] = max3(m4[3], s[c + 6], s[c + 7]);
      }
      const float mx = max3(m4[0], m4[1], fmaxf(m4[2], m4[3])) * sl2;
      if (j == 0) {
        m_ref = mx;
      } else if (__any_sync(0xffffffffu, mx > m_ref + kRescaleLog2)) {
        // O holds sum_t 2^(s_t - m_ref) v_t (the P V of block j-1 finished
        // before S(j) was handed over): rescale it to the new max
        const float mnew = fmaxf(m_ref, mx);
        const float alpha = ex2_ftz(m_ref - mnew);
        l *= alpha;
        m_ref = mnew;
#pragma unroll
        for (int c = 0; c < (HD + 31) / 32; ++c) {
          float tt[32];
          tmem_ld32(tO + c * 32, tt);
#pragma unroll
          for (int i = 0; i < 32; ++i) tt[i] *= alpha;
          tmem_st32(tO + c * 32, tt);
        }
      }
      if (t == 0) {
        if (j >= 1 && j - 1 < nb_o) named_sync(1);
      } else if (j < nb_o) {
        named_sync(2);
      }
      // p = 2^(s - m_ref) <= 2^8, FP16 pairs over the first 64 S columns
      uint64_t rsum = pk2(0.f, 0.f);
      const uint64_t SL = pk2(sl2, sl2), NM = pk2(-m_ref, -m_ref);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t w[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int c = hh * 64 + 2 * e;
          const uint64_t X = fma2(pk2(s[c], s[c + 1]), SL, NM);
          float x0, x1;
          upk2(X, x0, x1);
          // the exp2 unit alone would bound this loop: kPolyPairs of every
          // 4 pairs use the FMA-pipe polynomial instead
          float p0, p1;
          if ((e & 3) < kPolyPairs) {
            exp2_poly_pair(x0, x1, p0, p1);
          } else {
            p0 = ex2_ftz(x0);
            p1 = ex2_ftz(x1);
          }
          rsum = add2(rsum, pk2(p0, p1));
          const __half2 hp = __floats2half2_rn(p0, p1);
          w[e] = *reinterpret_cast<const uint32_t*>(&hp);
        }
        tmem_st32u(tS + hh * 32, w);
      }
      // hand the turn over
      if (t == 0) {
        if (j < nb_o) named_arrive(2);
      } else if (j + 1 < nb_o) {
        named_arrive(1);
      }
      tmem_wait_st();
      float rs0, rs1;
      upk2(rsum, rs0, rs1);
      l += rs0 + rs1;
      // P_t(j) (and any O rescale) is in TMEM: the MMA may read it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    // epilogue: O / l once the last P V has finished
    mbar_wait(&s_full[t], (uint32_t)(nb & 1), abort_flag, a.status);
    tc_fence_after();
    const float inv = 1.f / l;
    float* orow = a.out + (int64_t)qi * a.n_heads * HD + (int64_t)h * HD;
    const bool store = qi < a.L;
#pragma unroll
    for (int c = 0; c < HD / 32; ++c) {
      float tt[32];
      tmem_ld32(tO + c * 32, tt);
      if (store) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(orow + c * 32 + i) =
              make_float4(tt[i] * inv, tt[i + 1] * inv, tt[i + 2] * inv, tt[i + 3] * inv);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4 * NT + 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256 * NT);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_prefill() {
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

bool encode_f16_rows(CUtensorMap* map, const void* base, int64_t width, int64_t rows,
                     int64_t stride, std::string* err) {
  auto fn = encode_fn_prefill();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(stride * 2)};
  cuuint32_t box[2] = {32, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
    return false;
  }
  return true;
}

template <int HD, int NT>
int launch_hd(PrefillArgs a, cudaStream_t stream, std::string* err) {
  using SM = PrefillSmem<HD, NT>;
  const size_t smem = SM::kBytes + 1024;
  a.n_qblocks = (a.L + kBM * NT - 1) / (kBM * NT);
  const int grid = a.n_qblocks * a.n_heads;
  static std::atomic<uint64_t> smem_set{0};  // one per instantiation
  ensure_smem_attr(prefill_kernel<HD, NT>, smem, smem_set);
  prefill_kernel<HD, NT><<<grid, SM::kThreads, smem, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("prefill launch failed: ") + cudaGetErrorString(e);
    return GLA_ERR_CUDA;
  }
  return GLA_OK;
}

}  // namespace

int launch_prefill_f16(const uint16_t* q, const uint16_t* k, const uint16_t* v, float* out,
                       int32_t L, int32_t q_off, int64_t kv_stride, int32_t n_heads,
                       int32_t n_kv_heads, int32_t head_dim, float scale, int32_t* status,
                       const DeviceInfo& dev, cudaStream_t stream, std::string* err) {
  if (!(head_dim == 64 || head_dim == 96 || head_dim == 128)) {
    *err = "prefill head_dim must be 64, 96 or 128";
    return GLA_ERR_NOT_SUPPORTED;
  }
  // two 128-row query tiles per CTA
  const size_t need = (head_dim == 64    ? PrefillSmem<64, 2>::kBytes
                       : head_dim == 96 ? PrefillSmem<96, 2>::kBytes
                                        : PrefillSmem<128, 2>::kBytes) +
                      1024;
  if (need > (size_t)dev.smem_optin) {
    *err = "prefill shared memory layout does not fit";
    return GLA_ERR_NOT_SUPPORTED;
  }
  const int64_t qw = (int64_t)n_heads * head_dim, kvw = (int64_t)n_kv_heads * head_dim;
  if ((qw * 2) % 16 != 0 || (kv_stride * 2) % 16 != 0) {
    *err = "prefill row strides must be multiples of 16 bytes";
    return GLA_ERR_ALIGNMENT;
  }
  if (kv_stride < kvw || q_off < 0 || (int64_t)q_off + L > INT32_MAX) {
    *err = "bad prefill key/value rows";
    return GLA_ERR_INVALID_ARG;
  }
  PrefillArgs a{};
  if (!encode_f16_rows(&a.tq, q, qw, L, qw, err) ||
      !encode_f16_rows(&a.tk, k, kvw, (int64_t)q_off + L, kv_stride, err) ||
      !encode_f16_rows(&a.tv, v, kvw, (int64_t)q_off + L, kv_stride, err))
    return GLA_ERR_INVALID_ARG;
  a.out = out;
  a.L = L;
  a.q_off = q_off;
  a.n_heads = n_heads;
  a.kv_mul = n_heads / n_kv_heads;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.status = status;
  switch (head_dim) {
    case 64: return launch_hd<64, 2>(a, stream, err);
    case 96: return launch_hd<96, 2>(a, stream, err);
    default: return launch_hd<128, 2>(a, stream, err);
  }
}

}  // namespace gla
