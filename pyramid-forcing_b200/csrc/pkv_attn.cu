// Ragged-cache attention: softmax(Q K^T * scale) V for every (chunk, head)
// segment of the packed K/V workspace, non-causal.
//
// Reference call: flash_attn_varlen_func at pyramidkv/_mega_cache.py:550-559
// with Q permuted to (chunk, head, token) (:529-534) and the output permuted
// back (:562-569); cu_seqlens_q has stride rows_per_chunk, cu_seqlens_k comes
// from the planner.  Here Q and O are read / written in the caller's
// [1, L_q, H, D] layout directly, so both permute copies disappear.
//
// B200 design (head_dim 128), attn_tc2_kernel:
//   * one CTA per (segment, pair of 128-row query tiles), 1 CTA per SM;
//     segments longest first (7x spread of per-head KV lengths), the query
//     tiles of one segment side by side so they share K/V through L2;
//   * warp 0 issues TMA loads (both Q tiles once, K/V 128-row tiles through a
//     2-stage ring, 128B-swizzled so the tiles are valid UMMA operands as
//     loaded);
//   * warp 1 (one thread) issues tcgen05.mma for both tiles, interleaved so
//     the tensor pipe works on one tile while the other is in softmax;
//   * warps 2-5 and 6-9 (one thread per query row = TMEM lane) run the fp32
//     online softmax of tile 0 and tile 1 on S pulled out of TMEM with
//     tcgen05.ld, write P back as bf16 into the S columns, and rescale O in
//     TMEM only when a row maximum grows by more than 2^8 (exact: the final
//     O / l uses the same stale maximum); part of each row's exp2 runs as a
//     polynomial on the FMA pipe to offload the MUFU unit;
//   * every wait is bounded by a wall-clock limit; on expiry the kernel
//     raises a status bit, drains its own copies and MMAs, frees TMEM and
//     returns.
// Other head dims use a plain CUDA-core kernel.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

constexpr int kBM = 128;          // query rows per tile (= TMEM lanes)
constexpr int kBN = 128;          // keys per tile
constexpr int kHD = 128;          // head dim of the tensor-core path
constexpr uint32_t kHalfBytes = kBM * 64 * 2;   // [128 rows][64 bf16] = 16 KB
constexpr uint32_t kTileBytes = 2 * kHalfBytes; // one 128x128 bf16 tile
constexpr uint64_t kTimeoutNs = 4000000000ull;  // 4 s per wait
constexpr float kRescaleThreshold = 8.0f;        // log2 units

// ---- PTX wrappers -----------------------------------------------------------
__device__ __forceinline__ uint32_t su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false when the CTA is aborting (limit reached here or in
// another role).
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort,
                                          int32_t* status, uint64_t limit_ns = kTimeoutNs) {
  if (mbar_try(b, parity)) return true;
  const uint64_t t0 = now_ns();
  while (!mbar_try(b, parity)) {
    if (*abort) return false;
    if (now_ns() - t0 > limit_ns) {
      *abort = 1;
      flag(status, PKV_ST_TIMEOUT);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(su32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(su32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// Pull a tile of a tensor into L2 ahead of its load (no shared memory, no
// completion to wait for).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          su32(bar))
      : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// 32 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t addr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(addr));
}
__device__ __forceinline__ void tmem_st32(uint32_t addr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          addr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31]));
}
__device__ __forceinline__ void tmem_st16(uint32_t addr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16};" ::"r"(addr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// ---- paired fp32 arithmetic (sm_100 f32x2: two lanes per instruction) -------
struct f2 {
  uint64_t v;
};
__device__ __forceinline__ f2 mk2(float lo, float hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void un2(f2 a, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(a.v));
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair, on the FMA pipe: Cody-Waite reduction x = n + f with
// n = rint(x) (the 1.5 * 2^23 addend leaves n in the low mantissa bits) and
// f in [-0.5, 0.5], a cubic for 2^f, and n added to the exponent field.
// Cubic coefficients: minimax relative-error fit of 2^f on [-0.5, 0.5]
// (exp2_poly_fit.py beside this file), max relative error 7.5e-5 -- far below
// the 2^-8 step of the bf16 P it produces.  x is clamped at -125 so 2^n stays
// a normal number; such weights are below 2^-125 and vanish in the sums.
__device__ __forceinline__ f2 exp2_poly2(f2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  float x0, x1;
  un2(x, x0, x1);
  x = mk2(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const f2 rnd = mk2(kRound, kRound);
  const f2 t = add2(x, rnd);                            // n in the low bits of t
  const f2 f = sub2(x, sub2(t, rnd));                   // f = x - n
  f2 p = fma2(mk2(0.0551716685295105f, 0.0551716685295105f), f,
              mk2(0.2426111251115799f, 0.2426111251115799f));
  p = fma2(p, f, mk2(0.6932609677314758f, 0.6932609677314758f));
  p = fma2(p, f, mk2(0.9999280571937561f, 0.9999280571937561f));
  float p0, p1, t0, t1;
  un2(p, p0, p1);
  un2(t, t0, t1);
  // t's bit pattern is 0x4B400000 + n; shifting it left by 23 leaves n << 23
  const uint32_t e0 = __float_as_uint(t0) << 23, e1 = __float_as_uint(t1) << 23;
  return mk2(__uint_as_float(__float_as_uint(p0) + e0), __uint_as_float(__float_as_uint(p1) + e1));
}

// UMMA shared-memory descriptor, 128-byte swizzle (SM100 version bits = 1).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}
// Instruction descriptor, kind::f16: bf16 A/B, fp32 D, M=128, N=128.
__host__ __device__ constexpr uint32_t idesc_bf16(bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(b_mn_major) << 16) |
         (uint32_t(kBN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Work decomposition.  A unit is (segment, pair of 128-row query tiles); the
// last unit of a segment holds one tile when rows_per_chunk / 128 rounds up
// to an odd count (1560 rows: 6 pairs + one 24-row tile).  Units are ordered
// segment-major, longest segment first, so the units of one segment are
// neighbours and read its K/V from HBM once.
//
// Without a partial-result workspace (AttnArgs::part == nullptr), or with
// fewer units than a quarter of the SMs, the grid has one CTA per unit.
// Otherwise it is one persistent CTA per SM:
//   * phase 1 (only when the units outnumber the SMs): CTA b runs unit b
//     whole (the longest units, side by side as in the one-CTA-per-unit grid);
//   * phase 2: the remaining units are laid end to end on a cost axis (K/V
//     steps x a per-step weight: a pair step costs more than a lone-tile
//     step) and cut into one contiguous range per CTA, sized so that every
//     CTA's phase-1 + phase-2 cost is the same.  A range edge that falls
//     inside a unit splits the unit's K/V steps between CTAs (stream-K).
// Each piece of a split unit writes its unnormalised O, row maximum m and
// row sum l (fp32) to a per-CTA slot of the workspace; per (unit, tile, warp)
// an arrival counter picks the last piece to finish, which combines
//   O = sum_p 2^(m_p - M) O_p / sum_p 2^(m_p - M) l_p,  M = max_p m_p
// and stores the bf16 rows.  No CTA waits for another.
// ---------------------------------------------------------------------------
struct AttnArgs {
  const int32_t* cu;
  int n_seg, H, rows_per_chunk, m_tiles;
  float scale_log2;
  uint16_t* out;
  int64_t o_row_stride, o_head_stride;
  int32_t* status;
  float* part;     // [kMaxCtas][2 slots][2 tiles][kPartFloats] partials, or nullptr
  int32_t* cnt;    // [units][2 tiles][4 warps] arrival counters, zero between launches
  int w_pair, w_single, w_fixed;  // cost model: phase-1 step weights, per-piece cost
  int w2_pair, w2_single;         // phase-2 step weights
  int prefetch;                   // K/V steps pulled into L2 ahead of their loads
};

// ---------------------------------------------------------------------------
// Two query tiles per CTA (ping-pong).  Warp 0: TMA; warp 1: tcgen05.mma
// issue; warps 2-5: softmax of tile 0; warps 6-9: softmax of tile 1.  TMEM:
// S0 | S1 | O0 | O1, 128 columns each; P_t overwrites S_t as bf16 pairs.  MMA
// issue order per K/V tile j:
//   PV0(j-1)  QK0(j)  PV1(j-1)  QK1(j)
// so while one softmax warpgroup works on S_t(j) the tensor pipe runs the
// other tile's P·V and Q·K^T.  The tensor pipe executes one CTA's MMAs in
// issue order, so QK_t(j) (which overwrites S_t) runs after PV_t(j-1) (which
// reads P_t from the same columns), and the commit that signals S_t(j) also
// covers PV_t(j-1): a softmax warpgroup that sees S_t(j) may rescale O_t.
// Across pieces of a persistent CTA the barriers keep counting: the K/V ring
// by global step, S/P by per-tile step, O-final by per-tile piece, and a
// q_empty commit after a piece's last Q·K^T lets the next piece's Q load.
// The first P·V of a piece (which overwrites O_t) waits for P_t of that
// piece, which the softmax warps post only after reading O_t of the last one.
// Softmax: exp2 of 3 of every 16 column pairs on the FMA pipe (exp2_poly2),
// the rest on MUFU; the last (partial) K tile uses MUFU only, which maps the
// masked -inf scores to exactly 0.
// ---------------------------------------------------------------------------
constexpr int kThreads2 = 320;
constexpr int kStages2 = 2;
constexpr int kMaxSegLens = 1024;    // segment lengths / ranks staged in shared memory
constexpr int kMaxCtas = kAttnMaxCtas;  // persistent grid bound (>= SM count)
constexpr int kMaxSplitUnits = 2048;     // phase-2 units staged in shared memory
constexpr int64_t kPartFloats = kAttnPartFloats;  // O columns x rows, m, l, per-warp unit ids
static_assert(kAttnPartFloats == 130 * kBM + 32, "partial block layout");

struct __align__(1024) AttnSmem2 {
  uint8_t q[2][kTileBytes];
  uint8_t k[kStages2][kTileBytes];
  uint8_t v[kStages2][kTileBytes];
  uint64_t q_full, q_empty;
  uint64_t kv_full[kStages2];
  uint64_t kv_empty[kStages2];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_final[2];
  uint64_t mma_drain;
  uint32_t tmem_base;
  int abort;
  int seg1;                        // this CTA's phase-1 segment (lengths not staged)
  int64_t pre2[kMaxSplitUnits + 1];  // phase-2 cost prefix
  int64_t bnd[kMaxCtas + 1];         // CTA range bounds on the phase-2 axis
  int seg_len[kMaxSegLens];
  int16_t order[kMaxSegLens];        // segment of each length rank
};

// Row max over 128 raw scores held as bits (tree of 3-input max).
__device__ __forceinline__ float row_max128(const uint32_t (&s)[4][32]) {
  float m[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float a[11];
#pragma unroll
    for (int i = 0; i < 10; ++i)
      a[i] = max3(__uint_as_float(s[q][3 * i]), __uint_as_float(s[q][3 * i + 1]),
                  __uint_as_float(s[q][3 * i + 2]));
    a[10] = fmaxf(__uint_as_float(s[q][30]), __uint_as_float(s[q][31]));
    const float b0 = max3(a[0], a[1], a[2]), b1 = max3(a[3], a[4], a[5]);
    const float b2 = max3(a[6], a[7], a[8]), b3 = fmaxf(a[9], a[10]);
    m[q] = fmaxf(max3(b0, b1, b2), b3);
  }
  return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

// Which column pairs of a 32-column chunk take the FMA-pipe exp2: 3 of 16
// (pairs 2, 7, 12).  Measured on B200 (attention kernel case, one call):
// 0.5245 ms with 3 of 16, 0.5263 with 4, 0.5284 with 2, 0.543 with 6, 0.567
// with 8, and all on MUFU 1.4% slower than 6 of 16: the FMA / ALU side is
// the more contended pipe.
__host__ __device__ constexpr bool poly_pair(int i) { return i % 5 == 2; }

// P for 32 columns (16 pairs) of one row: p = 2^(s * scale - m), summed into
// two paired accumulators and packed to bf16 pairs.
template <bool kMixed>
__device__ __forceinline__ void softmax_chunk(const uint32_t (&s)[32], f2 scale2, f2 negm2,
                                              f2& acc0, f2& acc1, uint32_t (&pr)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const f2 x = fma2(mk2(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), scale2,
                      negm2);
    f2 p;
    if (kMixed && poly_pair(i)) {
      p = exp2_poly2(x);
    } else {
      float x0, x1;
      un2(x, x0, x1);
      p = mk2(fast_exp2(x0), fast_exp2(x1));
    }
    if (i & 1)
      acc1 = add2(acc1, p);
    else
      acc0 = add2(acc0, p);
    float p0, p1;
    un2(p, p0, p1);
    pr[i] = pack_bf16x2(p0, p1);
  }
}

// One piece of work: K/V steps [k0, k1) of unit q (segment seg, query tiles
// 2*unit and 2*unit+1 of each chunk's rows).
struct Piece {
  int q, seg, unit, ntile, k0, k1, kv0, lk, whole;
};

// Read-only view of the schedule every CTA computes in shared memory.
struct Sched {
  const AttnSmem2* sm;
  const int32_t* cu;
  int m_tiles, w_pair, w_single;  // phase-2 step weights
  int U, NU, G, n1, n2;  // units per segment, units, grid, phase-1 units, phase-2 units
  bool staged;           // segment lengths and ranks in shared memory

  __device__ int seg_len(int s) const { return staged ? sm->seg_len[s] : cu[s + 1] - cu[s]; }
  // Segment, query-tile pair, tile count and K/V steps of unit q.
  __device__ void unit(int q, int& seg, int& u, int& ntile, int& nkv) const {
    const int r = q / U;
    u = q - r * U;
    seg = staged ? int(sm->order[r]) : sm->seg1;
    ntile = (2 * u + 1 < m_tiles) ? 2 : 1;
    nkv = (seg_len(seg) + kBN - 1) / kBN;
  }
  __device__ int weight(int ntile) const { return ntile == 2 ? w_pair : w_single; }
  // K/V step at which cost position B cuts phase-2 unit q2.
  __device__ int cut(int64_t B, int q2, int w, int nkv) const {
    const int64_t base = sm->pre2[q2];
    if (B <= base) return 0;
    const int64_t k = (B - base) / w;
    return k >= nkv ? nkv : int(k);
  }
  __device__ void fill(Piece& p, int q, int seg, int u, int ntile, int k0, int k1,
                       int nkv) const {
    p.q = q;
    p.seg = seg;
    p.unit = u;
    p.ntile = ntile;
    p.k0 = k0;
    p.k1 = k1;
    p.kv0 = cu[seg];
    p.lk = seg_len(seg);
    p.whole = (k0 == 0 && k1 == nkv) ? 1 : 0;
  }
  // First phase-2 unit whose cost interval ends after position B.
  __device__ int first_unit_after(int64_t B) const {
    int lo = 0, hi = n2;  // smallest q2 with pre2[q2 + 1] > B
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (sm->pre2[mid + 1] > B)
        hi = mid;
      else
        lo = mid + 1;
    }
    return lo;
  }
  // Last CTA whose range starts at or before position B.
  __device__ int cta_at(int64_t B) const {
    int lo = 0, hi = G - 1;  // largest j with bnd[j] <= B
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (sm->bnd[mid] <= B)
        lo = mid;
      else
        hi = mid - 1;
    }
    return lo;
  }
};

// Pieces of CTA b in order: its phase-1 unit, then its phase-2 range.
struct Cursor {
  int stage, q2;
};

__device__ __forceinline__ bool next_piece(const Sched& S, int b, Cursor& cur, Piece& p) {
  int seg, u, ntile, nkv;
  if (cur.stage == 0) {
    cur.stage = 1;
    cur.q2 = S.n2 > 0 ? S.first_unit_after(S.sm->bnd[b]) : 0;
    if (b < S.n1) {
      S.unit(b, seg, u, ntile, nkv);
      if (nkv > 0) {
        S.fill(p, b, seg, u, ntile, 0, nkv, nkv);
        return true;
      }
    }
  }
  if (S.n2 == 0) return false;
  const int64_t lo = S.sm->bnd[b], hi = S.sm->bnd[b + 1];
  while (cur.q2 < S.n2 && S.sm->pre2[cur.q2] < hi) {
    const int q2 = cur.q2++;
    S.unit(S.n1 + q2, seg, u, ntile, nkv);
    if (nkv == 0) continue;
    const int w = S.weight(ntile);
    const int k0 = S.cut(lo, q2, w, nkv), k1 = S.cut(hi, q2, w, nkv);
    if (k1 > k0) {
      S.fill(p, S.n1 + q2, seg, u, ntile, k0, k1, nkv);
      return true;
    }
  }
  return false;
}

// Store one warp's 32 rows x 128 columns of fp32 as normalised bf16 rows.
__device__ __forceinline__ void store_row32(uint16_t* dst, const uint32_t (&o)[32], float inv) {
#pragma unroll
  for (int e = 0; e < 32; e += 8) {
    uint4 w;
    w.x = pack_bf16x2(__uint_as_float(o[e + 0]) * inv, __uint_as_float(o[e + 1]) * inv);
    w.y = pack_bf16x2(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
    w.z = pack_bf16x2(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
    w.w = pack_bf16x2(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
    *reinterpret_cast<uint4*>(dst + e) = w;
  }
}

__device__ __forceinline__ float* part_block(const AttnArgs& a, int cta, int slot, int t) {
  return a.part + (size_t(cta) * 4 + slot * 2 + t) * kPartFloats;
}

__global__ void __launch_bounds__(kThreads2, 1)
    attn_tc2_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  AttnSmem2& sm = *reinterpret_cast<AttnSmem2*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort = &sm.abort;
  const int b = blockIdx.x;

  Sched S;
  S.sm = &sm;
  S.cu = a.cu;
  S.m_tiles = a.m_tiles;
  S.w_pair = a.w2_pair;
  S.w_single = a.w2_single;
  S.U = (a.m_tiles + 1) >> 1;
  S.NU = a.n_seg * S.U;
  S.G = gridDim.x;
  S.staged = a.n_seg <= kMaxSegLens;
  // with a workspace: a whole first wave when the units outnumber the SMs,
  // else every unit cut between the SMs (phase 2 only)
  const bool split = a.part != nullptr && S.staged && S.G <= kMaxCtas &&
                     (S.NU > S.G ? S.NU - S.G : S.NU) <= kMaxSplitUnits;
  S.n1 = split ? (S.NU > S.G ? S.G : 0) : S.NU;
  S.n2 = split ? S.NU - S.n1 : 0;

  if (threadIdx.x == 0) {
    sm.seg1 = -1;
    sm.abort = 0;
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 1);
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_full[t], 4);
      mbar_init(&sm.o_final[t], 1);
    }
    mbar_init(&sm.mma_drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // ---- schedule: segment ranks (longest first, ties by index) ----
  if (S.staged)
    for (int s = threadIdx.x; s < a.n_seg; s += blockDim.x) sm.seg_len[s] = a.cu[s + 1] - a.cu[s];
  __syncthreads();
  {
    const int my_order = b / S.U;  // phase-1 rank of this CTA (unstaged grids)
    for (int s = threadIdx.x; s < a.n_seg; s += blockDim.x) {
      const int ls = S.seg_len(s);
      int rank = 0;
      for (int o = 0; o < a.n_seg; ++o) {
        const int lo = S.seg_len(o);
        rank += (lo > ls) || (lo == ls && o < s);
      }
      if (S.staged)
        sm.order[rank] = int16_t(s);
      else if (rank == my_order)
        sm.seg1 = s;
    }
  }
  __syncthreads();
  // ---- schedule: phase-2 cost prefix and CTA ranges (warp 0) ----
  // Costs are in units of the measured step times: phase-1 steps weigh
  // w_pair / w_single, phase-2 steps w2_pair / w2_single (a piece's steps run
  // a little slower there, its K/V less often found in L2), every piece
  // w_fixed more.  CTA b's phase-2 range is its share of the phase-2 work
  // that brings it to the mean total cost.
  if (split && warp == 0) {
    int seg, u, ntile, nkv;
    const int per = (S.n2 + 31) / 32;
    const int i0 = min(S.n2, lane * per), i1 = min(S.n2, i0 + per);
    int64_t run = 0;
    for (int i = i0; i < i1; ++i) {
      S.unit(S.n1 + i, seg, u, ntile, nkv);
      run += int64_t(nkv) * S.weight(ntile);
    }
    int64_t incl = run;  // inclusive warp scan of the lane totals
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    run = incl - run;
    for (int i = i0; i < i1; ++i) {
      S.unit(S.n1 + i, seg, u, ntile, nkv);
      run += int64_t(nkv) * S.weight(ntile);
      sm.pre2[i + 1] = run;
    }
    if (lane == 0) sm.pre2[0] = 0;
    const int64_t P2 = __shfl_sync(0xffffffffu, incl, 31);
    // phase-1 cost of this lane's CTAs (a contiguous chunk of <= 5)
    const int per1 = (S.G + 31) / 32;
    const int c0 = min(S.G, lane * per1), c1e = min(S.G, c0 + per1);
    int64_t c1 = 0;
    for (int i = c0; i < c1e && i < S.n1; ++i) {
      S.unit(i, seg, u, ntile, nkv);
      c1 += nkv > 0 ? int64_t(nkv) * (ntile == 2 ? a.w_pair : a.w_single) + a.w_fixed : 0;
    }
    int64_t c1_all = c1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c1_all += __shfl_xor_sync(0xffffffffu, c1_all, o);
    const double T = double(c1_all + P2 + int64_t(S.n2) * a.w_fixed) / S.G;
    double bl = 0.0;  // this lane's budgets: T - phase-1 cost, at least 0
    for (int i = c0; i < c1e; ++i) {
      int64_t c = 0;
      if (i < S.n1) {
        S.unit(i, seg, u, ntile, nkv);
        c = nkv > 0 ? int64_t(nkv) * (ntile == 2 ? a.w_pair : a.w_single) + a.w_fixed : 0;
      }
      bl += fmax(0.0, T - double(c));
    }
    double binc = bl;  // inclusive scan of the lane budget sums
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, binc, o);
      if (lane >= o) binc += y;
    }
    const double bsum = __shfl_sync(0xffffffffu, binc, 31);
    const double scale = bsum > 0.0 ? double(P2) / bsum : 0.0;
    double acc = binc - bl;
    for (int i = c0; i < c1e; ++i) {
      if (bsum > 0.0) {
        sm.bnd[i] = int64_t(acc * scale);
        int64_t c = 0;
        if (i < S.n1) {
          S.unit(i, seg, u, ntile, nkv);
          c = nkv > 0 ? int64_t(nkv) * (ntile == 2 ? a.w_pair : a.w_single) + a.w_fixed : 0;
        }
        acc += fmax(0.0, T - double(c));
      } else {
        sm.bnd[i] = int64_t(double(P2) * (double(i) / S.G));
      }
    }
    if (lane == 0) sm.bnd[S.G] = P2;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     su32(&sm.tmem_base)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      Cursor cur{0, 0};
      Piece p;
      int pi = 0, gs = 0, q_issued = -1;
      while (!*abort && next_piece(S, b, cur, p)) {
        if (pi > 0 && !mbar_wait(&sm.q_empty, (pi - 1) & 1, abort, a.status)) break;
        const int c = p.seg / a.H, h = p.seg - c * a.H;
        const int row0 = c * a.rows_per_chunk + 2 * p.unit * kBM;
        mbar_expect_tx(&sm.q_full, p.ntile * kTileBytes);
        for (int t = 0; t < p.ntile; ++t) {
          tma_load_3d(sm.q[t], &tm_q, &sm.q_full, 0, h, row0 + t * kBM);
          tma_load_3d(sm.q[t] + kHalfBytes, &tm_q, &sm.q_full, 64, h, row0 + t * kBM);
        }
        q_issued = pi;
        bool ok = true;
        // K/V tiles the ring reaches in the next steps go to L2 now, so their
        // loads find them there even when no neighbouring CTA read them
        for (int j = p.k0; j < p.k1 && j < p.k0 + a.prefetch; ++j) {
          const int y = p.kv0 + j * kBN;
          tma_prefetch_2d(&tm_k, 0, y);
          tma_prefetch_2d(&tm_k, 64, y);
          tma_prefetch_2d(&tm_v, 0, y);
          tma_prefetch_2d(&tm_v, 64, y);
        }
        for (int j = p.k0; j < p.k1; ++j, ++gs) {
          const int s = gs % kStages2;
          if (gs >= kStages2 &&
              !mbar_wait(&sm.kv_empty[s], ((gs / kStages2) + 1) & 1, abort, a.status)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&sm.kv_full[s], 2 * kTileBytes);
          const int y = p.kv0 + j * kBN;
          tma_load_2d(sm.k[s], &tm_k, &sm.kv_full[s], 0, y);
          tma_load_2d(sm.k[s] + kHalfBytes, &tm_k, &sm.kv_full[s], 64, y);
          tma_load_2d(sm.v[s], &tm_v, &sm.kv_full[s], 0, y);
          tma_load_2d(sm.v[s] + kHalfBytes, &tm_v, &sm.kv_full[s], 64, y);
          if (a.prefetch > 0 && j + a.prefetch < p.k1) {
            const int yp = y + a.prefetch * kBN;
            tma_prefetch_2d(&tm_k, 0, yp);
            tma_prefetch_2d(&tm_k, 64, yp);
            tma_prefetch_2d(&tm_v, 0, yp);
            tma_prefetch_2d(&tm_v, 64, yp);
          }
        }
        if (!ok) break;
        ++pi;
      }
      if (*abort) {
        // drain this CTA's own copies before the shared memory goes away
        if (q_issued >= 0) {
          const uint64_t t0 = now_ns();
          while (!mbar_try(&sm.q_full, q_issued & 1) && now_ns() - t0 < kTimeoutNs) {
          }
        }
        for (int g = gs > kStages2 ? gs - kStages2 : 0; g < gs; ++g) {
          const uint64_t t1 = now_ns();
          while (!mbar_try(&sm.kv_full[g % kStages2], (g / kStages2) & 1) &&
                 now_ns() - t1 < kTimeoutNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t id_qk = idesc_bf16(false);
      constexpr uint32_t id_pv = idesc_bf16(true);
      // Descriptor words computed once: the start-address field (bits 0-13,
      // address >> 4) of a tile plus a constant offset stays inside the field
      // (shared memory ends below 256 KB), so each MMA's descriptor is one
      // add on the low word.  One thread keeps the tensor pipe fed with
      // 128x128x16 MMAs (64 cycles each) only if little scalar work sits
      // between them: measured on B200, issue takes 64 cycles per MMA with
      // precomputed descriptors and 110-260 with per-MMA address arithmetic.
      const uint64_t dq0 = sdesc_sw128(su32(sm.q[0]), 16, 1024);
      const uint32_t d_hi = uint32_t(dq0 >> 32);  // SBO and layout bits, the same for all
      const uint32_t q_lo0 = uint32_t(dq0);
      const uint32_t q_lo1 = uint32_t(sdesc_sw128(su32(sm.q[1]), 16, 1024));
      const uint32_t k_lo0 = uint32_t(sdesc_sw128(su32(sm.k[0]), 16, 1024));
      const uint32_t k_lo1 = uint32_t(sdesc_sw128(su32(sm.k[1]), 16, 1024));
      const uint32_t v_lo0 = uint32_t(sdesc_sw128(su32(sm.v[0]), kHalfBytes, 1024));
      const uint32_t v_lo1 = uint32_t(sdesc_sw128(su32(sm.v[1]), kHalfBytes, 1024));
      static_assert(kStages2 == 2, "descriptor words are kept for two stages");
      auto desc = [d_hi](uint32_t lo) { return (uint64_t(d_hi) << 32) | lo; };
      auto issue_qk = [&](int t, int g) {
        const uint32_t q_lo = t ? q_lo1 : q_lo0;
        const uint32_t k_lo = (g & 1) ? k_lo1 : k_lo0;
        const uint32_t d_tm = tmem + t * 128;
#pragma unroll
        for (int kk = 0; kk < kHD / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4;
          mma_ss(d_tm, desc(q_lo + off), desc(k_lo + off), id_qk, kk > 0 ? 1u : 0u);
        }
        tc_commit(&sm.s_full[t]);
      };
      auto issue_pv = [&](int t, int g, bool first) {
        const uint32_t v_lo = (g & 1) ? v_lo1 : v_lo0;
        const uint32_t d_tm = tmem + 256 + t * 128, p_tm = tmem + t * 128;
        const uint32_t acc0 = first ? 0u : 1u;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // A = P_t (TMEM, 2 bf16 per column), B = V rows kk*16.. (MN-major)
          mma_ts(d_tm, p_tm + kk * 8, desc(v_lo + ((kk * 2048) >> 4)), id_pv,
                 kk > 0 ? 1u : acc0);
        }
      };
      Cursor cur{0, 0};
      Piece p;
      int pi = 0, gs = 0, ts0 = 0, ts1 = 0;
      bool ok = true;
      while (ok && next_piece(S, b, cur, p)) {
        const int n = p.k1 - p.k0;
        ok = mbar_wait(&sm.q_full, pi & 1, abort, a.status);
        if (ok) ok = mbar_wait(&sm.kv_full[gs % kStages2], (gs / kStages2) & 1, abort, a.status);
        if (!ok) break;
        tc_fence_after();
        for (int t = 0; t < p.ntile; ++t) issue_qk(t, gs);
        for (int j = 0; j < n; ++j) {
          const int g = gs + j;
          const bool more = j + 1 < n;
          if (!mbar_wait(&sm.p_full[0], (ts0 + j) & 1, abort, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(0, g, j == 0);
          if (!more) tc_commit(&sm.o_final[0]);
          if (more) {
            if (!mbar_wait(&sm.kv_full[(g + 1) % kStages2], ((g + 1) / kStages2) & 1, abort,
                           a.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_qk(0, g + 1);
          }
          if (p.ntile == 2) {
            if (!mbar_wait(&sm.p_full[1], (ts1 + j) & 1, abort, a.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(1, g, j == 0);
            if (!more) tc_commit(&sm.o_final[1]);
          }
          tc_commit(&sm.kv_empty[g % kStages2]);
          if (p.ntile == 2 && more) issue_qk(1, g + 1);
        }
        if (!ok) break;
        tc_commit(&sm.q_empty);  // every Q·K^T of this piece has been issued
        gs += n;
        ts0 += n;
        if (p.ntile == 2) ts1 += n;
        ++pi;
      }
      // every MMA issued here completes before the CTA frees TMEM
      tc_commit(&sm.mma_drain);
      const uint64_t t0 = now_ns();
      while (!mbar_try(&sm.mma_drain, 0) && now_ns() - t0 < kTimeoutNs) {
      }
    }
  } else {
    // ---------------- softmax / correction / epilogue of tile t ----------------
    const int t = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = uint32_t(quad * 32) << 16;
    const uint32_t s_tm = tmem + t * 128 + lane_off;
    const uint32_t o_tm = tmem + 256 + t * 128 + lane_off;
    const float sc = a.scale_log2;
    // empty segments: zero their output rows (segments b, b + G, ...)
    for (int s = b; s < a.n_seg; s += S.G) {
      if (S.seg_len(s) != 0) continue;
      const int c = s / a.H, h = s - c * a.H;
      for (int r = threadIdx.x - 64; r < a.rows_per_chunk; r += kThreads2 - 64) {
        uint16_t* dst = a.out + int64_t(c * a.rows_per_chunk + r) * a.o_row_stride +
                        int64_t(h) * a.o_head_stride;
        for (int e = 0; e < kHD; e += 8)
          *reinterpret_cast<uint4*>(dst + e) = make_uint4(0, 0, 0, 0);
      }
    }
    Cursor cur{0, 0};
    Piece p;
    int ts = 0, tp = 0, slots = 0;
    bool ok = true;
    while (ok && next_piece(S, b, cur, p)) {
      if (t >= p.ntile) continue;
      const int n = p.k1 - p.k0;
      float m_ref = -INFINITY;  // running reference maximum (log2 domain)
      float l_sum = 0.0f;
      for (int j = 0; j < n; ++j) {
        if (!mbar_wait(&sm.s_full[t], (ts + j) & 1, abort, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(s_tm + q * 32, sr[q]);
        tmem_wait_ld();
        const int valid = p.lk - (p.k0 + j) * kBN;  // keys of this tile inside the segment
        const bool partial = valid < kBN;
        if (partial) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (q * 32 + e >= valid) sr[q][e] = __float_as_uint(-INFINITY);
        }
        const float m_new = fmaxf(m_ref, row_max128(sr) * sc);
        const bool grow = m_new > m_ref + kRescaleThreshold || j == 0;
        float alpha = 1.0f;
        if (grow) {
          alpha = (j == 0) ? 0.0f : fast_exp2(m_ref - m_new);
          m_ref = m_new;
        }
        const f2 scale2 = mk2(sc, sc), negm2 = mk2(-m_ref, -m_ref);
        f2 acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = mk2(0.0f, 0.0f);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t pr[16];
          if (partial)
            softmax_chunk<false>(sr[q], scale2, negm2, acc[2 * q], acc[2 * q + 1], pr);
          else
            softmax_chunk<true>(sr[q], scale2, negm2, acc[2 * q], acc[2 * q + 1], pr);
          tmem_st16(s_tm + q * 16, pr);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = add2(acc[i], acc[i + 4]);
        acc[0] = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
        float r0, r1;
        un2(acc[0], r0, r1);
        l_sum = l_sum * alpha + (r0 + r1);
        // O_t *= alpha for the rows whose reference maximum moved.  S_t(j)
        // was committed after PV_t(j-1), so O_t is complete here.
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t orr[32];
            tmem_ld32(o_tm + q * 32, orr);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
            tmem_st32(o_tm + q * 32, orr);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[t]);
      }
      if (!ok || !mbar_wait(&sm.o_final[t], tp & 1, abort, a.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      ts += n;
      ++tp;
      const int c = p.seg / a.H, h = p.seg - c * a.H;
      const int grow_row = (2 * p.unit + t) * kBM + row;
      const bool store = grow_row < a.rows_per_chunk;
      uint16_t* dst = a.out + int64_t(c * a.rows_per_chunk + grow_row) * a.o_row_stride +
                      int64_t(h) * a.o_head_stride;
      if (p.whole) {
        const float inv = l_sum > 0.0f ? 1.0f / l_sum : 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t orr[32];
          tmem_ld32(o_tm + q * 32, orr);
          tmem_wait_ld();
          if (store) store_row32(dst + q * 32, orr, inv);
        }
        continue;
      }
      // ---- a piece of a split unit: partial out, last arrival combines ----
      if (slots >= 2) {  // cannot happen: only a range's first and last pieces split
        flag(a.status, PKV_ST_SLOT_RANGE);
        continue;
      }
      float* mine = part_block(a, b, slots++, t);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t orr[32];
        tmem_ld32(o_tm + q * 32, orr);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) mine[(q * 32 + e) * kBM + row] = __uint_as_float(orr[e]);
      }
      mine[128 * kBM + row] = m_ref;
      mine[129 * kBM + row] = l_sum;
      if (lane == 0) reinterpret_cast<int*>(mine + 130 * kBM)[quad] = p.q;
      __threadfence();
      __syncwarp();
      const int q2 = p.q - S.n1;
      const int w = S.weight(p.ntile);
      const int nkv = (p.lk + kBN - 1) / kBN;
      const int64_t u_lo = sm.pre2[q2], u_hi = sm.pre2[q2 + 1];
      const int j_lo = S.cta_at(u_lo);
      int last = 0;
      if (lane == 0) {
        int npieces = 0;
        for (int j = j_lo; j < S.G && sm.bnd[j] < u_hi; ++j)
          npieces += S.cut(sm.bnd[j + 1], q2, w, nkv) > S.cut(sm.bnd[j], q2, w, nkv);
        int* ctr = a.cnt + (size_t(p.q) * 2 + t) * 4 + quad;
        const int old = atomicAdd(ctr, 1);
        last = old == npieces - 1;
        if (last) *ctr = 0;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      __threadfence();
      // combine every piece's rows (this one's included, from the workspace)
      float M = -INFINITY;
      for (int j = j_lo; j < S.G && sm.bnd[j] < u_hi; ++j) {
        if (S.cut(sm.bnd[j + 1], q2, w, nkv) <= S.cut(sm.bnd[j], q2, w, nkv)) continue;
        const float* pj = part_block(a, j, 0, t);
        if (__ldcg(reinterpret_cast<const int*>(pj + 130 * kBM) + quad) != p.q)
          pj = part_block(a, j, 1, t);
        M = fmaxf(M, __ldcg(pj + 128 * kBM + row));
      }
      float L = 0.0f;
      for (int j = j_lo; j < S.G && sm.bnd[j] < u_hi; ++j) {
        if (S.cut(sm.bnd[j + 1], q2, w, nkv) <= S.cut(sm.bnd[j], q2, w, nkv)) continue;
        const float* pj = part_block(a, j, 0, t);
        if (__ldcg(reinterpret_cast<const int*>(pj + 130 * kBM) + quad) != p.q)
          pj = part_block(a, j, 1, t);
        L += fast_exp2(__ldcg(pj + 128 * kBM + row) - M) * __ldcg(pj + 129 * kBM + row);
      }
      const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        float accv[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) accv[e] = 0.0f;
        for (int j = j_lo; j < S.G && sm.bnd[j] < u_hi; ++j) {
          if (S.cut(sm.bnd[j + 1], q2, w, nkv) <= S.cut(sm.bnd[j], q2, w, nkv)) continue;
          const float* pj = part_block(a, j, 0, t);
          if (__ldcg(reinterpret_cast<const int*>(pj + 130 * kBM) + quad) != p.q)
            pj = part_block(a, j, 1, t);
          const float wj = fast_exp2(__ldcg(pj + 128 * kBM + row) - M);
#pragma unroll
          for (int e = 0; e < 32; ++e) accv[e] = fmaf(wj, __ldcg(pj + (q * 32 + e) * kBM + row), accv[e]);
        }
        uint32_t ob[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) ob[e] = __float_as_uint(accv[e]);
        if (store) store_row32(dst + q * 32, ob, inv);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// ---------------------------------------------------------------------------
// CUDA-core path (any even head_dim <= 256): one thread per query row,
// K/V tiles staged in shared memory, fp32 online softmax.
// ---------------------------------------------------------------------------
constexpr int kSimtRows = 64;
constexpr int kSimtKeys = 16;
constexpr int kSimtMaxD = 256;

__global__ void __launch_bounds__(kSimtRows)
    attn_simt_kernel(const uint16_t* __restrict__ q, int64_t q_rs, int64_t q_hs,
                     const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                     const int32_t* __restrict__ cu, int H, int rows_per_chunk, int D,
                     float scale, uint16_t* __restrict__ out, int64_t o_rs, int64_t o_hs) {
  __shared__ float ks[kSimtKeys][kSimtMaxD + 1];
  __shared__ float vs[kSimtKeys][kSimtMaxD + 1];
  const int seg = blockIdx.y;
  const int c = seg / H, h = seg - c * H;
  const int r = blockIdx.x * kSimtRows + threadIdx.x;
  const bool live = r < rows_per_chunk;
  const int kv0 = cu[seg], lk = cu[seg + 1] - kv0;
  float qv[kSimtMaxD], acc[kSimtMaxD];
  const uint16_t* qr = q + int64_t(c * rows_per_chunk + (live ? r : 0)) * q_rs + int64_t(h) * q_hs;
  for (int d = 0; d < D; ++d) {
    qv[d] = live ? bf16_bits_to_f32(qr[d]) * scale : 0.0f;
    acc[d] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;
  for (int t0 = 0; t0 < lk; t0 += kSimtKeys) {
    const int nt = min(kSimtKeys, lk - t0);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * D; i += blockDim.x) {
      const int t = i / D, d = i - t * D;
      ks[t][d] = bf16_bits_to_f32(k[int64_t(kv0 + t0 + t) * D + d]);
      vs[t][d] = bf16_bits_to_f32(v[int64_t(kv0 + t0 + t) * D + d]);
    }
    __syncthreads();
    for (int t = 0; t < nt; ++t) {
      float s = 0.0f;
      for (int d = 0; d < D; ++d) s = fmaf(qv[d], ks[t][d], s);
      const float mn = fmaxf(m, s);
      const float corr = __expf(m - mn);
      const float p = __expf(s - mn);
      l = l * corr + p;
      for (int d = 0; d < D; ++d) acc[d] = fmaf(p, vs[t][d], acc[d] * corr);
      m = mn;
    }
  }
  if (!live) return;
  const float inv = l > 0.0f ? 1.0f / l : 0.0f;
  uint16_t* orow = out + int64_t(c * rows_per_chunk + r) * o_rs + int64_t(h) * o_hs;
  for (int d = 0; d < D; ++d) orow[d] = static_cast<uint16_t>(f32_to_bf16_bits(acc[d] * inv));
}

// Self-test of the bounded wait: one thread waits on an mbarrier that nothing
// arrives at, with the attention kernel's wait helper and a caller-chosen
// limit, so the timeout path (status bit, return) runs on the GPU without a
// fault or a hang.
__global__ void wait_selftest_kernel(int32_t* status, uint64_t limit_ns, int32_t* result) {
  __shared__ uint64_t bar;
  __shared__ int abort;
  if (threadIdx.x != 0) return;
  abort = 0;
  mbar_init(&bar, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  const bool ok = mbar_wait(&bar, 0, &abort, status, limit_ns);
  *result = ok ? 1 : 0;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

static bool make_map(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
                     const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims,
                        strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Cost weights of the schedule: a phase-1 K/V step of a tile pair and of a
// lone tile, the fixed cost of one piece, a phase-2 step of a pair and of a
// lone tile; and how many K/V steps ahead the producer pulls tiles into L2
// (0: none; measured no gain).  PKV_ATTN_COST="p1,s1,fixed,p2,s2" and
// PKV_ATTN_PREFETCH=steps override them (tuning).
static void attn_weights(AttnArgs& a) {
  static int w[6] = {0, 0, 0, 0, 0, 0};
  static std::once_flag once;
  std::call_once(once, [] {
    // measured on B200 (C2 attend shape): a lone-tile step takes 0.89 of a
    // pair step, phase-2 steps ~1.08 of phase-1 ones, a piece ~1.3 steps more
    const int def[6] = {9, 8, 12, 10, 9, 0};
    for (int i = 0; i < 6; ++i) w[i] = def[i];
    if (const char* e = getenv("PKV_ATTN_COST")) {
      int v[5] = {0, 0, 0, 0, 0};
      if (sscanf(e, "%d,%d,%d,%d,%d", &v[0], &v[1], &v[2], &v[3], &v[4]) == 5 && v[0] > 0 &&
          v[1] > 0 && v[2] >= 0 && v[3] > 0 && v[4] > 0)
        for (int i = 0; i < 5; ++i) w[i] = v[i];
    }
    if (const char* e = getenv("PKV_ATTN_PREFETCH")) {
      const int d = atoi(e);
      if (d >= 0 && d <= 8) w[5] = d;
    }
  });
  a.w_pair = w[0];
  a.w_single = w[1];
  a.w_fixed = w[2];
  a.w2_pair = w[3];
  a.w2_single = w[4];
  a.prefetch = w[5];
}

int launch_attention(const uint16_t* q, int64_t q_rs, int64_t q_hs, const uint16_t* k,
                     const uint16_t* v, int64_t kv_rows, const int32_t* cu, int num_chunks,
                     int H, int rows_per_chunk, int D, float scale, uint16_t* out, int64_t o_rs,
                     int64_t o_hs, int32_t* status, const AttnWorkspace* ws,
                     cudaStream_t stream) {
  if (num_chunks == 0 || H == 0 || rows_per_chunk == 0) return PKV_OK;
  if (!q || !k || !v || !cu || !out || num_chunks < 0 || H < 0 || rows_per_chunk < 0 || D <= 0)
    return PKV_EINVAL;
  const int n_seg = num_chunks * H;
  const bool tc_ok = D == kHD && scale > 0.0f && kv_rows > 0 && kv_rows < (int64_t(1) << 31) &&
                     (reinterpret_cast<uintptr_t>(q) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(k) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(v) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(out) % 16 == 0) && q_rs % 8 == 0 &&
                     q_hs % 8 == 0 && o_rs % 8 == 0 && o_hs % 8 == 0 && q_rs > 0 && q_hs >= 0 &&
                     int64_t(num_chunks) * rows_per_chunk < (int64_t(1) << 31);
  if (tc_ok) {
    CUtensorMap mq, mk, mv;
    const cuuint64_t kv_dims[2] = {cuuint64_t(kHD), cuuint64_t(kv_rows)};
    const cuuint64_t kv_str[1] = {cuuint64_t(kHD) * 2};
    const cuuint32_t kv_box[2] = {64, kBN};
    const cuuint64_t q_dims[3] = {cuuint64_t(kHD), cuuint64_t(H),
                                  cuuint64_t(num_chunks) * rows_per_chunk};
    const cuuint64_t q_str[2] = {cuuint64_t(q_hs > 0 ? q_hs : kHD) * 2, cuuint64_t(q_rs) * 2};
    const cuuint32_t q_box[3] = {64, 1, kBM};
    if (make_map(&mk, k, 2, kv_dims, kv_str, kv_box) &&
        make_map(&mv, v, 2, kv_dims, kv_str, kv_box) &&
        make_map(&mq, q, 3, q_dims, q_str, q_box)) {
      AttnArgs a{};
      a.cu = cu;
      a.n_seg = n_seg;
      a.H = H;
      a.rows_per_chunk = rows_per_chunk;
      a.m_tiles = (rows_per_chunk + kBM - 1) / kBM;
      a.scale_log2 = scale * 1.4426950408889634f;
      a.out = out;
      a.o_row_stride = o_rs;
      a.o_head_stride = o_hs;
      a.status = status;
      attn_weights(a);
      const size_t smem = sizeof(AttnSmem2) + 1024;
      static std::mutex mu;
      static int attr_done[kMaxDevices] = {};
      if (per_device_once(attr_done, mu, [smem] {
            return cudaFuncSetAttribute(attn_tc2_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(smem)) == cudaSuccess
                       ? 1
                       : 0;
          }) <= 0) {
        cudaGetLastError();
        return PKV_ELAUNCH;
      }
      const int64_t units = int64_t(n_seg) * ((a.m_tiles + 1) / 2);
      // persistent stream-K grid when a workspace is given and the units
      // outnumber the SMs (the schedule's arrays fit shared memory)
      int grid = int(units);
      const int G = sm_count() < kMaxCtas ? sm_count() : kMaxCtas;
      // (units fewer than a quarter of the SMs stay one CTA per unit: too
      // little work to cut)
      if (ws != nullptr && ws->part != nullptr && ws->cnt != nullptr && units * 4 > G &&
          units <= ws->cnt_units && n_seg <= kMaxSegLens &&
          (units > G ? units - G : units) <= kMaxSplitUnits) {
        a.part = ws->part;
        a.cnt = ws->cnt;
        grid = G;
      }
      if (units >= (int64_t(1) << 31)) return PKV_EUNSUPPORTED;
      attn_tc2_kernel<<<grid, kThreads2, smem, stream>>>(mq, mk, mv, a);
      return launch_status();
    }
  }
  if (D > kSimtMaxD || (D & 1)) return PKV_EUNSUPPORTED;
  dim3 grid((rows_per_chunk + kSimtRows - 1) / kSimtRows, n_seg);
  attn_simt_kernel<<<grid, kSimtRows, 0, stream>>>(q, q_rs, q_hs, k, v, cu, H, rows_per_chunk,
                                                   D, scale, out, o_rs, o_hs);
  return launch_status();
}

}  // namespace pkv

using namespace pkv;

extern "C" int pkv_attention(const uint16_t* q, int64_t q_row_stride, int64_t q_head_stride,
                             const uint16_t* k, const uint16_t* v, int64_t kv_rows,
                             const int32_t* cu_seqlens_k, int num_chunks, int num_heads,
                             int rows_per_chunk, int head_dim, float softmax_scale, uint16_t* out,
                             int64_t o_row_stride, int64_t o_head_stride, pkv_stream_t stream) {
  return launch_attention(q, q_row_stride, q_head_stride, k, v, kv_rows, cu_seqlens_k,
                          num_chunks, num_heads, rows_per_chunk, head_dim, softmax_scale, out,
                          o_row_stride, o_head_stride, nullptr, nullptr,
                          static_cast<cudaStream_t>(stream));
}

extern "C" int64_t pkv_attention_workspace_bytes(int num_chunks, int num_heads,
                                                 int rows_per_chunk) {
  if (num_chunks < 0 || num_heads < 0 || rows_per_chunk < 0) return 0;
  const int64_t tiles = (int64_t(rows_per_chunk) + kBM - 1) / kBM;
  const int64_t units = int64_t(num_chunks) * num_heads * ((tiles + 1) / 2);
  return align256(kAttnPartBytes) + align256(units * kAttnCntPerUnit * 4);
}

extern "C" int pkv_attention_ws(const uint16_t* q, int64_t q_row_stride, int64_t q_head_stride,
                                const uint16_t* k, const uint16_t* v, int64_t kv_rows,
                                const int32_t* cu_seqlens_k, int num_chunks, int num_heads,
                                int rows_per_chunk, int head_dim, float softmax_scale,
                                uint16_t* out, int64_t o_row_stride, int64_t o_head_stride,
                                void* workspace, int64_t workspace_bytes, pkv_stream_t stream) {
  if (workspace == nullptr)
    return pkv_attention(q, q_row_stride, q_head_stride, k, v, kv_rows, cu_seqlens_k,
                         num_chunks, num_heads, rows_per_chunk, head_dim, softmax_scale, out,
                         o_row_stride, o_head_stride, stream);
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0 ||
      workspace_bytes < pkv_attention_workspace_bytes(num_chunks, num_heads, rows_per_chunk))
    return PKV_EINVAL;
  AttnWorkspace ws{};
  char* base = static_cast<char*>(workspace);
  ws.part = reinterpret_cast<float*>(base);
  ws.cnt = reinterpret_cast<int32_t*>(base + align256(kAttnPartBytes));
  ws.cnt_units = (workspace_bytes - align256(kAttnPartBytes)) / (kAttnCntPerUnit * 4);
  return launch_attention(q, q_row_stride, q_head_stride, k, v, kv_rows, cu_seqlens_k,
                          num_chunks, num_heads, rows_per_chunk, head_dim, softmax_scale, out,
                          o_row_stride, o_head_stride, nullptr, &ws,
                          static_cast<cudaStream_t>(stream));
}

extern "C" int pkv_wait_selftest(int32_t* status, int64_t limit_ns, int32_t* result,
                                 pkv_stream_t stream) {
  if (!status || !result || limit_ns <= 0 || limit_ns > int64_t(kTimeoutNs)) return PKV_EINVAL;
  pkv::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      status, uint64_t(limit_ns), result);
  return pkv::launch_status();
}
