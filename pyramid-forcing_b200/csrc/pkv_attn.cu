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

#include "pkv_common.cuh"

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

struct AttnArgs {
  const int32_t* cu;
  int n_seg, H, rows_per_chunk, m_tiles;
  float scale_log2;
  uint16_t* out;
  int64_t o_row_stride, o_head_stride;
  int32_t* status;
};

// ---------------------------------------------------------------------------
// Two query tiles per CTA (ping-pong).  One CTA per (segment, pair of 128-row
// query tiles); both tiles stream the same K/V tiles.  Warp 0: TMA; warp 1:
// tcgen05.mma issue; warps 2-5: softmax of tile 0; warps 6-9: softmax of
// tile 1.  TMEM: S0 | S1 | O0 | O1, 128 columns each; P_t overwrites S_t as
// bf16 pairs.  MMA issue order per K/V tile j:
//   PV0(j-1)  QK0(j)  PV1(j-1)  QK1(j)
// so while one softmax warpgroup works on S_t(j) the tensor pipe runs the
// other tile's P·V and Q·K^T.  The tensor pipe executes one CTA's MMAs in
// issue order, so QK_t(j) (which overwrites S_t) runs after PV_t(j-1) (which
// reads P_t from the same columns), and the commit that signals S_t(j) also
// covers PV_t(j-1): a softmax warpgroup that sees S_t(j) may rescale O_t.
// Softmax: exp2 of 2 of every 5 column pairs on the FMA pipe (exp2_poly2),
// the rest on MUFU; the last (partial) K tile uses MUFU only, which maps the
// masked -inf scores to exactly 0.
// ---------------------------------------------------------------------------
constexpr int kThreads2 = 320;
constexpr int kStages2 = 2;
constexpr int kMaxSegLens = 1024;  // segment lengths staged in shared memory

struct __align__(1024) AttnSmem2 {
  uint8_t q[2][kTileBytes];
  uint8_t k[kStages2][kTileBytes];
  uint8_t v[kStages2][kTileBytes];
  uint64_t q_full;
  uint64_t kv_full[kStages2];
  uint64_t kv_empty[kStages2];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_final[2];
  uint64_t mma_drain;
  uint32_t tmem_base;
  int abort;
  int seg, unit;
  int seg_len[kMaxSegLens];
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

// Which column pairs of a 32-column chunk take the FMA-pipe exp2: 6 of 16.
__host__ __device__ constexpr bool poly_pair(int i) { return i % 5 == 1 || i % 5 == 3; }

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

__global__ void __launch_bounds__(kThreads2, 1)
    attn_tc2_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  AttnSmem2& sm = *reinterpret_cast<AttnSmem2*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort = &sm.abort;
  // Segment-major: the units of one segment are adjacent CTAs, so they run
  // side by side and read its K/V from HBM once (scheduling the odd last
  // tiles after all pairs measured slower: their K/V had left L2).
  const int units = (a.m_tiles + 1) >> 1;
  const int order = blockIdx.x / units;
  const int unit_of_block = blockIdx.x - order * units;

  if (threadIdx.x == 0) {
    sm.seg = -1;
    sm.unit = unit_of_block;
    sm.abort = 0;
    mbar_init(&sm.q_full, 1);
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
  // Longest segments first: the segment whose rank (#segments longer, ties
  // by index) equals this CTA's order; one thread per candidate segment,
  // lengths staged in shared memory when they fit.
  const bool lens_in_smem = a.n_seg <= kMaxSegLens;
  if (lens_in_smem)
    for (int s = threadIdx.x; s < a.n_seg; s += blockDim.x) sm.seg_len[s] = a.cu[s + 1] - a.cu[s];
  __syncthreads();
  for (int s = threadIdx.x; s < a.n_seg; s += blockDim.x) {
    const int ls = lens_in_smem ? sm.seg_len[s] : a.cu[s + 1] - a.cu[s];
    int rank = 0;
    for (int o = 0; o < a.n_seg; ++o) {
      const int lo = lens_in_smem ? sm.seg_len[o] : a.cu[o + 1] - a.cu[o];
      rank += (lo > ls) || (lo == ls && o < s);
    }
    if (rank == order) sm.seg = s;
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

  const int seg = sm.seg;
  const int unit = sm.unit;
  const uint32_t tmem = sm.tmem_base;
  const int c = seg >= 0 ? seg / a.H : 0;
  const int h = seg >= 0 ? seg - c * a.H : 0;
  const int kv0 = seg >= 0 ? a.cu[seg] : 0;
  const int lk = seg >= 0 ? a.cu[seg + 1] - kv0 : 0;
  const int nkv = (lk + kBN - 1) / kBN;
  const int ntile = (2 * unit + 1 < a.m_tiles) ? 2 : 1;  // query tiles in this CTA
  const int row0 = c * a.rows_per_chunk + 2 * unit * kBM;  // global query row of tile 0

  if (seg >= 0 && nkv > 0) {
    if (warp == 0) {
      // ---------------- TMA producer ----------------
      if (lane == 0) {
        mbar_expect_tx(&sm.q_full, ntile * kTileBytes);
        for (int t = 0; t < ntile; ++t) {
          tma_load_3d(sm.q[t], &tm_q, &sm.q_full, 0, h, row0 + t * kBM);
          tma_load_3d(sm.q[t] + kHalfBytes, &tm_q, &sm.q_full, 64, h, row0 + t * kBM);
        }
        int issued = 0;
        for (int j = 0; j < nkv; ++j) {
          const int s = j % kStages2;
          if (j >= kStages2 &&
              !mbar_wait(&sm.kv_empty[s], ((j / kStages2) + 1) & 1, abort, a.status))
            break;
          mbar_expect_tx(&sm.kv_full[s], 2 * kTileBytes);
          const int y = kv0 + j * kBN;
          tma_load_2d(sm.k[s], &tm_k, &sm.kv_full[s], 0, y);
          tma_load_2d(sm.k[s] + kHalfBytes, &tm_k, &sm.kv_full[s], 64, y);
          tma_load_2d(sm.v[s], &tm_v, &sm.kv_full[s], 0, y);
          tma_load_2d(sm.v[s] + kHalfBytes, &tm_v, &sm.kv_full[s], 64, y);
          issued = j + 1;
        }
        if (*abort) {
          // drain this CTA's own copies before the shared memory goes away
          const uint64_t t0 = now_ns();
          while (!mbar_try(&sm.q_full, 0) && now_ns() - t0 < kTimeoutNs) {
          }
          for (int j = issued > kStages2 ? issued - kStages2 : 0; j < issued; ++j) {
            const uint64_t t1 = now_ns();
            while (!mbar_try(&sm.kv_full[j % kStages2], (j / kStages2) & 1) &&
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
        auto issue_qk = [&](int t, int j) {
          const uint32_t q_lo = t ? q_lo1 : q_lo0;
          const uint32_t k_lo = (j & 1) ? k_lo1 : k_lo0;
          const uint32_t d_tm = tmem + t * 128;
#pragma unroll
          for (int kk = 0; kk < kHD / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4;
            mma_ss(d_tm, desc(q_lo + off), desc(k_lo + off), id_qk, kk > 0 ? 1u : 0u);
          }
          tc_commit(&sm.s_full[t]);
        };
        auto issue_pv = [&](int t, int j) {
          const uint32_t v_lo = (j & 1) ? v_lo1 : v_lo0;
          const uint32_t d_tm = tmem + 256 + t * 128, p_tm = tmem + t * 128;
          const uint32_t acc0 = j > 0 ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            // A = P_t (TMEM, 2 bf16 per column), B = V rows kk*16.. (MN-major)
            mma_ts(d_tm, p_tm + kk * 8, desc(v_lo + ((kk * 2048) >> 4)), id_pv,
                   kk > 0 ? 1u : acc0);
          }
        };
        bool ok = mbar_wait(&sm.q_full, 0, abort, a.status);
        if (ok) ok = mbar_wait(&sm.kv_full[0], 0, abort, a.status);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < ntile; ++t) issue_qk(t, 0);
        }
        for (int j = 0; ok && j < nkv; ++j) {
          const bool more = j + 1 < nkv;
          if (!mbar_wait(&sm.p_full[0], j & 1, abort, a.status)) break;
          tc_fence_after();
          issue_pv(0, j);
          if (!more) tc_commit(&sm.o_final[0]);
          if (more) {
            const int s1 = (j + 1) % kStages2;
            if (!mbar_wait(&sm.kv_full[s1], ((j + 1) / kStages2) & 1, abort, a.status)) break;
            tc_fence_after();
            issue_qk(0, j + 1);
          }
          if (ntile == 2) {
            if (!mbar_wait(&sm.p_full[1], j & 1, abort, a.status)) break;
            tc_fence_after();
            issue_pv(1, j);
            if (!more) tc_commit(&sm.o_final[1]);
          }
          tc_commit(&sm.kv_empty[j % kStages2]);
          if (ntile == 2 && more) issue_qk(1, j + 1);
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
      if (t < ntile) {
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t lane_off = uint32_t(quad * 32) << 16;
        const uint32_t s_tm = tmem + t * 128 + lane_off;
        const uint32_t o_tm = tmem + 256 + t * 128 + lane_off;
        const float sc = a.scale_log2;
        float m_ref = -INFINITY;  // running reference maximum (log2 domain)
        float l_sum = 0.0f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
          if (!mbar_wait(&sm.s_full[t], j & 1, abort, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t sr[4][32];
#pragma unroll
          for (int q = 0; q < 4; ++q) tmem_ld32(s_tm + q * 32, sr[q]);
          tmem_wait_ld();
          const int valid = lk - j * kBN;  // keys of this tile inside the segment
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
              for (int e = 0; e < 32; ++e)
                orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
              tmem_st32(o_tm + q * 32, orr);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.p_full[t]);
        }
        if (ok && mbar_wait(&sm.o_final[t], 0, abort, a.status)) {
          tc_fence_after();
          const int grow_row = (2 * unit + t) * kBM + row;
          const bool store = grow_row < a.rows_per_chunk;
          const float inv = l_sum > 0.0f ? 1.0f / l_sum : 0.0f;
          uint16_t* dst = a.out + int64_t(c * a.rows_per_chunk + grow_row) * a.o_row_stride +
                          int64_t(h) * a.o_head_stride;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t orr[32];
            tmem_ld32(o_tm + q * 32, orr);
            tmem_wait_ld();
            if (store) {
#pragma unroll
              for (int e = 0; e < 32; e += 8) {
                uint4 w;
                w.x = pack_bf16x2(__uint_as_float(orr[e + 0]) * inv,
                                  __uint_as_float(orr[e + 1]) * inv);
                w.y = pack_bf16x2(__uint_as_float(orr[e + 2]) * inv,
                                  __uint_as_float(orr[e + 3]) * inv);
                w.z = pack_bf16x2(__uint_as_float(orr[e + 4]) * inv,
                                  __uint_as_float(orr[e + 5]) * inv);
                w.w = pack_bf16x2(__uint_as_float(orr[e + 6]) * inv,
                                  __uint_as_float(orr[e + 7]) * inv);
                *reinterpret_cast<uint4*>(dst + q * 32 + e) = w;
              }
            }
          }
        }
      }
    }
  } else if (seg >= 0 && warp >= 2) {
    // empty segment: zero this CTA's output rows
    const int t = (warp - 2) >> 2;
    const int grow_row = (2 * unit + t) * kBM + (warp & 3) * 32 + lane;
    if (t < ntile && grow_row < a.rows_per_chunk) {
      uint16_t* dst = a.out + int64_t(c * a.rows_per_chunk + grow_row) * a.o_row_stride +
                      int64_t(h) * a.o_head_stride;
      for (int e = 0; e < kHD; e += 8) *reinterpret_cast<uint4*>(dst + e) = make_uint4(0, 0, 0, 0);
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

int launch_attention(const uint16_t* q, int64_t q_rs, int64_t q_hs, const uint16_t* k,
                     const uint16_t* v, int64_t kv_rows, const int32_t* cu, int num_chunks,
                     int H, int rows_per_chunk, int D, float scale, uint16_t* out, int64_t o_rs,
                     int64_t o_hs, int32_t* status, cudaStream_t stream) {
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
      const size_t smem = sizeof(AttnSmem2) + 1024;
      static bool attr_set = false;
      if (!attr_set) {
        if (cudaFuncSetAttribute(attn_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(smem)) != cudaSuccess)
          return PKV_ELAUNCH;
        attr_set = true;
      }
      const int units = (a.m_tiles + 1) / 2;
      attn_tc2_kernel<<<n_seg * units, kThreads2, smem, stream>>>(mq, mk, mv, a);
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
                          o_row_stride, o_head_stride, nullptr, static_cast<cudaStream_t>(stream));
}

extern "C" int pkv_wait_selftest(int32_t* status, int64_t limit_ns, int32_t* result,
                                 pkv_stream_t stream) {
  if (!status || !result || limit_ns <= 0 || limit_ns > int64_t(kTimeoutNs)) return PKV_EINVAL;
  pkv::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      status, uint64_t(limit_ns), result);
  return pkv::launch_status();
}
