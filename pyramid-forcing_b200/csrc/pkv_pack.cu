// Pack: gather the planned segments of the sink / middle / recent / merge
// pools into the flat K/V/pos workspace that the attention kernel reads,
// rotating K by the 3D RoPE at the remapped time.
//
// Reference behaviour: pyramidkv/csrc/pyramidkv_pack.cu:28-185.  For a
// segment with t_remap >= 0 the time row of every token is t_remap, else the
// token's stored t; y / x rows come from the stored position; rows are
// clamped into each table; pair p of the 64 complex pairs of head_dim 128
// uses the t table for p < ft_cols, the y table for the next fy_cols and the
// x table for the rest.  V and pos are copied unchanged.
//
// B200 design: a persistent grid walks (segment, 32-token tile) units; every
// thread owns one 16-byte chunk (8 bf16 = 4 complex pairs) of a token row, so
// each warp reads and writes whole 512-byte row pairs with 128-bit accesses.
// The rotation of a pair is evaluated as fma(kr, fr, -(ki*fi)) /
// fma(kr, fi, ki*fr) (kRopeFmaFirst); the reference's compiled kernel is the
// authority on which order nvcc's contraction picks, and the GPU parity tests
// pin this choice against it.
#include "pkv_common.cuh"
#include "pkv_internal.h"
#include "pkv_plan.cuh"

namespace pkv {

constexpr int kPackTile = 32;
enum RopeMode : int { kRopeFmaFirst = 0, kRopeFmaSecond = 1, kRopeNoFma = 2 };

// Process-wide rotation order (see file comment); tests may switch it to
// compare against the reference's build.
static int g_rope_mode = kRopeFmaFirst;

struct PackArgs {
  const uint16_t* k[4];
  const uint16_t* v[4];
  const int64_t* pos[4];
  int64_t rows[4];  // slot rows per pool
  uint16_t* k_out;
  uint16_t* v_out;
  int64_t* pos_out;
  int64_t out_rows;
  const int32_t *sk, *sg, *sl, *dst;
  int n_seg;
  const int64_t* tremap;
  const float *ft, *fy, *fx;
  int ft_rows, ft_cols, fy_rows, fy_cols, fx_rows, fx_cols;
  int F, MTPA, D;
  int rope;         // fused RoPE enabled
  int rope_mode;
  int32_t* status;
};

__device__ __forceinline__ void rotate(float kr, float ki, float fr, float fi, int mode,
                                       float& nr, float& ni) {
  if (mode == kRopeFmaFirst) {
    nr = __fmaf_rn(kr, fr, -__fmul_rn(ki, fi));
    ni = __fmaf_rn(kr, fi, __fmul_rn(ki, fr));
  } else if (mode == kRopeFmaSecond) {
    nr = __fmaf_rn(-ki, fi, __fmul_rn(kr, fr));
    ni = __fmaf_rn(ki, fr, __fmul_rn(kr, fi));
  } else {
    nr = __fsub_rn(__fmul_rn(kr, fr), __fmul_rn(ki, fi));
    ni = __fadd_rn(__fmul_rn(kr, fi), __fmul_rn(ki, fr));
  }
}

__device__ __forceinline__ float2 freq_of(const PackArgs& a, int p, int64_t t, int64_t y,
                                          int64_t x) {
  const float* tab;
  int rows, cols, col;
  int64_t r;
  if (p < a.ft_cols) {
    tab = a.ft; rows = a.ft_rows; cols = a.ft_cols; col = p; r = t;
  } else if (p < a.ft_cols + a.fy_cols) {
    tab = a.fy; rows = a.fy_rows; cols = a.fy_cols; col = p - a.ft_cols; r = y;
  } else {
    tab = a.fx; rows = a.fx_rows; cols = a.fx_cols; col = p - a.ft_cols - a.fy_cols; r = x;
  }
  if (tab == nullptr) return make_float2(1.0f, 0.0f);
  int row = static_cast<int>(r);
  if (row < 0) row = 0;
  if (row >= rows) row = rows - 1;
  return __ldg(reinterpret_cast<const float2*>(tab + (int64_t(row) * cols + col) * 2));
}

template <bool kVec>
__global__ void __launch_bounds__(256) pack_kernel(PackArgs a) {
  const int max_len = a.F > a.MTPA ? a.F : a.MTPA;
  const int tiles = (max_len + kPackTile - 1) / kPackTile;
  const int64_t units = int64_t(a.n_seg) * tiles;
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    const int seg = int(u / tiles);
    const int tile = int(u - int64_t(seg) * tiles);
    const int kind = a.sk[seg];
    if (kind < 0) continue;
    const int len = a.sl[seg];
    if (len <= 0 || tile * kPackTile >= len) continue;
    if (kind > 3) {
      if (tile == 0 && threadIdx.x == 0) flag(a.status, PKV_ST_BAD_KIND);
      continue;
    }
    const int64_t slot = a.sg[seg];
    const int64_t dst0 = a.dst[seg];
    const int stride_tok = kind == kSrcMerge ? a.MTPA : a.F;
    // a segment may span consecutive slots (the legacy all-layer plan) but
    // must stay inside its pool
    if (slot < 0 || slot >= a.rows[kind] ||
        slot * stride_tok + len > a.rows[kind] * stride_tok || dst0 < 0 ||
        dst0 + len > a.out_rows || a.k[kind] == nullptr) {
      if (tile == 0 && threadIdx.x == 0)
        flag(a.status, dst0 + len > a.out_rows ? PKV_ST_PACK_OVERFLOW : PKV_ST_SLOT_RANGE);
      continue;
    }
    const int D = a.D;
    const uint16_t* sk = a.k[kind] + slot * stride_tok * D;
    const uint16_t* sv = a.v[kind] + slot * stride_tok * D;
    const int64_t* sp = a.pos[kind] ? a.pos[kind] + slot * stride_tok * 3 : nullptr;
    uint16_t* dk = a.k_out + dst0 * D;
    uint16_t* dv = a.v_out + dst0 * D;
    const bool rope = a.rope && sp != nullptr;
    const int64_t tm = rope ? a.tremap[seg] : -1;

    // a unit takes tiles tile, tile + tiles, ... of its segment (a legacy
    // all-layer plan's segment spans several slots)
    for (int tok0 = tile * kPackTile; tok0 < len; tok0 += tiles * kPackTile) {
      const int ntok = min(kPackTile, len - tok0);
      if (kVec) {
        const int cpr = D / 8;
        for (int i = threadIdx.x; i < ntok * cpr; i += blockDim.x) {
          const int r = i / cpr, ch = i - r * cpr;
          const int64_t e = int64_t(tok0 + r) * D + ch * 8;
          uint4 kk = *reinterpret_cast<const uint4*>(sk + e);
          const uint4 vv = *reinterpret_cast<const uint4*>(sv + e);
          if (rope) {
            const int64_t* pp = sp + int64_t(tok0 + r) * 3;
            const int64_t pt = tm >= 0 ? tm : pp[0];
            const int64_t py = pp[1], px = pp[2];
            uint32_t w[4] = {kk.x, kk.y, kk.z, kk.w};
  #pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 fq = freq_of(a, ch * 4 + j, pt, py, px);
              const float kr = bf16_bits_to_f32(w[j] & 0xffffu);
              const float ki = bf16_bits_to_f32(w[j] >> 16);
              float nr, ni;
              rotate(kr, ki, fq.x, fq.y, a.rope_mode, nr, ni);
              w[j] = f32_to_bf16_bits(nr) | (f32_to_bf16_bits(ni) << 16);
            }
            kk = make_uint4(w[0], w[1], w[2], w[3]);
          }
          *reinterpret_cast<uint4*>(dk + e) = kk;
          *reinterpret_cast<uint4*>(dv + e) = vv;
        }
      } else {
        const int ppr = D / 2;
        for (int i = threadIdx.x; i < ntok * ppr; i += blockDim.x) {
          const int r = i / ppr, p = i - r * ppr;
          const int64_t e = int64_t(tok0 + r) * D + p * 2;
          uint16_t k0 = sk[e], k1 = sk[e + 1];
          if (rope) {
            const int64_t* pp = sp + int64_t(tok0 + r) * 3;
            const int64_t pt = tm >= 0 ? tm : pp[0];
            const float2 fq = freq_of(a, p, pt, pp[1], pp[2]);
            float nr, ni;
            rotate(bf16_bits_to_f32(k0), bf16_bits_to_f32(k1), fq.x, fq.y, a.rope_mode, nr, ni);
            k0 = static_cast<uint16_t>(f32_to_bf16_bits(nr));
            k1 = static_cast<uint16_t>(f32_to_bf16_bits(ni));
          }
          dk[e] = k0;
          dk[e + 1] = k1;
          dv[e] = sv[e];
          dv[e + 1] = sv[e + 1];
        }
      }
      if (a.pos_out != nullptr && sp != nullptr) {
        int64_t* dp = a.pos_out + dst0 * 3;
        for (int e = threadIdx.x; e < ntok * 3; e += blockDim.x)
          dp[int64_t(tok0) * 3 + e] = sp[int64_t(tok0) * 3 + e];
      }
    }
  }
}

constexpr int kPack128MaxSeg = 2048;  // plans with more segments use pack_kernel

// ---------------------------------------------------------------------------
// Tiles of 64 tokens for the head_dim-128 pack (pack_ws_kernel below): the
// segments are cut into tiles, the tiles listed in segment order and dealt
// to the blocks in equal contiguous ranges.
// ---------------------------------------------------------------------------
constexpr int kBulkTok = 64;
constexpr uint64_t kBulkTimeoutNs = 4000000000ull;

struct BulkTileMeta {
  int64_t dst0;      // packed row of the segment's first token
  int64_t src_row;   // pool row of the tile's first token
  int64_t tm;        // remapped time (>= 0) or -1
  int tok0, ntok, kind;
  int bad;           // segment failed its bounds checks: skip
  int pos_in_smem;   // positions arrived with the bulk copy
};

// The pack that plans for itself (the path MegaCache.attend takes): the
// layer's planner inputs, each (chunk, head)'s sync time and cyclic phase,
// and per candidate segment of every (chunk, head) a descriptor and its
// packed row.
constexpr int kPlanPackMaxHeads = 16;
constexpr int kPlanPackMaxPairs = kPack128MaxSeg / kCand;
// descriptor: kind << 28 | remap source << 26 | slot in the layered pool
constexpr uint32_t kRemapNone = 0, kRemapSync = 1, kRemapMedian = 2;
constexpr int kDescSlotBits = 26;
// The planner inputs (PlanStage) are only read before the first tile is
// issued, so they borrow the stage buffers; the merge medians the producer
// reads later are copied out of them.
struct PlannedSmem {
  uint32_t cand_desc[kPack128MaxSeg];
  int cand_off[kPack128MaxSeg + 1];
  int64_t pair_sync[kPlanPackMaxPairs];
  int pair_phase[kPlanPackMaxPairs];
  int64_t median[kPlanPackMaxHeads * kCandMerge];
  int warp_tok[32];
};

// Row r of a table with `rows` rows, clamped into [0, rows) (rows >= 1).
__device__ __forceinline__ int clamp_row(int64_t r, int rows) {
  if (static_cast<uint64_t>(r) < static_cast<uint64_t>(rows)) return static_cast<int>(r);
  return r < 0 ? 0 : rows - 1;
}
// Two f32 -> one bf16 pair (lo, hi), each rounded to nearest even: the same
// bits as two f32_to_bf16_bits conversions, in one instruction.
__device__ __forceinline__ uint32_t pack_bf16_pair(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ uint32_t pk_smem(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t pk_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool pk_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(pk_smem(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait on a stage; false after kBulkTimeoutNs
__device__ __forceinline__ bool pk_wait(uint64_t* b, uint32_t parity) {
  if (pk_try(b, parity)) return true;
  const uint64_t t0 = pk_now();
  while (!pk_try(b, parity))
    if (pk_now() - t0 > kBulkTimeoutNs) return false;
  return true;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(pk_smem(dst)), "l"(src), "r"(bytes), "r"(pk_smem(b))
      : "memory");
}
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
               ::"l"(dst), "r"(pk_smem(src)), "r"(bytes)
               : "memory");
}

// ---------------------------------------------------------------------------
// The tile list both pack kernels share.  Every thread of the block takes
// part; on return (after a block barrier) tile_start[j] is the first tile of
// segment j and tile_start[n] the total, and with kPlanned the candidates'
// descriptors and packed rows are in `ps` and block 0 has written
// cu_seqlens_k, the token total and the counter.  The planner inputs borrow
// `stage_mem` (>= sizeof(PlanStage<kPlanPackMaxHeads>)) until then.
// kPlanned: the segments are the planner's candidates (pkv_plan.cuh), which
// every block evaluates itself from the staged state records.  Otherwise
// they come from a plan in global memory (sk / sg / sl / dst / tremap).
// ---------------------------------------------------------------------------
template <bool kPlanned>
__device__ int pack_tile_list(const PackArgs& a, const PlanArgs& pa, int* tile_start,
                              int* warp_tot, PlannedSmem& ps, void* stage_mem) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = kPlanned ? pa.C * pa.H * kCand : a.n_seg;
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int s_begin = min(n, int(threadIdx.x) * per), s_end = min(n, s_begin + per);
  int run = 0, tok = 0;  // this thread's tiles and (planned) tokens
  if (kPlanned) {
    // ---- plan: every candidate's descriptor and length, in place of the
    // planner's descriptor arrays
    PlanStage<kPlanPackMaxHeads>& in = *reinterpret_cast<PlanStage<kPlanPackMaxHeads>*>(stage_mem);
    stage_plan_inputs(in, pa, threadIdx.x, blockDim.x);
    __syncthreads();
    for (int pr = threadIdx.x; pr < pa.C * pa.H; pr += blockDim.x) {
      const int c = pr / pa.H, h = pr - c * pa.H;
      const int64_t ct = chunk_time(pa, c);
      ps.pair_sync[pr] = map_sink_time(ct, pa.sink_mode, pa.cmin, pa.cmax, pa.lag);
      ps.pair_phase[pr] = head_phase(in.st[h], ct);
    }
    for (int i = threadIdx.x; i < pa.H * kCandMerge; i += blockDim.x)
      ps.median[i] = in.st[i / kCandMerge].done_median_t[i % kCandMerge];
    __syncthreads();
    for (int j = s_begin; j < s_end; ++j) {
      const int pr = j / kCand, cand = j - pr * kCand;
      const int h = pr % pa.H;
      int kind = 0, slot = 0, len = 0;
      int64_t traw = 0, tremap = -1;
      if (!plan_candidate_at(pa, in, h, cand, ps.pair_sync[pr], ps.pair_phase[pr], kind, slot,
                             len, traw, tremap))
        len = 0;
      const uint32_t src = tremap < 0 ? kRemapNone : kind == kSrcMerge ? kRemapMedian : kRemapSync;
      ps.cand_desc[j] = uint32_t(kind) << 28 | src << kDescSlotBits |
                        uint32_t(len > 0 ? layer_slot(pa, kind, slot) : 0);
      ps.cand_off[j] = len;  // the length until the scan below
      const int nt = (len + kBulkTok - 1) / kBulkTok;
      tile_start[j] = nt;
      run += nt;
      tok += len;
    }
    // the stage buffers' generic-proxy accesses end before the bulk copies
    // (async proxy) write them
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  } else {
    // ---- compact tile list (as pack128_kernel)
    for (int sg = s_begin; sg < s_end; ++sg) {
      const int kind = a.sk[sg], len = a.sl[sg];
      int nt = 0;
      if (kind >= 0 && len > 0) {
        if (kind > 3) {
          if (blockIdx.x == 0) flag(a.status, PKV_ST_BAD_KIND);
        } else {
          nt = (len + kBulkTok - 1) / kBulkTok;
        }
      }
      tile_start[sg] = nt;
      run += nt;
    }
  }
  int incl = run, tincl = tok;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    const int z = __shfl_up_sync(0xffffffffu, tincl, o);
    if (lane >= o) {
      incl += y;
      tincl += z;
    }
  }
  if (lane == 31) {
    warp_tot[warp] = incl;
    if (kPlanned) ps.warp_tok[warp] = tincl;
  }
  __syncthreads();
  int before = 0, total = 0, tbefore = 0, ttotal = 0;
  for (int w = 0; w < int(blockDim.x >> 5); ++w) {
    if (w < warp) before += warp_tot[w];
    total += warp_tot[w];
    if (kPlanned) {
      if (w < warp) tbefore += ps.warp_tok[w];
      ttotal += ps.warp_tok[w];
    }
  }
  int acc = before + incl - run, tacc = tbefore + tincl - tok;
  for (int sg = s_begin; sg < s_end; ++sg) {
    const int nt = tile_start[sg];
    tile_start[sg] = acc;
    acc += nt;
    if (kPlanned) {
      const int len = ps.cand_off[sg];
      ps.cand_off[sg] = tacc;
      tacc += len;
    }
  }
  if (threadIdx.x == 0) {
    tile_start[n] = total;
    if (kPlanned) ps.cand_off[n] = ttotal;
  }
  __syncthreads();
  if (kPlanned && blockIdx.x == 0) {
    // the planner's outputs: cu_seqlens_k, the token total and counter
    const int npair = pa.C * pa.H;
    for (int pr = threadIdx.x; pr <= npair; pr += blockDim.x) pa.cu[pr] = ps.cand_off[pr * kCand];
    if (threadIdx.x == 0) {
      if (pa.total_out) *pa.total_out = ttotal;
      if (pa.counter)
        atomicAdd(reinterpret_cast<unsigned long long*>(pa.counter),
                  static_cast<unsigned long long>(ttotal));
      if (pa.check_capacity && int64_t(ttotal) > pa.capacity) flag(pa.status, PKV_ST_PACK_OVERFLOW);
    }
  }

  return total;
}

struct PackTile {
  int64_t dst0;     // packed row of the segment's first token
  int64_t src_row;  // pool row of the tile's first token
  int64_t tm;       // remapped time (>= 0) or -1
  int tok0, ntok, kind, len;
  int bad;          // segment failed its bounds checks: skip
};

// Tile u of the list; `iseg` is the walker's segment cursor (tiles visited in
// increasing order).  A bad segment's first tile sets the status bit.
template <bool kPlanned>
__device__ __forceinline__ PackTile pack_tile(const PackArgs& a, const PlanArgs& pa,
                                              const int* tile_start, const PlannedSmem& ps,
                                              int& iseg, int u) {
  while (tile_start[iseg + 1] <= u) ++iseg;
  int kind, len;
  int64_t slot, dst0, seg_tremap;
  if (kPlanned) {
    const uint32_t d = ps.cand_desc[iseg];
    kind = int(d >> 28);
    slot = int64_t(d & ((1u << kDescSlotBits) - 1u));
    dst0 = ps.cand_off[iseg];
    len = ps.cand_off[iseg + 1] - ps.cand_off[iseg];
    const uint32_t src = (d >> kDescSlotBits) & 3u;
    const int pr = iseg / kCand;
    seg_tremap = src == kRemapSync ? ps.pair_sync[pr]
                 : src == kRemapMedian
                     ? ps.median[(pr % pa.H) * kCandMerge + iseg - pr * kCand -
                                 (kCandSink + kCandRecent + kCandMiddle)]
                     : int64_t(-1);
  } else {
    kind = a.sk[iseg];
    len = a.sl[iseg];
    slot = a.sg[iseg];
    dst0 = a.dst[iseg];
    seg_tremap = a.tremap != nullptr ? a.tremap[iseg] : -1;
  }
  PackTile t;
  const int stride_tok = kind == kSrcMerge ? a.MTPA : a.F;
  t.kind = kind;
  t.len = len;
  t.tok0 = (u - tile_start[iseg]) * kBulkTok;
  t.ntok = min(kBulkTok, len - t.tok0);
  t.dst0 = dst0;
  // a segment may span consecutive slots (the legacy all-layer plan) but
  // must stay inside its pool
  t.bad = slot < 0 || slot >= a.rows[kind] ||
          slot * stride_tok + len > a.rows[kind] * stride_tok || dst0 < 0 ||
          dst0 + len > a.out_rows || a.k[kind] == nullptr;
  t.src_row = slot * stride_tok + t.tok0;
  t.tm = (a.rope && a.pos[kind] != nullptr) ? seg_tremap : -1;
  return t;
}

// ---------------------------------------------------------------------------
// pack_ws_kernel (head_dim 128): one block per SM, the roles split over
// warps.  Warp 0 keeps a 4-stage ring of K (+ positions) tiles loading with
// cp.async.bulk global -> shared (a plain per-block copy); warp 1 moves V on
// a 5-stage ring of its own (bulk load, then bulk store straight back out,
// the slot reused once the store has read it), which no other warp waits
// on; warps 2..17 rotate and store K and copy the positions, releasing each
// K stage through an mbarrier instead of a block barrier.  Up to 9 tiles
// (150 KB) per SM stay in flight without spending registers on them; the
// earlier design (two blocks per SM, each refilling one 2-stage K+V ring
// only after a block barrier) kept about one tile per block in flight.
// ---------------------------------------------------------------------------
constexpr int kWsKStages = 4;
constexpr int kWsVStages = 5;
constexpr int kWsConsumers = 512;  // 16 warps
constexpr int kWsThreads = kWsConsumers + 64;

struct __align__(128) WsKStage {
  uint16_t k[kBulkTok * 128];
  int64_t pos[kBulkTok * 3];
};
struct __align__(128) WsVStage {
  uint16_t v[kBulkTok * 128];
};
struct WsVMeta {
  int64_t drow;  // packed row of the tile's first token
  int ntok, bad;
};
struct WsSmem {
  WsKStage ks[kWsKStages];
  WsVStage vs[kWsVStages];
  uint64_t kfull[kWsKStages], kempty[kWsKStages], vfull[kWsVStages];
  BulkTileMeta meta[kWsKStages];
  WsVMeta vmeta[kWsVStages];
  int tile_start[kPack128MaxSeg + 1];
  int warp_tot[32];
};
static_assert(sizeof(PlanStage<kPlanPackMaxHeads>) <= sizeof(WsKStage) * kWsKStages,
              "the planner inputs fit the K stage buffers");

__device__ __forceinline__ void pk_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(pk_smem(b)) : "memory");
}
__device__ __forceinline__ void pk_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(pk_smem(b)),
               "r"(bytes)
               : "memory");
}

template <bool kPlanned>
__global__ void __launch_bounds__(kWsThreads, 1) pack_ws_kernel(PackArgs a, PlanArgs pa) {
  extern __shared__ uint8_t pk_raw[];
  WsSmem& sm = *reinterpret_cast<WsSmem*>(
      (reinterpret_cast<uintptr_t>(pk_raw) + 127) & ~uintptr_t(127));
  PlannedSmem& ps = *reinterpret_cast<PlannedSmem*>(
      (reinterpret_cast<uintptr_t>(pk_raw) + 127 + sizeof(WsSmem) + 127) & ~uintptr_t(127));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int st = 0; st < kWsKStages; ++st) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(pk_smem(&sm.kfull[st])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(pk_smem(&sm.kempty[st])),
                   "r"(kWsConsumers / 32));
    }
    for (int st = 0; st < kWsVStages; ++st)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(pk_smem(&sm.vfull[st])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  const int n = kPlanned ? pa.C * pa.H * kCand : a.n_seg;
  const int total = pack_tile_list<kPlanned>(a, pa, sm.tile_start, sm.warp_tot, ps, sm.ks);
  const int per_block = (total + int(gridDim.x) - 1) / int(gridDim.x);
  const int u_begin = min(total, int(blockIdx.x) * per_block);
  const int count = min(total, u_begin + per_block) - u_begin;
  if (count <= 0) return;
  // segment of the block's first tile: tile_start[lo] <= u_begin < tile_start[lo + 1]
  auto first_seg = [&]() {
    int lo = 0, hi = n;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (sm.tile_start[mid] <= u_begin) lo = mid; else hi = mid;
    }
    return lo;
  };

  if (warp == 0) {
    // ---- K producer
    if (lane != 0) return;
    int iseg = first_seg();
    int issued = 0;
    for (; issued < count; ++issued) {
      const int st = issued % kWsKStages;
      if (issued >= kWsKStages &&
          !pk_wait(&sm.kempty[st], uint32_t(issued / kWsKStages - 1) & 1u)) {
        flag(a.status, PKV_ST_TIMEOUT);
        break;
      }
      const PackTile t = pack_tile<kPlanned>(a, pa, sm.tile_start, ps, iseg, u_begin + issued);
      BulkTileMeta& m = sm.meta[st];
      m.kind = t.kind;
      m.tok0 = t.tok0;
      m.ntok = t.ntok;
      m.dst0 = t.dst0;
      m.bad = t.bad;
      m.src_row = t.src_row;
      m.tm = t.tm;
      if (t.bad) {
        if (t.tok0 == 0)
          flag(a.status, t.dst0 + t.len > a.out_rows ? PKV_ST_PACK_OVERFLOW : PKV_ST_SLOT_RANGE);
        m.pos_in_smem = 0;
        pk_arrive(&sm.kfull[st]);
        continue;
      }
      // 16-byte rule of the bulk copy: 24 * src_row and 24 * ntok must be multiples of 16
      m.pos_in_smem = a.pos[t.kind] != nullptr && (t.src_row & 1) == 0 && (t.ntok & 1) == 0;
      const uint32_t k_bytes = uint32_t(t.ntok) * 256;
      const uint32_t pos_bytes = m.pos_in_smem ? uint32_t(t.ntok) * 24 : 0;
      pk_expect(&sm.kfull[st], k_bytes + pos_bytes);
      bulk_g2s(sm.ks[st].k, a.k[t.kind] + t.src_row * 128, k_bytes, &sm.kfull[st]);
      if (pos_bytes)
        bulk_g2s(sm.ks[st].pos, a.pos[t.kind] + t.src_row * 3, pos_bytes, &sm.kfull[st]);
    }
    // let the loads still in flight land before the block's shared memory goes
    for (int i = max(0, issued - kWsKStages); i < issued; ++i)
      pk_wait(&sm.kfull[i % kWsKStages], uint32_t(i / kWsKStages) & 1u);
    return;
  }

  if (warp == 1) {
    // ---- V mover: load -> store, each slot reused once its store has read it
    if (lane != 0) return;
    int iseg = first_seg();
    auto load = [&](int i) {
      const int st = i % kWsVStages;
      const PackTile t = pack_tile<kPlanned>(a, pa, sm.tile_start, ps, iseg, u_begin + i);
      WsVMeta& vm = sm.vmeta[st];
      vm.drow = t.dst0 + t.tok0;
      vm.ntok = t.ntok;
      vm.bad = t.bad;
      if (t.bad) {
        pk_arrive(&sm.vfull[st]);
        return;
      }
      const uint32_t bytes = uint32_t(t.ntok) * 256;
      pk_expect(&sm.vfull[st], bytes);
      bulk_g2s(sm.vs[st].v, a.v[t.kind] + t.src_row * 128, bytes, &sm.vfull[st]);
    };
    int issued = 0;
    for (; issued < min(kWsVStages, count); ++issued) load(issued);
    int j = 0;
    for (; j < count; ++j) {
      const int st = j % kWsVStages;
      if (!pk_wait(&sm.vfull[st], uint32_t(j / kWsVStages) & 1u)) {
        flag(a.status, PKV_ST_TIMEOUT);
        break;
      }
      const WsVMeta vm = sm.vmeta[st];
      if (!vm.bad) bulk_s2g(a.v_out + vm.drow * 128, sm.vs[st].v, uint32_t(vm.ntok) * 256);
      // one group per tile (empty for a bad one), so the groups count tiles
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      if (j >= 1 && issued < count) {
        // tile j - 1's store has read its slot: refill it
        asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        load(issued++);
      }
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    for (int i = j; i < issued; ++i)  // after a timeout: loads still in flight
      pk_wait(&sm.vfull[i % kWsVStages], uint32_t(i / kWsVStages) & 1u);
    return;
  }

  // ---- consumers: rotate K into the packed buffer, copy the positions
  const int ctid = int(threadIdx.x) - 64;
  const int ch = ctid & 15;
  const float2* ftab[4];
  int fcols[4], fsel[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int pp = ch * 4 + j;
    const float* tab;
    int col;
    if (pp < a.ft_cols) {
      tab = a.ft; fcols[j] = a.ft_cols; col = pp; fsel[j] = 0;
    } else if (pp < a.ft_cols + a.fy_cols) {
      tab = a.fy; fcols[j] = a.fy_cols; col = pp - a.ft_cols; fsel[j] = 1;
    } else {
      tab = a.fx; fcols[j] = a.fx_cols; col = pp - a.ft_cols - a.fy_cols; fsel[j] = 2;
    }
    ftab[j] = tab ? reinterpret_cast<const float2*>(tab) + col : nullptr;
  }
  const int rope_mode = a.rope_mode;
  for (int i = 0; i < count; ++i) {
    const int st = i % kWsKStages;
    if (!pk_wait(&sm.kfull[st], uint32_t(i / kWsKStages) & 1u)) {
      if (ctid == 0) flag(a.status, PKV_ST_TIMEOUT);
      break;
    }
    const BulkTileMeta m = sm.meta[st];
    if (!m.bad) {
      const WsKStage& sb = sm.ks[st];
      const int64_t drow = m.dst0 + m.tok0;
      const bool has_pos = a.pos[m.kind] != nullptr;
      const bool rope = a.rope && has_pos;
      const int64_t* gpos = has_pos ? a.pos[m.kind] + m.src_row * 3 : nullptr;
#pragma unroll
      for (int q = 0; q < (kBulkTok * 16) / kWsConsumers; ++q) {
        const int r = (ctid + kWsConsumers * q) >> 4;
        if (r >= m.ntok) continue;
        uint4 kk = *reinterpret_cast<const uint4*>(sb.k + r * 128 + ch * 8);
        if (rope) {
          int64_t pt, py, px;
          if (m.pos_in_smem) {
            pt = sb.pos[r * 3]; py = sb.pos[r * 3 + 1]; px = sb.pos[r * 3 + 2];
          } else {
            pt = __ldg(gpos + r * 3); py = __ldg(gpos + r * 3 + 1); px = __ldg(gpos + r * 3 + 2);
          }
          if (m.tm >= 0) pt = m.tm;
          const int rt = clamp_row(pt, a.ft_rows), ry = clamp_row(py, a.fy_rows);
          const int rx = clamp_row(px, a.fx_rows);
          uint32_t w[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float2 fq = make_float2(1.0f, 0.0f);
            if (ftab[j] != nullptr)
              fq = __ldg(ftab[j] + (fsel[j] == 0 ? rt : fsel[j] == 1 ? ry : rx) * fcols[j]);
            const float kr = bf16_bits_to_f32(w[j] & 0xffffu);
            const float ki = bf16_bits_to_f32(w[j] >> 16);
            float nr, ni;
            rotate(kr, ki, fq.x, fq.y, rope_mode, nr, ni);
            w[j] = pack_bf16_pair(nr, ni);
          }
          kk = make_uint4(w[0], w[1], w[2], w[3]);
        }
        *reinterpret_cast<uint4*>(a.k_out + (drow + r) * 128 + ch * 8) = kk;
      }
      if (a.pos_out != nullptr && has_pos) {
        int64_t* dp = a.pos_out + drow * 3;
        for (int e = ctid; e < m.ntok * 3; e += kWsConsumers)
          dp[e] = m.pos_in_smem ? sb.pos[e] : __ldg(gpos + e);
      }
    }
    __syncwarp();
    if (lane == 0) pk_arrive(&sm.kempty[st]);
  }
}

namespace {

// The pools, the packed outputs and the RoPE tables of a pack launch.
PackArgs pack_args(const pkv_cache_t* c, const float* ft, int ft_rows, int ft_cols,
                   const float* fy, int fy_rows, int fy_cols, const float* fx, int fx_rows,
                   int fx_cols) {
  PackArgs a{};
  const int64_t lh = int64_t(c->num_layers) * c->num_heads;
  a.k[0] = c->sink_k; a.v[0] = c->sink_v; a.pos[0] = c->sink_pos; a.rows[0] = lh * c->max_sink;
  a.k[1] = c->middle_k; a.v[1] = c->middle_v; a.pos[1] = c->middle_pos;
  a.rows[1] = lh * c->max_middle;
  a.k[2] = c->recent_k; a.v[2] = c->recent_v; a.pos[2] = c->recent_pos;
  a.rows[2] = lh * c->max_recent;
  a.k[3] = c->merge_k; a.v[3] = c->merge_v; a.pos[3] = c->merge_pos;
  a.rows[3] = lh * c->max_merge_blocks;
  // pos packing needs every pool's pos (pyramidkv_pack.cu:37-42)
  a.k_out = c->k_flat;
  a.v_out = c->v_flat;
  a.pos_out = c->pos_flat;
  a.out_rows = c->max_pack_tokens;
  a.ft = ft; a.fy = fy; a.fx = fx;
  a.ft_rows = ft ? ft_rows : 0; a.ft_cols = ft ? ft_cols : 0;
  a.fy_rows = fy ? fy_rows : 0; a.fy_cols = fy ? fy_cols : 0;
  a.fx_rows = fx ? fx_rows : 0; a.fx_cols = fx ? fx_cols : 0;
  a.F = c->frame_seqlen;
  a.MTPA = c->max_merge_tokens;
  a.D = c->head_dim;
  a.rope_mode = g_rope_mode;
  a.status = c->status;
  return a;
}

bool pack_vec_ok(const PackArgs& a) {
  bool vec = (a.D % 8 == 0);
  for (int i = 0; i < 4; ++i)
    vec = vec && ((reinterpret_cast<uintptr_t>(a.k[i]) | reinterpret_cast<uintptr_t>(a.v[i])) % 16 == 0);
  return vec;
}

// The head_dim-128 pack's 16-byte rules: head_dim 128, every pool and output
// 16-byte aligned, the segment list within the kernel's tile table.
bool pack_bulk_ok(const PackArgs& a, int n_seg) {
  return pack_vec_ok(a) && a.D == 128 && n_seg <= kPack128MaxSeg &&
         ((reinterpret_cast<uintptr_t>(a.k_out) | reinterpret_cast<uintptr_t>(a.v_out)) % 16 == 0) &&
         ((reinterpret_cast<uintptr_t>(a.pos[0]) | reinterpret_cast<uintptr_t>(a.pos[1]) |
           reinterpret_cast<uintptr_t>(a.pos[2]) | reinterpret_cast<uintptr_t>(a.pos[3])) % 16 == 0);
}

template <bool kPlanned>
constexpr int ws_smem_bytes() {
  return int(sizeof(WsSmem)) + 128 + (kPlanned ? int(sizeof(PlannedSmem)) + 128 : 0);
}

template <bool kPlanned>
int launch_ws(const PackArgs& a, const PlanArgs& pa, cudaStream_t stream) {
  static std::mutex mu;
  static int attr_done[kMaxDevices] = {};
  constexpr int smem = ws_smem_bytes<kPlanned>();
  if (per_device_once(attr_done, mu, [] {
        return cudaFuncSetAttribute(pack_ws_kernel<kPlanned>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    smem) == cudaSuccess ? 1 : 0;
      }) <= 0) {
    cudaGetLastError();
    return PKV_ELAUNCH;
  }
  pack_ws_kernel<kPlanned><<<sm_count(), kWsThreads, smem, stream>>>(a, pa);
  return launch_status();
}

// A persistent grid of exactly the resident blocks.
}  // namespace

int launch_pack(const pkv_cache_t* c, const int32_t* sk, const int32_t* sg, const int32_t* sl,
                const int32_t* dst, int n_seg, const int64_t* tremap, const float* ft,
                int ft_rows, int ft_cols, const float* fy, int fy_rows, int fy_cols,
                const float* fx, int fx_rows, int fx_cols, cudaStream_t stream) {
  if (n_seg == 0) return PKV_OK;
  if (!c || !sk || !sg || !sl || !dst || n_seg < 0 || !c->k_flat || !c->v_flat)
    return PKV_EINVAL;
  PackArgs a = pack_args(c, ft, ft_rows, ft_cols, fy, fy_rows, fy_cols, fx, fx_rows, fx_cols);
  a.sk = sk; a.sg = sg; a.sl = sl; a.dst = dst;
  a.n_seg = n_seg;
  a.tremap = tremap;
  a.rope = tremap != nullptr && (ft != nullptr || fy != nullptr || fx != nullptr);
  if (pack_bulk_ok(a, n_seg)) return launch_ws<false>(a, PlanArgs{}, stream);
  const int max_len = a.F > a.MTPA ? a.F : a.MTPA;
  const int64_t units = int64_t(n_seg) * ((max_len + kPackTile - 1) / kPackTile);
  int64_t grid = int64_t(sm_count()) * 8;
  if (units < grid) grid = units;
  if (grid < 1) grid = 1;
  if (pack_vec_ok(a)) {
    pack_kernel<true><<<int(grid), 256, 0, stream>>>(a);
  } else {
    pack_kernel<false><<<int(grid), 256, 0, stream>>>(a);
  }
  return launch_status();
}

bool plan_pack_fits(const pkv_cache_t* c, const PlanArgs& pa) {
  // every valid candidate is a segment the planner would emit: at most
  // max_sink + max_recent + 24 + 6 <= S of them per (chunk, head), so the
  // planner's per-head cap never binds
  if (!c || !c->k_flat || !c->v_flat || !pa.cu) return false;
  if (!(pa.H <= kPlanPackMaxHeads && pa.C * pa.H * kCand <= kPack128MaxSeg &&
        pa.max_sink <= kCandSink && pa.max_recent <= kCandRecent && pa.mmb <= kCandMerge &&
        pa.max_middle + pa.mmb >= kCandMiddle + kCandMerge && pa.add_layer_offset == 1))
    return false;
  const PackArgs a = pack_args(c, nullptr, 0, 0, nullptr, 0, 0, nullptr, 0, 0);
  for (int k = 0; k < 4; ++k)  // a slot fits its descriptor field
    if (a.rows[k] > (int64_t(1) << kDescSlotBits)) return false;
  return pack_bulk_ok(a, pa.C * pa.H * kCand);
}

int launch_pack_planned(const pkv_cache_t* c, const PlanArgs& pa, const float* ft, int ft_rows,
                        int ft_cols, const float* fy, int fy_rows, int fy_cols, const float* fx,
                        int fx_rows, int fx_cols, cudaStream_t stream) {
  if (!plan_pack_fits(c, pa)) return PKV_EINVAL;
  PackArgs a = pack_args(c, ft, ft_rows, ft_cols, fy, fy_rows, fy_cols, fx, fx_rows, fx_cols);
  a.rope = ft != nullptr || fy != nullptr || fx != nullptr;
  return launch_ws<true>(a, pa, stream);
}

}  // namespace pkv

using namespace pkv;

extern "C" int pkv_pack(const pkv_cache_t* c, const int32_t* src_kind,
                        const int32_t* src_slot_global, const int32_t* seg_lengths,
                        const int32_t* dst_token_offsets, int num_segments,
                        const int64_t* anchor_t_remap, const float* ft, int ft_rows,
                        int ft_cols, const float* fy, int fy_rows, int fy_cols, const float* fx,
                        int fx_rows, int fx_cols, pkv_stream_t stream) {
  return launch_pack(c, src_kind, src_slot_global, seg_lengths, dst_token_offsets,
                     num_segments, anchor_t_remap, ft, ft_rows, ft_cols, fy, fy_rows, fy_cols,
                     fx, fx_rows, fx_cols, static_cast<cudaStream_t>(stream));
}

// Select the evaluation order of the RoPE pair rotation (0: fma on the first
// product, 1: fma on the second, 2: no contraction).  Returns the previous
// order.  Not part of the reference interface; used by the parity tests.
extern "C" int pkv_set_rope_rounding(int mode) {
  const int prev = g_rope_mode;
  if (mode >= 0 && mode <= 2) g_rope_mode = mode;
  return prev;
}
