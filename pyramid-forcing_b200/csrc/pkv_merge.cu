// Merge-strategy accumulation: per merge head, the frames of one block are
// averaged over spatial patch groups (patch_size x patch_size tokens of every
// frame of the block) in fp32 and finalized into the merge anchor pool.
//
// Reference behaviour: pyramidkv/csrc/mega_merge_accum.cu:52-252.
//   * a new block zeroes the accumulator rows [0, MTPA), derives the group of
//     every token from its (y, x) position ((y/ps)*cols + x/ps, cols and rows
//     from the frame's max x / y), counts tokens per group (x block_frames =
//     the finalize divisor) and records each group's (t, y0, x0);
//   * every merge frame adds its bf16 K/V into the group rows in fp32;
//   * the block's last frame writes sum * (1/divisor) as bf16 into
//     merge_*_pool[finalize_idx], the group positions, and the group count.
//
// B200 design: the reference runs one CTA of D threads per head and walks the
// 1560 tokens serially.  Here a CTA owns (head, tile of 32 groups): it builds
// the token list of each of its groups in ascending token order (one warp,
// match/ballot ranking), then every warp reduces whole groups with its lanes
// spread over head_dim (for head_dim 128, 4 dims per lane, a group's token rows
// loaded 8 at a time before they are added).  Each accumulator element still
// receives its tokens in ascending order, frame after frame, so the fp32 sums
// are bit-identical to the reference's sequential loop.  The finalize multiplies by the
// correctly rounded reciprocal (__frcp_rn), which equals the reference's
// fast-math reciprocal for the power-of-two divisors these grids produce.
#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

constexpr int kGroupsPerCta = 32;
constexpr int kMergeThreads = 256;

struct SlotCache {
  int valid;       // group ids of this accumulator slot are loaded in smem
  int num_groups;  // safe_ng of the slot
};

__device__ __forceinline__ void pos_of(const MergeLaunch& m, int f, int h, int t, int64_t& pt,
                                       int32_t& y, int32_t& x) {
  if (m.new_pos != nullptr) {
    const int64_t* p = m.new_pos + ((int64_t(f) * m.H + h) * m.FSEQ + t) * 3;
    pt = p[0];
    y = static_cast<int32_t>(p[1]);
    x = static_cast<int32_t>(p[2]);
  } else {
    pt = (m.t_dev != nullptr ? __ldg(m.t_dev) : m.first_t) + f;
    y = t / m.pos_width;
    x = t % m.pos_width;
  }
}

// dynamic smem: gid[2][FSEQ] int16, list[2][FSEQ] int16, off[2][G+1] int32,
// tpg[2][G] float
__global__ void __launch_bounds__(kMergeThreads) merge_kernel(MergeLaunch m) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int FSEQ = m.FSEQ;
  int16_t* gid_s = reinterpret_cast<int16_t*>(smem);                 // [2][FSEQ]
  int16_t* list_s = gid_s + 2 * FSEQ;                                // [2][FSEQ]
  int32_t* off_s = reinterpret_cast<int32_t*>(
      smem + ((4 * FSEQ * sizeof(int16_t) + 15) & ~size_t(15)));     // [2][G+1]
  float* tpg_s = reinterpret_cast<float*>(off_s + 2 * (kGroupsPerCta + 1));  // [2][G]
  __shared__ SlotCache cache[kMaxMergeActive];
  __shared__ int red_x, red_y;
  __shared__ int run_s[kGroupsPerCta];

  const int h = blockIdx.x;
  const int g0 = blockIdx.y * kGroupsPerCta;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool leader_cta = blockIdx.y == 0;
  if (tid < kMaxMergeActive) cache[tid].valid = 0;
  const int32_t bf = m.states[h].block_frames;
  const int32_t ps = m.states[h].patch_size;
  const int MMA = m.MMA, MTPA = m.MTPA, D = m.D;
  __syncthreads();

  for (int f = 0; f < m.F; ++f) {
    const int di = h * m.F + f;
    const int32_t kind = m.dkind[di], a = m.dslot[di], fresh = m.dnew[di], fin = m.dfin[di];
    if (kind != kDstMergeAccum || a < 0) continue;  // uniform across the CTA
    if (a >= MMA || fin >= m.MMB) {
      if (tid == 0 && leader_cta) flag(m.status, PKV_ST_SLOT_RANGE);
      continue;
    }
    const int64_t arow = (int64_t(h) * MMA + a) * MTPA;  // first accumulator row of slot
    int16_t* gid = gid_s + a * FSEQ;
    int16_t* list = list_s + a * FSEQ;
    int32_t* off = off_s + a * (kGroupsPerCta + 1);
    float* tpg = tpg_s + a * kGroupsPerCta;

    if (fresh) {
      // ---- new block: spatial grid of this frame ----------------------------
      if (tid == 0) { red_x = -1; red_y = -1; }
      __syncthreads();
      int mx = -1, my = -1;
      for (int t = tid; t < FSEQ; t += kMergeThreads) {
        int64_t pt; int32_t y, x;
        pos_of(m, f, h, t, pt, y, x);
        mx = max(mx, x);
        my = max(my, y);
      }
      for (int o = 16; o > 0; o >>= 1) {
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        my = max(my, __shfl_xor_sync(0xffffffffu, my, o));
      }
      if (lane == 0) { atomicMax(&red_x, mx); atomicMax(&red_y, my); }
      __syncthreads();
      const int32_t pc = (red_x >= 0 && ps > 0) ? (red_x / ps + 1) : 1;
      const int32_t pr = (red_y >= 0 && ps > 0) ? (red_y / ps + 1) : 1;
      const int32_t ng = pr * pc;
      const int32_t sng = ng > MTPA ? MTPA : ng;
      for (int t = tid; t < FSEQ; t += kMergeThreads) {
        int64_t pt; int32_t y, x;
        pos_of(m, f, h, t, pt, y, x);
        const int32_t py = ps > 0 ? y / ps : 0, px = ps > 0 ? x / ps : 0;
        int32_t g = py * pc + px;
        if (g < 0 || g >= sng) g = 0;
        gid[t] = static_cast<int16_t>(g);
      }
      if (tid == 0) cache[a].num_groups = sng;
      __syncthreads();
      if (leader_cta) {
        // group bookkeeping visible to later launches and to the accessors
        int32_t* ggid = m.acc_gid + (int64_t(h) * MMA + a) * FSEQ;
        for (int t = tid; t < FSEQ; t += kMergeThreads) ggid[t] = gid[t];
        int64_t pt0; int32_t y0, x0;
        pos_of(m, f, h, 0, pt0, y0, x0);
        int64_t* gpos = m.acc_pos + arow * 3;
        for (int g = tid; g < sng; g += kMergeThreads) {
          gpos[g * 3 + 0] = pt0;
          gpos[g * 3 + 1] = (g / pc) * ps;
          gpos[g * 3 + 2] = (g % pc) * ps;
        }
        if (tid == 0) m.acc_ng[h * MMA + a] = sng;
      }
      cache[a].valid = 2;  // list below must be rebuilt
    } else if (cache[a].valid == 0) {
      // continuing a block begun in an earlier launch: group ids from global
      const int32_t* ggid = m.acc_gid + (int64_t(h) * MMA + a) * FSEQ;
      for (int t = tid; t < FSEQ; t += kMergeThreads) gid[t] = static_cast<int16_t>(ggid[t]);
      if (tid == 0) cache[a].num_groups = m.acc_ng[h * MMA + a];
      __syncthreads();
      cache[a].valid = 2;
    }
    __syncthreads();

    if (cache[a].valid == 2) {
      // ---- token lists of this CTA's groups, ascending token order ----------
      if (tid < kGroupsPerCta) run_s[tid] = 0;
      __syncthreads();
      for (int t = tid; t < FSEQ; t += kMergeThreads) {
        const int g = gid[t] - g0;
        if (g >= 0 && g < kGroupsPerCta) atomicAdd(&run_s[g], 1);
      }
      __syncthreads();
      if (tid == 0) {
        int acc = 0;
        for (int g = 0; g < kGroupsPerCta; ++g) {
          off[g] = acc;
          acc += run_s[g];
          run_s[g] = 0;
        }
        off[kGroupsPerCta] = acc;
      }
      __syncthreads();
      if (warp == 0) {
        for (int base = 0; base < FSEQ; base += 32) {
          const int t = base + lane;
          const int g = t < FSEQ ? gid[t] - g0 : -1;
          const bool mine = g >= 0 && g < kGroupsPerCta;
          const unsigned same = __match_any_sync(0xffffffffu, mine ? g : -1 - lane);
          if (mine) {
            const int rank = __popc(same & ((1u << lane) - 1u));
            list[off[g] + run_s[g] + rank] = static_cast<int16_t>(t);
          }
          __syncwarp();
          if (mine && (same & ((1u << lane) - 1u)) == 0) run_s[g] += __popc(same);
          __syncwarp();
        }
      }
      __syncthreads();
      // divisor of each group = token count * block_frames
      if (tid < kGroupsPerCta)
        tpg[tid] = static_cast<float>(off[tid + 1] - off[tid]) * static_cast<float>(bf);
      if (fresh && tid < kGroupsPerCta && g0 + tid < MTPA) {
        // each CTA owns the divisor entries of its own groups (zero past ng)
        m.acc_tpg[arow + g0 + tid] = (g0 + tid < cache[a].num_groups) ? tpg[tid] : 0.0f;
      }
      if (tid == 0) cache[a].valid = 1;
      __syncthreads();
    }

    // ---- accumulate (and finalize) every group of the tile -----------------
    const int ng = cache[a].num_groups;
    const uint16_t* kbase = m.new_k + int64_t(f) * m.frame_stride + int64_t(h) * m.head_stride;
    const uint16_t* vbase = m.new_v + int64_t(f) * m.frame_stride + int64_t(h) * m.head_stride;
    // head_dim 128 with 8-byte aligned rows: lane owns dims 4*lane..4*lane+3,
    // and a group's token rows are loaded 8 at a time before they are added
    // in list order (the adds stay sequential per element, as the reference's)
    const bool vec4 = D == 128 && (m.tok_stride & 3) == 0 &&
                      ((reinterpret_cast<uintptr_t>(kbase) | reinterpret_cast<uintptr_t>(vbase)) & 7) == 0;
    for (int gl = warp; gl < kGroupsPerCta; gl += kMergeThreads / 32) {
      const int g = g0 + gl;
      if (g >= MTPA) break;
      const int lo = off[gl], hi = off[gl + 1];
      float* ak = m.acc_k + (arow + g) * D;
      float* av = m.acc_v + (arow + g) * D;
      const float divisor = tpg[gl];
      const float inv = divisor > 0.0f ? __frcp_rn(divisor) : 0.0f;
      const int64_t prow = (int64_t(h) * m.MMB + fin) * MTPA + g;
      if (vec4) {
        const int d0 = lane * 4;
        float sk[4], sv[4];
        if (fresh) {
#pragma unroll
          for (int e = 0; e < 4; ++e) sk[e] = sv[e] = 0.0f;
        } else {
          const float4 k4 = *reinterpret_cast<const float4*>(ak + d0);
          const float4 v4 = *reinterpret_cast<const float4*>(av + d0);
          sk[0] = k4.x; sk[1] = k4.y; sk[2] = k4.z; sk[3] = k4.w;
          sv[0] = v4.x; sv[1] = v4.y; sv[2] = v4.z; sv[3] = v4.w;
        }
        for (int i0 = lo; i0 < hi; i0 += 8) {
          uint2 kr[8], vr[8];
#pragma unroll
          for (int b = 0; b < 8; ++b) {
            if (i0 + b < hi) {
              const int64_t t = list[i0 + b];
              kr[b] = *reinterpret_cast<const uint2*>(kbase + t * m.tok_stride + d0);
              vr[b] = *reinterpret_cast<const uint2*>(vbase + t * m.tok_stride + d0);
            }
          }
#pragma unroll
          for (int b = 0; b < 8; ++b) {
            if (i0 + b < hi) {
              const uint32_t kw[2] = {kr[b].x, kr[b].y}, vw[2] = {vr[b].x, vr[b].y};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const uint32_t kb = (e & 1) ? (kw[e >> 1] >> 16) : (kw[e >> 1] & 0xffffu);
                const uint32_t vb = (e & 1) ? (vw[e >> 1] >> 16) : (vw[e >> 1] & 0xffffu);
                sk[e] = __fadd_rn(sk[e], bf16_bits_to_f32(kb));
                sv[e] = __fadd_rn(sv[e], bf16_bits_to_f32(vb));
              }
            }
          }
        }
        *reinterpret_cast<float4*>(ak + d0) = make_float4(sk[0], sk[1], sk[2], sk[3]);
        *reinterpret_cast<float4*>(av + d0) = make_float4(sv[0], sv[1], sv[2], sv[3]);
        if (fin >= 0 && g < ng) {
          uint2 ok, ov;
          ok.x = f32_to_bf16_bits(__fmul_rn(sk[0], inv)) | (f32_to_bf16_bits(__fmul_rn(sk[1], inv)) << 16);
          ok.y = f32_to_bf16_bits(__fmul_rn(sk[2], inv)) | (f32_to_bf16_bits(__fmul_rn(sk[3], inv)) << 16);
          ov.x = f32_to_bf16_bits(__fmul_rn(sv[0], inv)) | (f32_to_bf16_bits(__fmul_rn(sv[1], inv)) << 16);
          ov.y = f32_to_bf16_bits(__fmul_rn(sv[2], inv)) | (f32_to_bf16_bits(__fmul_rn(sv[3], inv)) << 16);
          *reinterpret_cast<uint2*>(m.mk + prow * D + d0) = ok;
          *reinterpret_cast<uint2*>(m.mv + prow * D + d0) = ov;
        }
        continue;
      }
      for (int d = lane; d < D; d += 32) {
        float sk = fresh ? 0.0f : ak[d];
        float sv = fresh ? 0.0f : av[d];
        for (int i = lo; i < hi; ++i) {
          const int64_t t = list[i];
          sk = __fadd_rn(sk, bf16_bits_to_f32(kbase[t * m.tok_stride + d]));
          sv = __fadd_rn(sv, bf16_bits_to_f32(vbase[t * m.tok_stride + d]));
        }
        ak[d] = sk;
        av[d] = sv;
        if (fin >= 0 && g < ng) {
          m.mk[prow * D + d] = static_cast<uint16_t>(f32_to_bf16_bits(__fmul_rn(sk, inv)));
          m.mv[prow * D + d] = static_cast<uint16_t>(f32_to_bf16_bits(__fmul_rn(sv, inv)));
        }
      }
    }
    if (fin >= 0 && leader_cta) {
      // group positions were recorded at block start (possibly by this CTA
      // earlier in this launch: same-CTA global writes are visible after the
      // barrier above)
      const int64_t* gpos = m.acc_pos + arow * 3;
      int64_t* ppos = m.mpos + (int64_t(h) * m.MMB + fin) * MTPA * 3;
      for (int e = tid; e < ng * 3; e += kMergeThreads) ppos[e] = gpos[e];
      if (tid == 0) m.mtc[h * m.MMB + fin] = ng;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// merge_grid_kernel: the same accumulation when token positions come from the
// frame grid (t -> y = t / W, x = t % W; the MegaCache path).  A group's
// tokens are then a closed form: rows py*ps .. py*ps+ps-1, columns
// px*ps .. px*ps+ps-1 of the grid, enumerated row by row, which is ascending
// token order; no per-launch token lists.  One warp owns one group of one
// head for the whole launch and keeps its fp32 sums in registers across the
// frames (lane = 4 dims of head_dim 128), flushing them to the accumulator
// rows when the frame's slot changes and at the end.  Heads whose grid does
// not fit the closed form (patch size <= 0, or more groups than MTPA, where
// the reference folds the excess tokens into group 0) take a warp-wide scan
// of the frame's tokens, still in ascending order.
// ---------------------------------------------------------------------------
constexpr int kGridGroupsPerCta = 8;  // one warp per group
constexpr int kGridThreads = kGridGroupsPerCta * 32;

struct MergeGrid {
  int W, pc, sng, ps;
  bool closed;
  __device__ __forceinline__ int gid(int t) const {
    const int y = t / W, x = t - y * W;
    int g = ps > 0 ? (y / ps) * pc + x / ps : 0;
    return (g < 0 || g >= sng) ? 0 : g;
  }
};

// Token i (< ps * ps) of group g in the closed form, or -1 outside the frame.
__device__ __forceinline__ int grid_token(const MergeGrid& G, int FSEQ, int g, int i) {
  const int py = g / G.pc, px = g - py * G.pc;
  const int dy = i / G.ps, dx = i - dy * G.ps;
  const int y = py * G.ps + dy, x = px * G.ps + dx;
  if (x >= G.W) return -1;
  const int t = y * G.W + x;
  return t < FSEQ ? t : -1;
}

__device__ __forceinline__ void add_row(float (&sk)[4], float (&sv)[4], uint2 kr, uint2 vr) {
  const uint32_t kw[2] = {kr.x, kr.y}, vw[2] = {vr.x, vr.y};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t kb = (e & 1) ? (kw[e >> 1] >> 16) : (kw[e >> 1] & 0xffffu);
    const uint32_t vb = (e & 1) ? (vw[e >> 1] >> 16) : (vw[e >> 1] & 0xffffu);
    sk[e] = __fadd_rn(sk[e], bf16_bits_to_f32(kb));
    sv[e] = __fadd_rn(sv[e], bf16_bits_to_f32(vb));
  }
}

__device__ __forceinline__ void store_acc(const MergeLaunch& m, int64_t row, int d0,
                                          const float (&sk)[4], const float (&sv)[4]) {
  *reinterpret_cast<float4*>(m.acc_k + row * 128 + d0) = make_float4(sk[0], sk[1], sk[2], sk[3]);
  *reinterpret_cast<float4*>(m.acc_v + row * 128 + d0) = make_float4(sv[0], sv[1], sv[2], sv[3]);
}

constexpr int kMergeBatch = 3;     // frames whose rows are loaded together (a block's 3)
constexpr int kMergeBatchTok = 4;  // tokens per group in the prefetched form (patch 2 x 2)

__global__ void __launch_bounds__(kGridThreads, 2) merge_grid_kernel(MergeLaunch m) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, tile = blockIdx.y;
  const int g = tile * kGridGroupsPerCta + warp;
  const int FSEQ = m.FSEQ, MMA = m.MMA, MTPA = m.MTPA;
  const int32_t bf = m.states[h].block_frames;
  MergeGrid G;
  G.W = m.pos_width;
  G.ps = m.states[h].patch_size;
  // the frame's spatial extent: max x and max y over its tokens
  const int mx = (G.W < FSEQ ? G.W : FSEQ) - 1, my = (FSEQ - 1) / G.W;
  G.pc = G.ps > 0 ? mx / G.ps + 1 : 1;
  const int pr = G.ps > 0 ? my / G.ps + 1 : 1;
  const int ng = pr * G.pc;
  G.sng = ng > MTPA ? MTPA : ng;
  G.closed = G.ps > 0 && ng <= MTPA;
  const int d0 = lane * 4;
  // the group's tokens are the same in every frame: with at most 4 of them
  // (patch 2 x 2) a batch of frames' rows is loaded at once
  const bool pre = G.closed && G.ps * G.ps <= kMergeBatchTok && g < MTPA;
  int tt[kMergeBatchTok];
  int ntok = 0;
#pragma unroll
  for (int i = 0; i < kMergeBatchTok; ++i) {
    tt[i] = pre && i < G.ps * G.ps ? grid_token(G, FSEQ, g, i) : -1;
    ntok += tt[i] >= 0;
  }
  int cur = -1;  // accumulator slot whose sums the registers hold
  float sk[4] = {0.f, 0.f, 0.f, 0.f}, sv[4] = {0.f, 0.f, 0.f, 0.f};
  for (int f0 = 0; f0 < m.F; f0 += kMergeBatch) {
    // ---- this batch's descriptors, then (prefetched form) its rows
    int32_t kind[kMergeBatch], slot[kMergeBatch], fresh[kMergeBatch], fin[kMergeBatch];
#pragma unroll
    for (int b = 0; b < kMergeBatch; ++b) {
      kind[b] = -1;
      slot[b] = fresh[b] = 0;
      fin[b] = -1;
      if (f0 + b < m.F) {
        const int di = h * m.F + f0 + b;
        kind[b] = m.dkind[di];
        slot[b] = m.dslot[di];
        fresh[b] = m.dnew[di];
        fin[b] = m.dfin[di];
      }
    }
    uint2 kr[kMergeBatch][kMergeBatchTok], vr[kMergeBatch][kMergeBatchTok];
    float4 pk = make_float4(0.f, 0.f, 0.f, 0.f), pv = pk;
    int pslot = -1;  // slot whose accumulator rows pk / pv hold
    if (pre) {
#pragma unroll
      for (int b = 0; b < kMergeBatch; ++b) {
        if (kind[b] != kDstMergeAccum || slot[b] < 0 || slot[b] >= MMA) continue;
        const int64_t fo = int64_t(f0 + b) * m.frame_stride + int64_t(h) * m.head_stride;
#pragma unroll
        for (int i = 0; i < kMergeBatchTok; ++i) {
          if (tt[i] < 0) continue;
          kr[b][i] = *reinterpret_cast<const uint2*>(m.new_k + fo + int64_t(tt[i]) * m.tok_stride + d0);
          vr[b][i] = *reinterpret_cast<const uint2*>(m.new_v + fo + int64_t(tt[i]) * m.tok_stride + d0);
        }
      }
      // the first merge frame's accumulator rows, when it continues a block
#pragma unroll
      for (int b = kMergeBatch - 1; b >= 0; --b) {
        if (kind[b] == kDstMergeAccum && slot[b] >= 0 && slot[b] < MMA) pslot = fresh[b] ? -1 : slot[b];
      }
      if (pslot >= 0 && pslot != cur) {
        const int64_t row = (int64_t(h) * MMA + pslot) * MTPA + g;
        pk = *reinterpret_cast<const float4*>(m.acc_k + row * 128 + d0);
        pv = *reinterpret_cast<const float4*>(m.acc_v + row * 128 + d0);
      }
    }
#pragma unroll
    for (int b = 0; b < kMergeBatch; ++b) {
      const int f = f0 + b;
      const int32_t a = slot[b];
      if (kind[b] != kDstMergeAccum || a < 0) continue;  // uniform across the CTA
      if (a >= MMA || fin[b] >= m.MMB) {
        if (threadIdx.x == 0 && tile == 0) flag(m.status, PKV_ST_SLOT_RANGE);
        continue;
      }
      const int64_t arow = (int64_t(h) * MMA + a) * MTPA;
      if (fresh[b]) {
        // new block: group bookkeeping visible to later launches and the accessors
        if (tile == 0) {
          int32_t* ggid = m.acc_gid + (int64_t(h) * MMA + a) * FSEQ;
          for (int t = threadIdx.x; t < FSEQ; t += kGridThreads) ggid[t] = G.gid(t);
          if (threadIdx.x == 0) m.acc_ng[h * MMA + a] = G.sng;
        }
        if (g < G.sng && lane == 0) {
          const int64_t pt0 = (m.t_dev != nullptr ? __ldg(m.t_dev) : m.first_t) + f;
          int64_t* gp = m.acc_pos + (arow + g) * 3;
          gp[0] = pt0;
          gp[1] = int64_t(g / G.pc) * G.ps;
          gp[2] = int64_t(g % G.pc) * G.ps;
        }
      }
      if (g >= MTPA) continue;  // warp-uniform
      if (a != cur) {
        if (cur >= 0) {
          store_acc(m, (int64_t(h) * MMA + cur) * MTPA + g, d0, sk, sv);
          if (cur == pslot) pslot = -1;  // the prefetched rows are stale now
        }
        cur = a;
        if (fresh[b]) {
#pragma unroll
          for (int e = 0; e < 4; ++e) sk[e] = sv[e] = 0.0f;
        } else {
          float4 k4 = pk, v4 = pv;
          if (a != pslot) {
            k4 = *reinterpret_cast<const float4*>(m.acc_k + (arow + g) * 128 + d0);
            v4 = *reinterpret_cast<const float4*>(m.acc_v + (arow + g) * 128 + d0);
          }
          sk[0] = k4.x; sk[1] = k4.y; sk[2] = k4.z; sk[3] = k4.w;
          sv[0] = v4.x; sv[1] = v4.y; sv[2] = v4.z; sv[3] = v4.w;
        }
      } else if (fresh[b]) {
#pragma unroll
        for (int e = 0; e < 4; ++e) sk[e] = sv[e] = 0.0f;
      }
      int count = 0;  // the group's tokens in this frame
      if (pre) {
#pragma unroll
        for (int i = 0; i < kMergeBatchTok; ++i)
          if (tt[i] >= 0) add_row(sk, sv, kr[b][i], vr[b][i]);
        count = ntok;
      } else {
        const uint16_t* kbase = m.new_k + int64_t(f) * m.frame_stride + int64_t(h) * m.head_stride;
        const uint16_t* vbase = m.new_v + int64_t(f) * m.frame_stride + int64_t(h) * m.head_stride;
        if (G.closed) {
          const int n = G.ps * G.ps;
          for (int i0 = 0; i0 < n; i0 += 8) {
            uint2 kb[8], vb[8];
            int tb[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              tb[j] = i0 + j < n ? grid_token(G, FSEQ, g, i0 + j) : -1;
              if (tb[j] >= 0) {
                kb[j] = *reinterpret_cast<const uint2*>(kbase + int64_t(tb[j]) * m.tok_stride + d0);
                vb[j] = *reinterpret_cast<const uint2*>(vbase + int64_t(tb[j]) * m.tok_stride + d0);
              }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if (tb[j] >= 0) {
                add_row(sk, sv, kb[j], vb[j]);
                ++count;
              }
            }
          }
        } else if (g < G.sng) {
          for (int base = 0; base < FSEQ; base += 32) {
            const int t = base + lane;
            unsigned mine = __ballot_sync(0xffffffffu, t < FSEQ && G.gid(t) == g);
            count += __popc(mine);
            while (mine) {
              const int tk = base + __ffs(mine) - 1;
              mine &= mine - 1;
              const uint2 kx = *reinterpret_cast<const uint2*>(kbase + int64_t(tk) * m.tok_stride + d0);
              const uint2 vx = *reinterpret_cast<const uint2*>(vbase + int64_t(tk) * m.tok_stride + d0);
              add_row(sk, sv, kx, vx);
            }
          }
        }
      }
      if (fresh[b] && lane == 0)  // divisor = token count * block_frames (zero past the groups)
        m.acc_tpg[arow + g] = g < G.sng ? static_cast<float>(count) * static_cast<float>(bf) : 0.0f;
      if (fin[b] >= 0 && g < G.sng) {
        // every frame of a block has the same grid, so this frame's count gives
        // the block's divisor
        const float divisor = static_cast<float>(count) * static_cast<float>(bf);
        const float inv = divisor > 0.0f ? __frcp_rn(divisor) : 0.0f;
        const int64_t prow = (int64_t(h) * m.MMB + fin[b]) * MTPA + g;
        uint2 ok, ov;
        ok.x = f32_to_bf16_bits(__fmul_rn(sk[0], inv)) | (f32_to_bf16_bits(__fmul_rn(sk[1], inv)) << 16);
        ok.y = f32_to_bf16_bits(__fmul_rn(sk[2], inv)) | (f32_to_bf16_bits(__fmul_rn(sk[3], inv)) << 16);
        ov.x = f32_to_bf16_bits(__fmul_rn(sv[0], inv)) | (f32_to_bf16_bits(__fmul_rn(sv[1], inv)) << 16);
        ov.y = f32_to_bf16_bits(__fmul_rn(sv[2], inv)) | (f32_to_bf16_bits(__fmul_rn(sv[3], inv)) << 16);
        *reinterpret_cast<uint2*>(m.mk + prow * 128 + d0) = ok;
        *reinterpret_cast<uint2*>(m.mv + prow * 128 + d0) = ov;
        __syncwarp();  // lane 0's group position of a block begun in this launch
        if (lane < 3) m.mpos[prow * 3 + lane] = m.acc_pos[(arow + g) * 3 + lane];
        if (g == 0 && lane == 0) m.mtc[h * m.MMB + fin[b]] = G.sng;
      }
    }
  }
  if (cur >= 0 && g < MTPA) store_acc(m, (int64_t(h) * MMA + cur) * MTPA + g, d0, sk, sv);
}

int launch_merge(const MergeLaunch& m, cudaStream_t stream) {
  if (m.H == 0 || m.F == 0) return PKV_OK;
  if (m.FSEQ <= 0 || m.FSEQ > 16384 || m.MTPA <= 0 || m.MTPA > 32767 || m.D <= 0)
    return PKV_EUNSUPPORTED;
  const size_t smem = ((4 * size_t(m.FSEQ) * sizeof(int16_t) + 15) & ~size_t(15)) +
                      2 * (kGroupsPerCta + 1) * sizeof(int32_t) +
                      2 * kGroupsPerCta * sizeof(float);
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(smem)) != cudaSuccess)
      return PKV_ELAUNCH;
  }
  // positions from the frame grid, head_dim 128 with 8-byte aligned rows:
  // warp per group with the closed-form token lists
  const bool grid_ok =
      m.new_pos == nullptr && m.pos_width > 0 && m.D == 128 && (m.tok_stride & 3) == 0 &&
      (m.frame_stride & 3) == 0 && (m.head_stride & 3) == 0 &&
      ((reinterpret_cast<uintptr_t>(m.new_k) | reinterpret_cast<uintptr_t>(m.new_v)) & 7) == 0 &&
      ((reinterpret_cast<uintptr_t>(m.acc_k) | reinterpret_cast<uintptr_t>(m.acc_v)) & 15) == 0 &&
      ((reinterpret_cast<uintptr_t>(m.mk) | reinterpret_cast<uintptr_t>(m.mv)) & 7) == 0;
  if (grid_ok) {
    dim3 grid(m.H, (m.MTPA + kGridGroupsPerCta - 1) / kGridGroupsPerCta);
    merge_grid_kernel<<<grid, kGridThreads, 0, stream>>>(m);
    return launch_status();
  }
  dim3 grid(m.H, (m.MTPA + kGroupsPerCta - 1) / kGroupsPerCta);
  merge_kernel<<<grid, kMergeThreads, smem, stream>>>(m);
  return launch_status();
}

}  // namespace pkv

using namespace pkv;

extern "C" int pkv_merge_accum(const uint8_t* states, const uint16_t* new_k,
                               const uint16_t* new_v, const int64_t* new_pos,
                               const int32_t* desc_dst_kind, const int32_t* desc_merge_accum_slot,
                               const int32_t* desc_merge_finalize_completed_idx,
                               const int32_t* desc_merge_is_new_block, float* accum_sum_k,
                               float* accum_sum_v, int64_t* accum_pos, int32_t* accum_group_ids,
                               float* accum_tokens_per_group, int32_t* accum_num_groups,
                               uint16_t* merge_k_pool, uint16_t* merge_v_pool,
                               int64_t* merge_pos_pool, int32_t* merge_token_count, int H, int F,
                               int FSEQ, int D, int MMA, int MMB, int MTPA, int32_t* status,
                               pkv_stream_t stream) {
  if (H == 0 || F == 0) return PKV_OK;
  if (!states || !new_k || !new_v || !new_pos || !desc_dst_kind || !desc_merge_accum_slot ||
      !desc_merge_finalize_completed_idx || !desc_merge_is_new_block || !accum_sum_k ||
      !accum_sum_v || !accum_pos || !accum_group_ids || !accum_tokens_per_group ||
      !accum_num_groups || !merge_k_pool || !merge_v_pool || !merge_pos_pool ||
      !merge_token_count || H < 0 || F < 0)
    return PKV_EINVAL;
  MergeLaunch m{};
  m.states = reinterpret_cast<const HeadState*>(states);
  m.new_k = new_k;
  m.new_v = new_v;
  m.frame_stride = int64_t(H) * FSEQ * D;
  m.head_stride = int64_t(FSEQ) * D;
  m.tok_stride = D;
  m.new_pos = new_pos;
  m.pos_width = 1;
  m.first_t = 0;
  m.t_dev = nullptr;
  m.dkind = desc_dst_kind;
  m.dslot = desc_merge_accum_slot;
  m.dfin = desc_merge_finalize_completed_idx;
  m.dnew = desc_merge_is_new_block;
  m.acc_k = accum_sum_k;
  m.acc_v = accum_sum_v;
  m.acc_pos = accum_pos;
  m.acc_gid = accum_group_ids;
  m.acc_tpg = accum_tokens_per_group;
  m.acc_ng = accum_num_groups;
  m.mk = merge_k_pool;
  m.mv = merge_v_pool;
  m.mpos = merge_pos_pool;
  m.mtc = merge_token_count;
  m.H = H;
  m.F = F;
  m.FSEQ = FSEQ;
  m.D = D;
  m.MMA = MMA;
  m.MMB = MMB;
  m.MTPA = MTPA;
  m.status = status;
  return launch_merge(m, static_cast<cudaStream_t>(stream));
}
