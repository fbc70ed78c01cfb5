// Device planner: the ragged K/V layout of one layer's attention call.
//
// Reference behaviour: pyramidkv/csrc/mega_plan.cc:133-264 (emit_chunk_plan),
// :510-654 (mega_plan_multi) and :63-80 (map_sink_time).  For every query
// chunk c and head h the planner lists the frames (segments) the head's
// queries attend, in this order:
//   sink slots     s < min(valid sink, sink_capacity)   t_remap = sync_t
//   recent slots   r < valid recent                     t_remap = -1 (stored t)
//   cyclic slots   of phase current_t % period, skipping t < sink_capacity,
//                  t_remap = sync_t
//   stride / lag   tkey slots in ring-slot order, skipping t < sink_capacity,
//                  t_remap = sync_t (stride) / -1 (lag)
//   merge anchors  finalized blocks with start_t > 0 and a token count,
//                  length = token count, t_remap = median t
// with sync_t = map_sink_time(current_t) and a running token offset; the
// reference's quirks (recent dedup disabled, merge slot aliasing after FIFO
// eviction, block 0 never emitted) are kept because the packed layout must be
// bit-identical.
//
// B200 design: the reference pulls valid_count, merge_token_count and the
// states to the host (3 blocking D2H copies) and pushes 7 descriptor arrays
// back (7 H2D copies) on every call, which also blocks CUDA-graph capture.
// Here one CTA does the whole plan in device memory.  The layer's state
// records, valid counts and merge token counts are staged in shared memory
// by all threads; then one warp per (chunk, head) evaluates the head's
// candidate segments in parallel (lane = candidate: sink slot, recent slot,
// cyclic / tkey slot, merge block, in the reference's order), places the
// valid ones with a ballot prefix count and their token offsets with a warp
// scan; a block-wide scan of the (chunk, head) totals gives cu_seqlens_k, and
// every lane writes its descriptor (or the reference's padding) in place.
// Shapes beyond the candidate list's compiled bounds take plan_kernel, where
// thread (c, h) walks its segments twice around a block-wide scan.  The
// capacity check becomes a status bit the pack kernel also honours, so an
// overflowing plan never writes out of bounds.
#include "pkv_common.cuh"

namespace pkv {

struct PlanArgs {
  const int64_t* vc;        // [L,H,3]
  const int32_t* mtc;       // [L,H,MMB]
  const HeadState* states;  // this layer's H records
  int layer, H, F, max_sink, max_middle, max_recent, mmb, S, C;
  int sink_mode, cmin, cmax, lag;
  int add_layer_offset, check_capacity;
  int64_t capacity;
  int64_t t[PKV_MAX_CHUNKS];
  const int64_t* t_dev;  // device time of chunk 0 (nullable): chunk c at *t_dev + c
  int32_t *cu, *sk, *sg, *sl, *dst;
  int64_t *traw, *tremap;
  int64_t *total_out, *counter;
  int32_t* status;
};

__device__ __forceinline__ int64_t map_sink_time(int64_t t, int mode, int cmin, int cmax,
                                                 int lag) {
  if (mode == 1) {
    int64_t delta = t;
    if (delta < cmin) delta = cmin;
    if (delta > cmax) delta = cmax;
    const int64_t out = t - delta;
    return out < 0 ? 0 : out;
  }
  const int64_t out = t - lag;
  return out < 0 ? 0 : out;
}

// Calls emit(kind, slot_in_layer, len, t_raw, t_remap) for every segment of
// (chunk c, head h) in the reference's order; returns the segment count.
// Time of chunk c: from the launch parameters, or chunk 0's time read from
// device memory when the caller keeps it there (graph replay across blocks).
__device__ __forceinline__ int64_t chunk_time(const PlanArgs& a, int c) {
  return a.t_dev != nullptr ? __ldg(a.t_dev) + c : a.t[c];
}

template <class Emit>
__device__ int walk_segments(const PlanArgs& a, int c, int h, Emit&& emit) {
  const HeadState& s = a.states[h];
  const int64_t ct = chunk_time(a, c);
  const int64_t sync_t = map_sink_time(ct, a.sink_mode, a.cmin, a.cmax, a.lag);
  const int thr = s.sink_capacity;
  const int64_t* vch = a.vc + (int64_t(a.layer) * a.H + h) * 3;
  int fp = 0;
  const int nsr = static_cast<int>(vch[0]);
  const int ns = (thr > 0 && thr < nsr) ? thr : nsr;
  for (int k = 0; k < ns && k < a.max_sink; ++k, ++fp)
    emit(fp, kDstSink, h * a.max_sink + k, a.F, int64_t(k), sync_t);
  const int nr = static_cast<int>(vch[2]);
  for (int k = 0; k < nr && k < a.max_recent; ++k, ++fp)
    emit(fp, kDstRecent, h * a.max_recent + k, a.F, int64_t(-1), int64_t(-1));
  if (s.kind == kCyclic) {
    const int period = s.period > 0 ? s.period : 1;
    const int bcap = s.bucket_cap > 0 ? s.bucket_cap : 1;
    const int phase = static_cast<int>(((ct % period) + period) % period);
    const int pb = phase * kMaxBucket;
    const int pe = pb + (bcap < kMaxBucket ? bcap : kMaxBucket);
    for (int i = pb; i < pe && i < kMaxPhase * kMaxBucket; ++i) {
      if (s.cyclic_slot[i] < 0) continue;
      if (s.cyclic_t[i] < thr) continue;
      emit(fp, kDstMiddle, h * a.max_middle + i, a.F, int64_t(s.cyclic_t[i]), sync_t);
      ++fp;
      if (fp >= a.S) break;
    }
  } else if (s.kind == kStride || s.kind == kLag) {
    const int tc = s.tkey_count;
    for (int i = 0; i < tc && i < kMaxTKeyed; ++i) {
      if (s.tkey_t[i] < thr) continue;
      emit(fp, kDstMiddle, h * a.max_middle + i, a.F, int64_t(s.tkey_t[i]),
           s.kind == kStride ? sync_t : int64_t(-1));
      ++fp;
      if (fp >= a.S) break;
    }
  }
  if (s.kind == kMerge) {
    const int mcc = s.done_count;
    for (int i = 0; i < mcc && i < kMaxMergeBlocks; ++i) {
      const int bs = s.done_slot[i];
      if (bs < 0 || bs >= a.mmb) continue;
      if (s.done_start_t[i] <= 0) continue;
      const int32_t tok = a.mtc[(int64_t(a.layer) * a.H + h) * a.mmb + bs];
      if (tok <= 0) continue;
      if (fp >= a.S) break;
      emit(fp, kSrcMerge, h * a.mmb + bs, tok, int64_t(0), int64_t(s.done_median_t[i]));
      ++fp;
    }
  }
  return fp;
}

__global__ void plan_kernel(PlanArgs a) {
  __shared__ int64_t warp_sums[32];
  const int i = threadIdx.x;  // = c*H + h
  const int n = a.C * a.H;
  const bool active = i < n;
  const int c = active ? i / a.H : 0;
  const int h = active ? i - c * a.H : 0;

  // pass 1: token count of (c, h)
  int64_t mine = 0;
  if (active) {
    walk_segments(a, c, h, [&](int, int, int, int len, int64_t, int64_t) { mine += len; });
  }
  // block-wide inclusive scan of the counts (c-major, h-minor = reference order)
  const int lane = i & 31, warp = i >> 5;
  int64_t x = mine;
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) / 32;
    int64_t w = lane < nw ? warp_sums[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) warp_sums[lane] = w;  // inclusive per-warp prefix
  }
  __syncthreads();
  const int64_t incl = x + (warp > 0 ? warp_sums[warp - 1] : 0);
  const int64_t excl = incl - mine;
  const int64_t total = warp_sums[(blockDim.x + 31) / 32 - 1];

  if (i == 0) {
    a.cu[0] = 0;
    if (a.total_out) *a.total_out = total;
    if (a.counter) atomicAdd(reinterpret_cast<unsigned long long*>(a.counter),
                             static_cast<unsigned long long>(total));
    if (a.check_capacity && total > a.capacity) flag(a.status, PKV_ST_PACK_OVERFLOW);
  }
  if (!active) return;
  a.cu[i + 1] = static_cast<int32_t>(incl);

  // pass 2: descriptors at their offsets, padding for the unused positions
  const int base = i * a.S;
  int64_t run = excl;
  const int slots_of[4] = {a.max_sink, a.max_middle, a.max_recent, a.mmb};
  const int used = walk_segments(
      a, c, h, [&](int fp, int kind, int slot, int len, int64_t traw, int64_t tremap) {
        const int j = base + fp;
        int32_t sg = slot;
        if (a.add_layer_offset) {
          const int ki = kind == kDstSink ? 0 : kind == kDstMiddle ? 1 : kind == kDstRecent ? 2 : 3;
          sg += a.layer * a.H * slots_of[ki];
        }
        a.sk[j] = kind;
        a.sg[j] = sg;
        a.sl[j] = len;
        a.dst[j] = static_cast<int32_t>(run);
        a.traw[j] = traw;
        a.tremap[j] = tremap;
        run += len;
      });
  for (int fp = used; fp < a.S; ++fp) {
    const int j = base + fp;
    a.sk[j] = -1;
    a.sg[j] = 0;
    a.sl[j] = 0;
    a.dst[j] = 0;
    a.traw[j] = -1;
    a.tremap[j] = -1;
  }
}

// ---------------------------------------------------------------------------
// Warp-per-(chunk, head) planner.  Candidate j of a head (j < kCand) is:
//   [0, 3)        sink slot j               valid while j < min(valid sink, cap)
//   [3, 7)        recent slot j - 3         valid while < valid recent
//   [7, 31)       middle slot j - 7         cyclic: inside the phase's buckets,
//                                           stride / lag: inside the tkey ring
//   [31, 37)      merge completed entry j - 31
// (the pools' compiled bounds: 3 sink, 4 recent, 24 middle, 6 merge slots).
// A lane's candidate is emitted at position (valid candidates before it)
// unless that position reaches S, which is where the reference walk stops.
// ---------------------------------------------------------------------------
constexpr int kPlanWarpThreads = 1024;
constexpr int kCandSink = 3, kCandRecent = 4, kCandMiddle = 24, kCandMerge = 6;
constexpr int kCand = kCandSink + kCandRecent + kCandMiddle + kCandMerge;  // 37
constexpr int kPlanMaxHeads = 64;

struct PlanSmem {
  HeadState st[kPlanMaxHeads];
  int64_t vc[kPlanMaxHeads * 3];
  int32_t mtc[kPlanMaxHeads * 8];
  int64_t pair_total[1024];  // (chunk, head) pairs: launch_plan bounds them at 1024
};

// Candidate j of (chunk c, head h): kind, slot in layer, length, t_raw,
// t_remap; false when the candidate is not a segment.
__device__ __forceinline__ bool plan_candidate(const PlanArgs& a, const PlanSmem& sm, int c,
                                               int h, int j, int& kind, int& slot, int& len,
                                               int64_t& traw, int64_t& tremap) {
  const HeadState& s = sm.st[h];
  const int64_t ct = chunk_time(a, c);
  const int64_t sync_t = map_sink_time(ct, a.sink_mode, a.cmin, a.cmax, a.lag);
  const int thr = s.sink_capacity;
  if (j < kCandSink) {
    const int nsr = static_cast<int>(sm.vc[h * 3 + 0]);
    const int ns = (thr > 0 && thr < nsr) ? thr : nsr;
    if (j >= ns || j >= a.max_sink) return false;
    kind = kDstSink;
    slot = h * a.max_sink + j;
    len = a.F;
    traw = j;
    tremap = sync_t;
    return true;
  }
  j -= kCandSink;
  if (j < kCandRecent) {
    const int nr = static_cast<int>(sm.vc[h * 3 + 2]);
    if (j >= nr || j >= a.max_recent) return false;
    kind = kDstRecent;
    slot = h * a.max_recent + j;
    len = a.F;
    traw = tremap = -1;
    return true;
  }
  j -= kCandRecent;
  if (j < kCandMiddle) {
    if (s.kind == kCyclic) {
      const int period = s.period > 0 ? s.period : 1;
      const int bcap = s.bucket_cap > 0 ? s.bucket_cap : 1;
      const int phase = static_cast<int>(((ct % period) + period) % period);
      const int pb = phase * kMaxBucket;
      const int pe = pb + (bcap < kMaxBucket ? bcap : kMaxBucket);
      if (j < pb || j >= pe || j >= kMaxPhase * kMaxBucket) return false;
      if (s.cyclic_slot[j] < 0 || s.cyclic_t[j] < thr) return false;
      kind = kDstMiddle;
      slot = h * a.max_middle + j;
      len = a.F;
      traw = s.cyclic_t[j];
      tremap = sync_t;
      return true;
    }
    if (s.kind == kStride || s.kind == kLag) {
      if (j >= s.tkey_count || j >= kMaxTKeyed) return false;
      if (s.tkey_t[j] < thr) return false;
      kind = kDstMiddle;
      slot = h * a.max_middle + j;
      len = a.F;
      traw = s.tkey_t[j];
      tremap = s.kind == kStride ? sync_t : int64_t(-1);
      return true;
    }
    return false;
  }
  j -= kCandMiddle;
  if (s.kind != kMerge || j >= s.done_count || j >= kMaxMergeBlocks) return false;
  const int bs = s.done_slot[j];
  if (bs < 0 || bs >= a.mmb || s.done_start_t[j] <= 0) return false;
  const int32_t tok = sm.mtc[h * a.mmb + bs];
  if (tok <= 0) return false;
  kind = kSrcMerge;
  slot = h * a.mmb + bs;
  len = tok;
  traw = 0;
  tremap = s.done_median_t[j];
  return true;
}

__global__ void __launch_bounds__(kPlanWarpThreads, 1) plan_warp_kernel(PlanArgs a) {
  extern __shared__ __align__(16) uint8_t plan_smem_raw[];
  PlanSmem& sm = *reinterpret_cast<PlanSmem*>(plan_smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int npair = a.C * a.H;
  // stage this layer's records, valid counts and merge token counts
  {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.states);
    uint32_t* dst = reinterpret_cast<uint32_t*>(sm.st);
    for (int i = tid; i < a.H * int(sizeof(HeadState) / 4); i += blockDim.x) dst[i] = src[i];
    const int64_t* vcl = a.vc + int64_t(a.layer) * a.H * 3;
    for (int i = tid; i < a.H * 3; i += blockDim.x) sm.vc[i] = vcl[i];
    const int32_t* ml = a.mtc + int64_t(a.layer) * a.H * a.mmb;
    for (int i = tid; i < a.H * a.mmb; i += blockDim.x) sm.mtc[i] = ml[i];
  }
  __syncthreads();
  // pass 1: each (chunk, head)'s token total
  for (int pr = warp; pr < npair; pr += nwarps) {
    const int c = pr / a.H, h = pr - c * a.H;
    int tot = 0, fp_base = 0;
    for (int j0 = 0; j0 < kCand; j0 += 32) {
      const int j = j0 + lane;
      int kind = 0, slot = 0, len = 0;
      int64_t traw = 0, tremap = 0;
      const bool v = j < kCand && plan_candidate(a, sm, c, h, j, kind, slot, len, traw, tremap);
      const uint32_t bal = __ballot_sync(0xffffffffu, v);
      const int fp = fp_base + __popc(bal & ((1u << lane) - 1u));
      tot += (v && fp < a.S) ? len : 0;
      fp_base += __popc(bal);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    if (lane == 0) sm.pair_total[pr] = tot;
  }
  __syncthreads();
  // exclusive scan of the pair totals (c-major, h-minor = reference order)
  if (warp == 0) {
    const int per = (npair + 31) / 32;
    const int p0 = min(npair, lane * per), p1 = min(npair, p0 + per);
    int64_t run = 0;
    for (int i = p0; i < p1; ++i) run += sm.pair_total[i];
    int64_t incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int64_t acc = incl - run;
    for (int i = p0; i < p1; ++i) {
      const int64_t t = sm.pair_total[i];
      sm.pair_total[i] = acc;  // now the exclusive offset
      a.cu[i + 1] = static_cast<int32_t>(acc + t);
      acc += t;
    }
    const int64_t total = __shfl_sync(0xffffffffu, incl, 31);
    if (lane == 0) {
      a.cu[0] = 0;
      if (a.total_out) *a.total_out = total;
      if (a.counter)
        atomicAdd(reinterpret_cast<unsigned long long*>(a.counter),
                  static_cast<unsigned long long>(total));
      if (a.check_capacity && total > a.capacity) flag(a.status, PKV_ST_PACK_OVERFLOW);
    }
  }
  __syncthreads();
  // pass 2: descriptors at their offsets, the reference's padding after them
  for (int pr = warp; pr < npair; pr += nwarps) {
    const int c = pr / a.H, h = pr - c * a.H;
    const int base = pr * a.S;
    int64_t run = sm.pair_total[pr];
    int fp_base = 0;
    for (int j0 = 0; j0 < kCand; j0 += 32) {
      const int j = j0 + lane;
      int kind = 0, slot = 0, len = 0;
      int64_t traw = 0, tremap = 0;
      const bool v = j < kCand && plan_candidate(a, sm, c, h, j, kind, slot, len, traw, tremap);
      const uint32_t bal = __ballot_sync(0xffffffffu, v);
      const int fp = fp_base + __popc(bal & ((1u << lane) - 1u));
      const bool emit = v && fp < a.S;
      const int off = emit ? len : 0;  // inclusive warp scan of the emitted lengths
      int incl = off;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (emit) {
        const int jj = base + fp;
        int32_t sg = slot;
        if (a.add_layer_offset) {
          const int per_head = kind == kDstSink     ? a.max_sink
                               : kind == kDstMiddle ? a.max_middle
                               : kind == kDstRecent ? a.max_recent
                                                    : a.mmb;
          sg += a.layer * a.H * per_head;
        }
        a.sk[jj] = kind;
        a.sg[jj] = sg;
        a.sl[jj] = len;
        a.dst[jj] = static_cast<int32_t>(run + incl - off);
        a.traw[jj] = traw;
        a.tremap[jj] = tremap;
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
      fp_base += __popc(bal);
    }
    const int used = fp_base < a.S ? fp_base : a.S;
    for (int fp = used + lane; fp < a.S; fp += 32) {
      const int jj = base + fp;
      a.sk[jj] = -1;
      a.sg[jj] = 0;
      a.sl[jj] = 0;
      a.dst[jj] = 0;
      a.traw[jj] = -1;
      a.tremap[jj] = -1;
    }
  }
}

int launch_plan(const pkv_cache_t* c, const uint8_t* states_layer, int layer,
                const int64_t* current_t, int num_chunks, int sink_mode, int cmin, int cmax,
                int lag, int check_capacity, int add_layer_offset, int32_t* cu, int32_t* sk,
                int32_t* sg, int32_t* sl, int32_t* dst, int64_t* traw, int64_t* tremap,
                int64_t* total, int64_t* counter, cudaStream_t stream,
                const int64_t* t_dev) {
  if (!c || !states_layer || !current_t || !cu || !sk || !sg || !sl || !dst || !traw ||
      !tremap || !c->valid_count || !c->merge_token_count)
    return PKV_EINVAL;
  if (num_chunks <= 0 || num_chunks > PKV_MAX_CHUNKS) return PKV_ECAPACITY;
  if (layer < 0 || layer >= c->num_layers) return PKV_EINVAL;
  const int n = num_chunks * c->num_heads;
  if (n > 1024) return PKV_ECAPACITY;
  PlanArgs a{};
  a.vc = c->valid_count;
  a.mtc = c->merge_token_count;
  a.states = reinterpret_cast<const HeadState*>(states_layer);
  a.layer = layer;
  a.H = c->num_heads;
  a.F = c->frame_seqlen;
  a.max_sink = c->max_sink;
  a.max_middle = c->max_middle;
  a.max_recent = c->max_recent;
  a.mmb = c->max_merge_blocks;
  a.S = int(plan_segments_per_head(c));
  a.C = num_chunks;
  a.sink_mode = sink_mode;
  a.cmin = cmin;
  a.cmax = cmax;
  a.lag = lag;
  a.add_layer_offset = add_layer_offset;
  a.check_capacity = check_capacity;
  a.capacity = c->max_pack_tokens;
  for (int i = 0; i < num_chunks; ++i) a.t[i] = current_t[i];
  a.t_dev = t_dev;
  a.cu = cu;
  a.sk = sk;
  a.sg = sg;
  a.sl = sl;
  a.dst = dst;
  a.traw = traw;
  a.tremap = tremap;
  a.total_out = total;
  a.counter = counter;
  a.status = c->status;
  // the warp planner covers the pool bounds its candidate list enumerates;
  // other shapes take the thread-per-(chunk, head) walk
  if (a.H <= kPlanMaxHeads && a.max_sink <= kCandSink && a.max_recent <= kCandRecent &&
      a.mmb <= kCandMerge) {
    const int warps = n < 32 ? n : 32;
    const size_t smem = sizeof(PlanSmem);
    static std::mutex mu;
    static int attr_done[kMaxDevices] = {};
    if (per_device_once(attr_done, mu, [smem] {
          return cudaFuncSetAttribute(plan_warp_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(smem)) == cudaSuccess ? 1 : 0;
        }) <= 0) {
      cudaGetLastError();
      return PKV_ELAUNCH;
    }
    plan_warp_kernel<<<1, warps * 32, smem, stream>>>(a);
    return launch_status();
  }
  const int threads = ((n + 31) / 32) * 32;
  plan_kernel<<<1, threads, 0, stream>>>(a);
  return launch_status();
}

}  // namespace pkv

using namespace pkv;

extern "C" int pkv_plan(const pkv_cache_t* c, const uint8_t* states_layer, int layer_idx,
                        const int64_t* current_t, int num_chunks, int sink_mode_code,
                        int sink_clamp_min, int sink_clamp_max, int decoupled_sink_lag,
                        int check_capacity, int add_layer_offset, int32_t* cu_seqlens_k,
                        int32_t* src_kind, int32_t* src_slot_global, int32_t* seg_lengths,
                        int32_t* dst_token_offsets, int64_t* anchor_t_raw,
                        int64_t* anchor_t_remap, int64_t* total_tokens, int64_t* token_counter,
                        pkv_stream_t stream) {
  return launch_plan(c, states_layer, layer_idx, current_t, num_chunks, sink_mode_code,
                     sink_clamp_min, sink_clamp_max, decoupled_sink_lag, check_capacity,
                     add_layer_offset, cu_seqlens_k, src_kind, src_slot_global, seg_lengths,
                     dst_token_offsets, anchor_t_raw, anchor_t_remap, total_tokens,
                     token_counter, static_cast<cudaStream_t>(stream), nullptr);
}
