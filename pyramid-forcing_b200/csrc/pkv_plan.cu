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
#include "pkv_plan.cuh"

namespace pkv {

// Calls emit(kind, slot_in_layer, len, t_raw, t_remap) for every segment of
// (chunk c, head h) in the reference's order; returns the segment count.
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

constexpr int kPlanWarpThreads = 1024;

struct PlanSmem {
  PlanStage<kPlanMaxHeads> in;
  int64_t pair_total[1024];  // (chunk, head) pairs: launch_plan bounds them at 1024
};

__global__ void __launch_bounds__(kPlanWarpThreads, 1) plan_warp_kernel(PlanArgs a) {
  extern __shared__ __align__(16) uint8_t plan_smem_raw[];
  PlanSmem& sm = *reinterpret_cast<PlanSmem*>(plan_smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int npair = a.C * a.H;
  // stage this layer's records, valid counts and merge token counts
  stage_plan_inputs(sm.in, a, tid, blockDim.x);
  __syncthreads();
  // pass 1: each (chunk, head)'s token total
  for (int pr = warp; pr < npair; pr += nwarps) {
    const int c = pr / a.H, h = pr - c * a.H;
    int tot = 0, fp_base = 0;
    for (int j0 = 0; j0 < kCand; j0 += 32) {
      const int j = j0 + lane;
      int kind = 0, slot = 0, len = 0;
      int64_t traw = 0, tremap = 0;
      const bool v = j < kCand && plan_candidate(a, sm.in, c, h, j, kind, slot, len, traw, tremap);
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
      const bool v = j < kCand && plan_candidate(a, sm.in, c, h, j, kind, slot, len, traw, tremap);
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
        const int32_t sg = a.add_layer_offset ? layer_slot(a, kind, slot) : slot;
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
  PlanArgs a = plan_args(c, states_layer, layer, current_t, num_chunks, sink_mode, cmin, cmax,
                         lag, check_capacity, add_layer_offset, cu, total, counter, t_dev);
  a.sk = sk;
  a.sg = sg;
  a.sl = sl;
  a.dst = dst;
  a.traw = traw;
  a.tremap = tremap;
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

// ---------------------------------------------------------------------------
// Legacy all-layer plan (the M1.4 op pyramidkv_plan, pyramidkv_plan.cc:48-173):
// every (layer, head) emits three descriptors in the order sink, recent,
// middle; an active kind (valid_count > 0) is one segment from the head's
// slot 0 spanning valid_count frames (slots assumed filled 0..n-1), an
// inactive one kind -1 with zero slot, length and offset.  Offsets run
// head-major through all layers; cu_seqlens_k has one entry per (layer,
// head).  The reference builds this on the host from a blocking copy of
// valid_count and copies five arrays back; here one CTA scans the heads'
// totals (1024 per round, carried between rounds) on the device.
// ---------------------------------------------------------------------------
constexpr int kLegacyPlanThreads = 1024;

__global__ void __launch_bounds__(kLegacyPlanThreads) legacy_plan_kernel(
    const int64_t* __restrict__ vc, int N, int F, int max_sink, int max_middle,
    int max_recent, int32_t* __restrict__ cu, int32_t* __restrict__ sk,
    int32_t* __restrict__ sg, int32_t* __restrict__ sl, int32_t* __restrict__ dst) {
  __shared__ int32_t warp_sum[kLegacyPlanThreads / 32];
  __shared__ int32_t carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kind_order[3] = {0, 2, 1};  // sink, recent, middle
  const int max_slots[3] = {max_sink, max_middle, max_recent};
  if (tid == 0) {
    carry = 0;
    cu[0] = 0;
  }
  __syncthreads();
  for (int base = 0; base < N; base += blockDim.x) {
    const int i = base + tid;
    int32_t len[3] = {0, 0, 0};
    int32_t tot = 0;
    if (i < N) {
#pragma unroll
      for (int kp = 0; kp < 3; ++kp) {
        const int64_t n = vc[int64_t(i) * 3 + kind_order[kp]];
        len[kp] = n > 0 ? static_cast<int32_t>(n) * F : 0;
        tot += len[kp];
      }
    }
    int32_t incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sum[warp] = incl;
    __syncthreads();
    int32_t before = carry, round_total = 0;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) {
      if (w < warp) before += warp_sum[w];
      round_total += warp_sum[w];
    }
    if (i < N) {
      int32_t run = before + incl - tot;
#pragma unroll
      for (int kp = 0; kp < 3; ++kp) {
        const int kind = kind_order[kp];
        const int64_t d = int64_t(i) * 3 + kp;
        if (len[kp] <= 0) {
          sk[d] = -1;
          sg[d] = 0;
          sl[d] = 0;
          dst[d] = 0;
          continue;
        }
        sk[d] = kind;
        sg[d] = i * max_slots[kind];  // (layer * H + head) * max_slots + slot 0
        sl[d] = len[kp];
        dst[d] = run;
        run += len[kp];
      }
      cu[i + 1] = run;
    }
    __syncthreads();
    if (tid == 0) carry += round_total;
    __syncthreads();
  }
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

extern "C" int pkv_legacy_plan(const pkv_cache_t* c, int32_t* cu_seqlens_k, int32_t* src_kind,
                               int32_t* src_slot_global, int32_t* seg_lengths,
                               int32_t* dst_token_offsets, pkv_stream_t stream) {
  if (!c || !c->valid_count || !cu_seqlens_k || !src_kind || !src_slot_global || !seg_lengths ||
      !dst_token_offsets)
    return PKV_EINVAL;
  const int64_t n = int64_t(c->num_layers) * c->num_heads;
  if (n <= 0) return PKV_EINVAL;
  if (n > (int64_t(1) << 28)) return PKV_ECAPACITY;
  legacy_plan_kernel<<<1, kLegacyPlanThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      c->valid_count, int(n), c->frame_seqlen, c->max_sink, c->max_middle, c->max_recent,
      cu_seqlens_k, src_kind, src_slot_global, seg_lengths, dst_token_offsets);
  return launch_status();
}
