// The planner's per-(chunk, head) segment rules, shared by the planner
// kernels (pkv_plan.cu) and the pack kernel that plans for itself
// (pkv_pack.cu).  Reference: pyramidkv/csrc/mega_plan.cc:133-264
// (emit_chunk_plan) and :63-80 (map_sink_time).
#pragma once

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

// Time of chunk c: from the launch parameters, or chunk 0's time read from
// device memory when the caller keeps it there (graph replay across blocks).
__device__ __forceinline__ int64_t chunk_time(const PlanArgs& a, int c) {
  return a.t_dev != nullptr ? __ldg(a.t_dev) + c : a.t[c];
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
constexpr int kCandSink = 3, kCandRecent = 4, kCandMiddle = 24, kCandMerge = 6;
constexpr int kCand = kCandSink + kCandRecent + kCandMiddle + kCandMerge;  // 37
constexpr int kPlanMaxHeads = 64;

// One layer's planner inputs staged in shared memory: state records, valid
// counts and merge token counts of up to kMaxH heads (at most 8 merge slots).
template <int kMaxH>
struct PlanStage {
  HeadState st[kMaxH];
  int64_t vc[kMaxH * 3];
  int32_t mtc[kMaxH * 8];
};

template <int kMaxH>
__device__ __forceinline__ void stage_plan_inputs(PlanStage<kMaxH>& sm, const PlanArgs& a,
                                                  int tid, int nthreads) {
  const uint32_t* src = reinterpret_cast<const uint32_t*>(a.states);
  uint32_t* dst = reinterpret_cast<uint32_t*>(sm.st);
  for (int i = tid; i < a.H * int(sizeof(HeadState) / 4); i += nthreads) dst[i] = src[i];
  const int64_t* vcl = a.vc + int64_t(a.layer) * a.H * 3;
  for (int i = tid; i < a.H * 3; i += nthreads) sm.vc[i] = vcl[i];
  const int32_t* ml = a.mtc + int64_t(a.layer) * a.H * a.mmb;
  for (int i = tid; i < a.H * a.mmb; i += nthreads) sm.mtc[i] = ml[i];
}

// Phase of a cyclic head at chunk time ct (0 for the other kinds).
__device__ __forceinline__ int head_phase(const HeadState& s, int64_t ct) {
  if (s.kind != kCyclic) return 0;
  const int period = s.period > 0 ? s.period : 1;
  return static_cast<int>(((ct % period) + period) % period);
}

// Candidate j of head h at chunk time ct (sync_t = map_sink_time(ct), phase
// = head_phase(ct)): kind, slot in layer, length, t_raw, t_remap; false when
// the candidate is not a segment.
template <class Stage>
__device__ __forceinline__ bool plan_candidate_at(const PlanArgs& a, const Stage& sm, int h,
                                                  int j, int64_t sync_t, int phase, int& kind,
                                                  int& slot, int& len, int64_t& traw,
                                                  int64_t& tremap) {
  const HeadState& s = sm.st[h];
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
      const int bcap = s.bucket_cap > 0 ? s.bucket_cap : 1;
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

// Candidate j of (chunk c, head h).
template <class Stage>
__device__ __forceinline__ bool plan_candidate(const PlanArgs& a, const Stage& sm, int c,
                                               int h, int j, int& kind, int& slot, int& len,
                                               int64_t& traw, int64_t& tremap) {
  const int64_t ct = chunk_time(a, c);
  const int64_t sync_t = map_sink_time(ct, a.sink_mode, a.cmin, a.cmax, a.lag);
  return plan_candidate_at(a, sm, h, j, sync_t, head_phase(sm.st[h], ct), kind, slot, len, traw,
                           tremap);
}


// The per-kind layer offset of a slot (pyramidkv/_mega_attention.py:349-385).
__device__ __forceinline__ int32_t layer_slot(const PlanArgs& a, int kind, int slot) {
  const int per_head = kind == kDstSink     ? a.max_sink
                       : kind == kDstMiddle ? a.max_middle
                       : kind == kDstRecent ? a.max_recent
                                            : a.mmb;
  return slot + a.layer * a.H * per_head;
}

// A layer's planner arguments (descriptor outputs left null).
inline PlanArgs plan_args(const pkv_cache_t* c, const uint8_t* states_layer, int layer,
                          const int64_t* current_t, int num_chunks, int sink_mode, int cmin,
                          int cmax, int lag, int check_capacity, int add_layer_offset,
                          int32_t* cu, int64_t* total, int64_t* counter, const int64_t* t_dev) {
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
  for (int i = 0; i < num_chunks && i < PKV_MAX_CHUNKS; ++i) a.t[i] = current_t[i];
  a.t_dev = t_dev;
  a.cu = cu;
  a.total_out = total;
  a.counter = counter;
  a.status = c->status;
  return a;
}

// The pack that plans for itself (pkv_pack.cu) covers shapes whose candidate
// list is complete: every valid candidate is a segment the planner emits.
bool plan_pack_fits(const pkv_cache_t* c, const PlanArgs& pa);
// Plan + pack in one launch: cu_seqlens_k, the token total and counter as
// the planner writes them, the packed K (RoPE'd) / V / positions as the pack.
int launch_pack_planned(const pkv_cache_t* c, const PlanArgs& pa, const float* ft, int ft_rows,
                        int ft_cols, const float* fy, int fy_rows, int fy_cols, const float* fx,
                        int fx_rows, int fx_cols, cudaStream_t stream);

}  // namespace pkv
