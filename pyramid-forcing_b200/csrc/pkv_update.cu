// Cache update kernels: the per-head strategy state machine, the frame
// scatter into the sink / middle / recent pools, and the fused one-layer
// MegaCache.update (routing + restore + state machine + writes + commit).
//
// Reference behaviour followed:
//   state machine  pyramidkv/csrc/anchor_store_update.cu:43-313
//   frame scatter  pyramidkv/csrc/pyramidkv_update.cu:21-110
//   layer update   pyramidkv/_mega_cache.py:136-414
//
// B200 design: the state machine is tiny and latency bound (one thread per
// head, a few dozen integer ops per frame), so it runs in one CTA and writes
// both the reference's descriptor arrays and a per-head copy work list.  The
// data movement (0.4 MB per frame and tensor) runs as a separate grid of
// 16-byte vector copies over (head, token tile) units that every SM shares.
#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

// ---------------------------------------------------------------------------
// State machine (one frame of one head).  Same transitions as the reference;
// inputs the reference would index out of its arrays with are flagged in the
// status word and the frame is skipped instead.
// ---------------------------------------------------------------------------
struct FrameDesc {
  int32_t kind, slot, accum_slot, local_idx, finalize_idx, is_new;
};

__device__ __forceinline__ void reset_live(HeadState& s, int a) {
  s.live_block[a] = -1;
#pragma unroll
  for (int j = 0; j < kMaxMergeFrames; ++j) s.live_seen[a][j] = 0;
  s.live_count[a] = 0;
}

__device__ FrameDesc advance_head(HeadState& s, int32_t t, int32_t* status) {
  FrameDesc d{kDstSkip, -1, -1, -1, -1, 0};
  switch (s.kind) {
    case kCyclic: {
      if (s.period <= 0 || s.bucket_cap <= 0) { flag(status, PKV_ST_STATE_RANGE); break; }
      const int32_t phase = t % s.period;
      if (phase < 0 || phase >= kMaxPhase) { flag(status, PKV_ST_STATE_RANGE); break; }
      const int32_t cursor = s.cyclic_cursor[phase];
      const int32_t slot = phase * s.bucket_cap + cursor;
      if (slot < 0 || slot >= kMaxPhase * kMaxBucket) { flag(status, PKV_ST_STATE_RANGE); break; }
      s.cyclic_slot[slot] = slot;
      s.cyclic_t[slot] = t;
      s.cyclic_cursor[phase] = static_cast<int8_t>((cursor + 1) % s.bucket_cap);
      d.kind = kDstMiddle;
      d.slot = slot;
      break;
    }
    case kStride:
    case kLag: {
      if (s.kind == kStride) {
        if (s.interval <= 0) { flag(status, PKV_ST_STATE_RANGE); break; }
        if (t % s.interval != 0) break;
      }
      if (s.capacity <= 0) { flag(status, PKV_ST_STATE_RANGE); break; }
      const int32_t slot = s.tkey_head;
      if (slot < 0 || slot >= kMaxTKeyed) { flag(status, PKV_ST_STATE_RANGE); break; }
      s.tkey_head = static_cast<int8_t>((slot + 1) % s.capacity);
      if (s.tkey_count < s.capacity) s.tkey_count = static_cast<int8_t>(s.tkey_count + 1);
      s.tkey_slot[slot] = slot;
      s.tkey_t[slot] = t;
      d.kind = kDstMiddle;
      d.slot = slot;
      break;
    }
    case kMerge: {
      const int32_t bf = s.block_frames;
      if (bf <= 0) break;
      if (bf > kMaxMergeFrames || s.capacity <= 0 || s.capacity > kMaxMergeBlocks) {
        flag(status, PKV_ST_STATE_RANGE);
        break;
      }
      const int32_t block = t / bf;
      const int32_t local = t % bf;
      if (local < 0) { flag(status, PKV_ST_STATE_RANGE); break; }
      int32_t a = -1;
      for (int i = 0; i < kMaxMergeActive; ++i)
        if (s.live_block[i] == block) { a = i; break; }
      int32_t fresh = 0;
      if (a < 0) {
        for (int i = 0; i < kMaxMergeActive; ++i)
          if (s.live_block[i] == -1) { a = i; break; }
        if (a < 0) a = 0;  // every accumulator busy: recycle slot 0
        reset_live(s, a);
        s.live_block[a] = block;
        fresh = 1;
      }
      if (s.live_seen[a][local] != 0) {  // duplicate frame: skipped
        flag(status, PKV_ST_MERGE_DUP);
        break;
      }
      s.live_seen[a][local] = 1;
      s.live_count[a] = static_cast<int8_t>(s.live_count[a] + 1);
      int32_t fin = -1;
      if (s.live_count[a] >= bf) {
        const int32_t start = block * bf;
        const int32_t end = start + bf - 1;
        int32_t ci;
        if (s.done_count < s.capacity) {
          ci = s.done_count;
          s.done_count = static_cast<int8_t>(s.done_count + 1);
        } else {
          // FIFO eviction as the reference does it: shift the metadata left
          // and reuse the last index (two entries then name slot cap-1).
          for (int i = 1; i < s.capacity; ++i) {
            s.done_slot[i - 1] = s.done_slot[i];
            s.done_block[i - 1] = s.done_block[i];
            s.done_start_t[i - 1] = s.done_start_t[i];
            s.done_end_t[i - 1] = s.done_end_t[i];
            s.done_median_t[i - 1] = s.done_median_t[i];
          }
          ci = s.capacity - 1;
        }
        s.done_slot[ci] = ci;
        s.done_block[ci] = block;
        s.done_start_t[ci] = start;
        s.done_end_t[ci] = end;
        s.done_median_t[ci] = (start + end) / 2;
        reset_live(s, a);
        fin = ci;
      }
      d.kind = kDstMergeAccum;
      d.accum_slot = a;
      d.local_idx = local;
      d.finalize_idx = fin;
      d.is_new = fresh;
      break;
    }
    default:
      break;  // recent-only heads have no middle anchors
  }
  return d;
}

struct DescOut {
  int32_t *kind, *slot, *frame, *head, *accum_slot, *local_idx, *finalize_idx, *is_new;
};

__device__ __forceinline__ void write_desc(const DescOut& o, int i, const FrameDesc& d, int f,
                                           int h) {
  o.kind[i] = d.kind;
  o.slot[i] = d.slot;
  o.frame[i] = f;
  o.head[i] = h;
  o.accum_slot[i] = d.accum_slot;
  o.local_idx[i] = d.local_idx;
  o.finalize_idx[i] = d.finalize_idx;
  o.is_new[i] = d.is_new;
}

// The state record is copied into registers/local memory, advanced, and
// written back; one thread owns one head.
__global__ void state_update_kernel(HeadState* __restrict__ states,
                                    const int64_t* __restrict__ t_vals, DescOut out, int H,
                                    int F, int pass_kind, int32_t* status) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= H) return;
  if (pass_kind != 1) {
    const FrameDesc skip{kDstSkip, -1, -1, -1, -1, 0};
    for (int f = 0; f < F; ++f) write_desc(out, h * F + f, skip, f, h);
    return;
  }
  HeadState s = states[h];
  for (int f = 0; f < F; ++f) {
    const FrameDesc d = advance_head(s, static_cast<int32_t>(t_vals[f]), status);
    write_desc(out, h * F + f, d, f, h);
  }
  states[h] = s;
}

// ---------------------------------------------------------------------------
// Frame scatter (op pyramidkv_update).  Work unit = (descriptor, token tile);
// each thread moves 16-byte chunks of K and V.
// ---------------------------------------------------------------------------
constexpr int kTileTokens = 32;

struct PoolView {
  uint16_t* k[3];
  uint16_t* v[3];
  int64_t* pos[3];
  int64_t rows[3];  // L*H*slots per kind
};

__host__ __forceinline__ PoolView pool_view(const pkv_cache_t* c) {
  PoolView p{};
  const int64_t lh = int64_t(c->num_layers) * c->num_heads;
  p.k[0] = c->sink_k; p.v[0] = c->sink_v; p.pos[0] = c->sink_pos; p.rows[0] = lh * c->max_sink;
  p.k[1] = c->middle_k; p.v[1] = c->middle_v; p.pos[1] = c->middle_pos;
  p.rows[1] = lh * c->max_middle;
  p.k[2] = c->recent_k; p.v[2] = c->recent_v; p.pos[2] = c->recent_pos;
  p.rows[2] = lh * c->max_recent;
  return p;
}

template <bool kVec>
__device__ __forceinline__ void copy_rows(uint16_t* __restrict__ dst,
                                          const uint16_t* __restrict__ src, int64_t src_stride,
                                          int tok0, int ntok, int D) {
  // dst rows are contiguous [tok][D]; src rows are src_stride apart.
  if (kVec) {
    const int cpr = D / 8;  // 16-byte chunks per row
    const int total = ntok * cpr;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const int r = i / cpr, c = i - r * cpr;
      const uint4 x = *reinterpret_cast<const uint4*>(src + int64_t(tok0 + r) * src_stride + c * 8);
      *reinterpret_cast<uint4*>(dst + int64_t(tok0 + r) * D + c * 8) = x;
    }
  } else {
    const int total = ntok * D;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const int r = i / D, c = i - r * D;
      dst[int64_t(tok0 + r) * D + c] = src[int64_t(tok0 + r) * src_stride + c];
    }
  }
}

template <bool kVec>
__global__ void update_frames_kernel(PoolView pools, const uint16_t* __restrict__ new_k,
                                     const uint16_t* __restrict__ new_v,
                                     const int64_t* __restrict__ new_pos,
                                     const int32_t* __restrict__ dkind,
                                     const int32_t* __restrict__ dslot,
                                     const int32_t* __restrict__ sframe,
                                     const int32_t* __restrict__ shead, int n_ops, int H,
                                     int FSEQ, int D, int32_t* status) {
  const int tiles = (FSEQ + kTileTokens - 1) / kTileTokens;
  for (int64_t u = blockIdx.x; u < int64_t(n_ops) * tiles; u += gridDim.x) {
    const int op = int(u / tiles);
    const int tile = int(u - int64_t(op) * tiles);
    const int kind = dkind[op];
    if (kind < 0) continue;
    if (kind > 2) {
      if (tile == 0 && threadIdx.x == 0) flag(status, PKV_ST_BAD_KIND);
      continue;
    }
    const int64_t slot = dslot[op];
    const int f = sframe[op], h = shead[op];
    if (slot < 0 || slot >= pools.rows[kind] || h < 0 || h >= H || f < 0) {
      if (tile == 0 && threadIdx.x == 0) flag(status, PKV_ST_SLOT_RANGE);
      continue;
    }
    const int tok0 = tile * kTileTokens;
    const int ntok = min(kTileTokens, FSEQ - tok0);
    const int64_t src = (int64_t(f) * H + h) * FSEQ * D;
    const int64_t dst = slot * FSEQ * D;
    copy_rows<kVec>(pools.k[kind] + dst, new_k + src, D, tok0, ntok, D);
    copy_rows<kVec>(pools.v[kind] + dst, new_v + src, D, tok0, ntok, D);
    if (new_pos != nullptr && pools.pos[kind] != nullptr) {
      const int64_t ps = (int64_t(f) * H + h) * FSEQ * 3 + int64_t(tok0) * 3;
      const int64_t pd = slot * FSEQ * 3 + int64_t(tok0) * 3;
      for (int i = threadIdx.x; i < ntok * 3; i += blockDim.x)
        pools.pos[kind][pd + i] = new_pos[ps + i];
    }
  }
}

// ---------------------------------------------------------------------------
// Fused one-layer update.
//
// route_kernel (one CTA, thread = head) reproduces _mega_cache.py:217-414's
// bookkeeping on the device: it restores valid_count from the committed
// snapshot, decides each head's sink / recent routing, runs the state machine
// on clean passes, writes the reference's descriptors (to scratch) and a
// per-head ordered list of frame copies, and commits valid_count.
//
// A copy item (4 x int32): src (>= 0: incoming frame index; < 0: committed
// recent slot -src-1), dst kind (0 sink / 1 middle / 2 recent) | commit<<8,
// dst slot within the layer-head ([0, slots)), unused.
//
// copy_kernel then runs over (head, token tile) units; each unit walks its
// head's items in list order and every thread owns the same chunk columns in
// every item, so a recent slot's shifted source (committed slot j+evict) is
// always read before the same thread overwrites it with the commit of slot
// j+evict.
// ---------------------------------------------------------------------------
struct RouteArgs {
  int64_t* vc;            // [L,H,3]
  int64_t* committed_vc;  // [L,H,3]
  const int64_t* sink_caps;
  HeadState* states;      // this layer's H records
  DescOut desc;
  int32_t* items;         // [H][items_per_head][4]
  int32_t* item_count;    // [H]
  int items_per_head;
  int layer, H, F, max_sink, max_middle, max_recent;
  int64_t first_t;
  int pass_kind;
  int32_t* status;
  const int64_t* t_dev;  // device first_t (nullable): replaces first_t when set
};

__global__ void route_kernel(RouteArgs a) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= a.H) return;
  const int64_t first_t = a.t_dev != nullptr ? __ldg(a.t_dev) : a.first_t;
  const int64_t vi = (int64_t(a.layer) * a.H + h) * 3;
  const int64_t sc = a.committed_vc[vi + 0];
  const int64_t mc = a.committed_vc[vi + 1];
  const int64_t rc = a.committed_vc[vi + 2];
  int64_t cap = a.sink_caps[int64_t(a.layer) * a.H + h];
  if (cap > a.max_sink) cap = a.max_sink;
  int64_t sw = cap - sc;
  if (sw > a.F) sw = a.F;
  if (sw < 0) sw = 0;
  const int rw = a.F - int(sw);
  const int mr = a.max_recent;

  int32_t* it = a.items + int64_t(h) * a.items_per_head * 4;
  int n = 0;
  auto push = [&](int src, int kind, int commit, int slot) {
    if (n < a.items_per_head) {
      it[n * 4 + 0] = src;
      it[n * 4 + 1] = kind | (commit << 8);
      it[n * 4 + 2] = slot;
      it[n * 4 + 3] = 0;
      ++n;
    }
  };
  const int commit = a.pass_kind == 1 ? 1 : 0;

  // Recent pool of this head, slot by slot, in increasing slot order.
  int64_t rc_post = rc;
  if (rw > 0 && rw > mr) {
    flag(a.status, PKV_ST_RECENT_RANGE);
  }
  if (rw == 0) {
    for (int j = 0; j < mr; ++j) push(-j - 1, kDstRecent, commit, j);
  } else if (rc + rw <= mr) {
    for (int j = 0; j < mr; ++j) {
      if (j >= rc && j < rc + rw) push(int(sw) + (j - int(rc)), kDstRecent, commit, j);
      else push(-j - 1, kDstRecent, commit, j);
    }
    rc_post = rc + rw;
  } else {
    const int ev = int(rc) + rw - mr;
    for (int j = 0; j < mr; ++j) {
      if (j >= mr - rw) push(int(sw) + (j - (mr - rw)), kDstRecent, commit, j);
      else if (j + ev < mr) push(-(j + ev) - 1, kDstRecent, commit, j);
      else push(-j - 1, kDstRecent, commit, j);
    }
    rc_post = mr;
  }
  for (int i = 0; i < int(sw); ++i) push(i, kDstSink, 0, int(sc) + i);

  a.vc[vi + 0] = sc + sw;
  a.vc[vi + 1] = mc;
  a.vc[vi + 2] = rc_post;

  if (a.pass_kind == 1) {
    HeadState s = a.states[h];
    for (int f = 0; f < a.F; ++f) {
      const FrameDesc d = advance_head(s, static_cast<int32_t>(first_t + f), a.status);
      write_desc(a.desc, h * a.F + f, d, f, h);
      if (d.kind == kDstMiddle) {
        if (d.slot >= 0 && d.slot < a.max_middle) push(f, kDstMiddle, 0, d.slot);
        else flag(a.status, PKV_ST_SLOT_RANGE);
      }
    }
    a.states[h] = s;
    a.committed_vc[vi + 0] = sc + sw;
    a.committed_vc[vi + 1] = mc;
    a.committed_vc[vi + 2] = rc_post;
  }
  a.item_count[h] = n;
}

struct CopyArgs {
  PoolView pools;
  uint16_t* committed_k;
  uint16_t* committed_v;
  int64_t* committed_pos;
  const uint16_t* new_k;
  const uint16_t* new_v;
  int64_t tok_stride, head_stride;  // of new_k / new_v (elements)
  const int32_t* items;
  const int32_t* item_count;
  int items_per_head;
  int layer, H, FSEQ, D, W;
  int max_sink, max_middle, max_recent;
  int64_t first_t;
  const int64_t* t_dev;  // device first_t (nullable): replaces first_t when set
};

template <bool kVec>
__global__ void copy_kernel(CopyArgs a) {
  const int64_t first_t = a.t_dev != nullptr ? __ldg(a.t_dev) : a.first_t;
  const int tiles = (a.FSEQ + kTileTokens - 1) / kTileTokens;
  const int slots[3] = {a.max_sink, a.max_middle, a.max_recent};
  for (int u = blockIdx.x; u < a.H * tiles; u += gridDim.x) {
    const int h = u / tiles;
    const int tile = u - h * tiles;
    const int tok0 = tile * kTileTokens;
    const int ntok = min(kTileTokens, a.FSEQ - tok0);
    const int n = a.item_count[h];
    const int32_t* it = a.items + int64_t(h) * a.items_per_head * 4;
    for (int i = 0; i < n; ++i) {
      // Items of one head run in list order: a later item may overwrite a
      // committed slot an earlier item read (the FIFO shift source).
      if (i > 0) __syncthreads();
      const int src = it[i * 4 + 0];
      const int kind = it[i * 4 + 1] & 0xff;
      const int commit = it[i * 4 + 1] >> 8;
      const int slot = it[i * 4 + 2];
      const int64_t row = (int64_t(a.layer) * a.H + h) * slots[kind] + slot;
      uint16_t* dk = a.pools.k[kind] + row * a.FSEQ * a.D;
      uint16_t* dv = a.pools.v[kind] + row * a.FSEQ * a.D;
      int64_t* dp = a.pools.pos[kind] + row * a.FSEQ * 3;
      const int64_t crow = (int64_t(a.layer) * a.H + h) * a.max_recent;
      if (src >= 0) {
        // incoming frame `src`: token t of head h at (src*F + t)*tok_stride + h*head_stride
        const uint16_t* sk = a.new_k + int64_t(src) * a.FSEQ * a.tok_stride + int64_t(h) * a.head_stride;
        const uint16_t* sv = a.new_v + int64_t(src) * a.FSEQ * a.tok_stride + int64_t(h) * a.head_stride;
        copy_rows<kVec>(dk, sk, a.tok_stride, tok0, ntok, a.D);
        copy_rows<kVec>(dv, sv, a.tok_stride, tok0, ntok, a.D);
        if (commit) {
          copy_rows<kVec>(a.committed_k + (crow + slot) * a.FSEQ * a.D, sk, a.tok_stride, tok0,
                          ntok, a.D);
          copy_rows<kVec>(a.committed_v + (crow + slot) * a.FSEQ * a.D, sv, a.tok_stride, tok0,
                          ntok, a.D);
        }
        const int64_t t = first_t + src;
        for (int r = threadIdx.x; r < ntok; r += blockDim.x) {
          const int tok = tok0 + r;
          const int64_t y = tok / a.W, x = tok % a.W;
          dp[int64_t(tok) * 3 + 0] = t;
          dp[int64_t(tok) * 3 + 1] = y;
          dp[int64_t(tok) * 3 + 2] = x;
          if (commit) {
            int64_t* cp = a.committed_pos + (crow + slot) * a.FSEQ * 3 + int64_t(tok) * 3;
            cp[0] = t; cp[1] = y; cp[2] = x;
          }
        }
      } else {
        // committed recent slot `cs` (restore / FIFO shift)
        const int cs = -src - 1;
        const uint16_t* sk = a.committed_k + (crow + cs) * a.FSEQ * a.D;
        const uint16_t* sv = a.committed_v + (crow + cs) * a.FSEQ * a.D;
        const int64_t* sp = a.committed_pos + (crow + cs) * a.FSEQ * 3;
        copy_rows<kVec>(dk, sk, a.D, tok0, ntok, a.D);
        copy_rows<kVec>(dv, sv, a.D, tok0, ntok, a.D);
        if (commit && cs != slot) {
          copy_rows<kVec>(a.committed_k + (crow + slot) * a.FSEQ * a.D, sk, a.D, tok0, ntok, a.D);
          copy_rows<kVec>(a.committed_v + (crow + slot) * a.FSEQ * a.D, sv, a.D, tok0, ntok, a.D);
        }
        for (int e = threadIdx.x; e < ntok * 3; e += blockDim.x) {
          const int64_t v = sp[int64_t(tok0) * 3 + e];
          dp[int64_t(tok0) * 3 + e] = v;
          if (commit && cs != slot)
            a.committed_pos[(crow + slot) * a.FSEQ * 3 + int64_t(tok0) * 3 + e] = v;
        }
      }
    }
  }
}

static int grid_for(int64_t units, int per_sm = 8) {
  int64_t g = int64_t(sm_count()) * per_sm;
  if (units < g) g = units;
  return int(g < 1 ? 1 : g);
}

}  // namespace pkv

using namespace pkv;

extern "C" int64_t pkv_state_perhead_size(void) { return int64_t(sizeof(HeadState)); }

extern "C" int64_t pkv_scratch_bytes(const pkv_cache_t* cache) {
  if (cache == nullptr) return 0;
  return scratch_layout(cache).bytes;
}

extern "C" const char* pkv_error_string(int code) {
  switch (code) {
    case PKV_OK: return "ok";
    case PKV_EINVAL: return "invalid argument";
    case PKV_ELAUNCH: return "CUDA launch failed";
    case PKV_ECAPACITY: return "request exceeds a sized or compiled capacity";
    case PKV_EUNSUPPORTED: return "unsupported configuration";
    case PKV_ENOALLOC_LIMIT:
      return "plan needs more scratch than the allocation-free entry point's fixed array";
    default: return "unknown error";
  }
}

extern "C" int pkv_mega_state_update(uint8_t* states, const int64_t* new_t_vals,
                                     int32_t* desc_dst_kind, int32_t* desc_dst_slot,
                                     int32_t* desc_src_frame, int32_t* desc_src_head,
                                     int32_t* desc_merge_accum_slot,
                                     int32_t* desc_merge_local_idx,
                                     int32_t* desc_merge_finalize_completed_idx,
                                     int32_t* desc_merge_is_new_block, int num_heads,
                                     int frames_in_block, int pass_kind, int32_t* status,
                                     pkv_stream_t stream) {
  if (num_heads == 0 || frames_in_block == 0) return PKV_OK;
  if (!states || !new_t_vals || !desc_dst_kind || !desc_dst_slot || !desc_src_frame ||
      !desc_src_head || !desc_merge_accum_slot || !desc_merge_local_idx ||
      !desc_merge_finalize_completed_idx || !desc_merge_is_new_block || num_heads < 0 ||
      frames_in_block < 0)
    return PKV_EINVAL;
  DescOut o{desc_dst_kind, desc_dst_slot, desc_src_frame, desc_src_head, desc_merge_accum_slot,
            desc_merge_local_idx, desc_merge_finalize_completed_idx, desc_merge_is_new_block};
  const int threads = 32;
  const int blocks = (num_heads + threads - 1) / threads;
  state_update_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<HeadState*>(states), new_t_vals, o, num_heads, frames_in_block,
      pass_kind, status);
  return launch_status();
}

extern "C" int pkv_update_frames(const pkv_cache_t* c, const uint16_t* new_k,
                                 const uint16_t* new_v, const int64_t* new_pos,
                                 const int32_t* dst_kind, const int32_t* dst_slot_global,
                                 const int32_t* src_frame_in_block, const int32_t* src_head,
                                 int num_ops, pkv_stream_t stream) {
  if (num_ops == 0) return PKV_OK;
  if (!c || !new_k || !new_v || !dst_kind || !dst_slot_global || !src_frame_in_block ||
      !src_head || num_ops < 0)
    return PKV_EINVAL;
  const PoolView p = pool_view(c);
  const int tiles = (c->frame_seqlen + kTileTokens - 1) / kTileTokens;
  const int grid = grid_for(int64_t(num_ops) * tiles);
  const bool vec = (c->head_dim % 8 == 0) && ((reinterpret_cast<uintptr_t>(new_k) |
                                               reinterpret_cast<uintptr_t>(new_v)) % 16 == 0);
  auto s = static_cast<cudaStream_t>(stream);
  if (vec)
    update_frames_kernel<true><<<grid, 256, 0, s>>>(p, new_k, new_v, new_pos, dst_kind,
                                                     dst_slot_global, src_frame_in_block,
                                                     src_head, num_ops, c->num_heads,
                                                     c->frame_seqlen, c->head_dim, c->status);
  else
    update_frames_kernel<false><<<grid, 256, 0, s>>>(p, new_k, new_v, new_pos, dst_kind,
                                                      dst_slot_global, src_frame_in_block,
                                                      src_head, num_ops, c->num_heads,
                                                      c->frame_seqlen, c->head_dim, c->status);
  return launch_status();
}

extern "C" int pkv_cache_update(const pkv_cache_t* c, uint8_t* states, int layer,
                                const uint16_t* new_k, const uint16_t* new_v,
                                int64_t tok_stride, int64_t head_stride, int frames,
                                int64_t first_t, int pass_kind, int has_merge_head,
                                pkv_stream_t stream) {
  if (!c || !states || !new_k || !new_v || !c->scratch || !c->committed_vc ||
      !c->committed_recent_k || !c->committed_recent_v || !c->committed_recent_pos ||
      !c->sink_caps || !c->valid_count)
    return PKV_EINVAL;
  if (layer < 0 || layer >= c->num_layers || frames <= 0) return PKV_EINVAL;
  if (frames > kMaxFramesPerUpdate) return PKV_ECAPACITY;
  if (pass_kind != 0 && pass_kind != 1) return PKV_OK;  // neither noisy nor clean: no-op
  const ScratchLayout sl = scratch_layout(c);
  if (c->scratch_bytes < sl.bytes) return PKV_ECAPACITY;
  char* scr = static_cast<char*>(c->scratch);
  const int H = c->num_heads;
  const int NF = H * frames;
  int32_t* d = reinterpret_cast<int32_t*>(scr + sl.desc);
  DescOut desc{d, d + NF, d + 2 * NF, d + 3 * NF, d + 4 * NF, d + 5 * NF, d + 6 * NF, d + 7 * NF};
  const int items_per_head = kMaxFramesPerUpdate + c->max_recent + kMaxFramesPerUpdate;
  int32_t* items = reinterpret_cast<int32_t*>(scr + sl.copy_items);
  int32_t* counts = items + int64_t(H) * items_per_head * 4;
  auto s = static_cast<cudaStream_t>(stream);
  uint8_t* layer_states = states + int64_t(layer) * H * sizeof(HeadState);

  RouteArgs ra{c->valid_count, c->committed_vc, c->sink_caps,
               reinterpret_cast<HeadState*>(layer_states), desc, items, counts, items_per_head,
               layer, H, frames, c->max_sink, c->max_middle, c->max_recent, first_t, pass_kind,
               c->status, c->first_t_dev};
  route_kernel<<<(H + 127) / 128, 128, 0, s>>>(ra);
  int rc = launch_status();
  if (rc != PKV_OK) return rc;

  CopyArgs ca{};
  ca.pools = pool_view(c);
  ca.committed_k = c->committed_recent_k;
  ca.committed_v = c->committed_recent_v;
  ca.committed_pos = c->committed_recent_pos;
  ca.new_k = new_k;
  ca.new_v = new_v;
  ca.tok_stride = tok_stride;
  ca.head_stride = head_stride;
  ca.items = items;
  ca.item_count = counts;
  ca.items_per_head = items_per_head;
  ca.layer = layer;
  ca.H = H;
  ca.FSEQ = c->frame_seqlen;
  ca.D = c->head_dim;
  ca.W = c->spatial_width > 0 ? c->spatial_width : 1;
  ca.max_sink = c->max_sink;
  ca.max_middle = c->max_middle;
  ca.max_recent = c->max_recent;
  ca.first_t = first_t;
  ca.t_dev = c->first_t_dev;
  const int tiles = (c->frame_seqlen + kTileTokens - 1) / kTileTokens;
  const int grid = grid_for(int64_t(H) * tiles);
  const bool vec = (c->head_dim % 8 == 0) && (tok_stride % 8 == 0) && (head_stride % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(new_k) | reinterpret_cast<uintptr_t>(new_v)) %
                        16 == 0);
  if (vec) copy_kernel<true><<<grid, 256, 0, s>>>(ca);
  else copy_kernel<false><<<grid, 256, 0, s>>>(ca);
  rc = launch_status();
  if (rc != PKV_OK) return rc;

  if (pass_kind == 1 && has_merge_head) {
    const int64_t lh = int64_t(layer) * H;
    const int MMA = c->max_merge_active, MMB = c->max_merge_blocks, MTPA = c->max_merge_tokens;
    const int64_t D = c->head_dim, F = c->frame_seqlen;
    MergeLaunch m{};
    m.states = reinterpret_cast<const HeadState*>(layer_states);
    m.new_k = new_k;
    m.new_v = new_v;
    m.frame_stride = F * tok_stride;
    m.head_stride = head_stride;
    m.tok_stride = tok_stride;
    m.new_pos = nullptr;
    m.pos_width = ca.W;
    m.first_t = first_t;
    m.t_dev = c->first_t_dev;
    m.dkind = desc.kind;
    m.dslot = desc.accum_slot;
    m.dfin = desc.finalize_idx;
    m.dnew = desc.is_new;
    m.acc_k = c->accum_sum_k + lh * MMA * MTPA * D;
    m.acc_v = c->accum_sum_v + lh * MMA * MTPA * D;
    m.acc_pos = c->accum_pos + lh * MMA * MTPA * 3;
    m.acc_gid = c->accum_group_ids + lh * MMA * F;
    m.acc_tpg = c->accum_tokens_per_group + lh * MMA * MTPA;
    m.acc_ng = c->accum_num_groups + lh * MMA;
    m.mk = c->merge_k + lh * MMB * MTPA * D;
    m.mv = c->merge_v + lh * MMB * MTPA * D;
    m.mpos = c->merge_pos + lh * MMB * MTPA * 3;
    m.mtc = c->merge_token_count + lh * MMB;
    m.H = H;
    m.F = frames;
    m.FSEQ = c->frame_seqlen;
    m.D = c->head_dim;
    m.MMA = MMA;
    m.MMB = MMB;
    m.MTPA = MTPA;
    m.status = c->status;
    rc = launch_merge(m, s);
  }
  return rc;
}
