// Shared device-side definitions of the B200 MegaCache library.
//
// HeadState is the 600-byte per-(layer, head) strategy record.  Its byte
// layout is an interface shared with every caller that builds or inspects
// the raw states buffer (the reference's numpy mirror
// pyramidkv/_mega_state_ops.py:36-77 and its C++ struct
// pyramidkv/csrc/anchor_store.cuh:62-132), so the field order, widths and
// padding are fixed; the static_asserts below pin them.
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/pkv.h"

namespace pkv {

constexpr int kMaxPhase = PKV_MAX_PHASE;
constexpr int kMaxBucket = PKV_MAX_BUCKET;
constexpr int kMaxTKeyed = PKV_MAX_T_KEYED;
constexpr int kMaxLag = PKV_MAX_LAG_OFFSETS;
constexpr int kMaxMergeBlocks = PKV_MAX_MERGE_BLOCKS;
constexpr int kMaxMergeActive = PKV_MAX_MERGE_ACTIVE;
constexpr int kMaxMergeFrames = PKV_MAX_MERGE_BLOCK_FRAMES;
constexpr int kMaxMergeTokens = PKV_MAX_MERGE_TOKENS;

// Strategy kinds (anchor_store.cuh:47-53).
enum : int8_t { kRecent = 0, kCyclic = 1, kStride = 2, kLag = 3, kMerge = 4 };

// Descriptor destination kinds shared with the pool kernels
// (anchor_store_update.cu:33-41, pyramidkv_pack.cu:75-77).
constexpr int32_t kDstSkip = -1;
constexpr int32_t kDstSink = 0;
constexpr int32_t kDstMiddle = 1;
constexpr int32_t kDstRecent = 2;
constexpr int32_t kSrcMerge = 3;
constexpr int32_t kDstMergeAccum = 5;

struct HeadState {
  int8_t kind;
  int8_t sink_capacity;
  int8_t pad0[2];
  int32_t period, bucket_cap, interval, capacity, patch_size, block_frames;
  int32_t lag_offsets[kMaxLag];
  int32_t lag_offset_count;
  int32_t cyclic_slot[kMaxPhase * kMaxBucket];
  int32_t cyclic_t[kMaxPhase * kMaxBucket];
  int8_t cyclic_cursor[kMaxPhase];
  int32_t tkey_slot[kMaxTKeyed];
  int32_t tkey_t[kMaxTKeyed];
  int8_t tkey_count, tkey_head;
  int8_t pad1[2];
  int32_t done_slot[kMaxMergeBlocks];
  int32_t done_block[kMaxMergeBlocks];
  int32_t done_start_t[kMaxMergeBlocks];
  int32_t done_end_t[kMaxMergeBlocks];
  int32_t done_median_t[kMaxMergeBlocks];
  int8_t done_count;
  int8_t pad2[3];
  int32_t live_block[kMaxMergeActive];
  int32_t live_slot[kMaxMergeActive];
  int8_t live_seen[kMaxMergeActive][kMaxMergeFrames];
  int8_t live_count[kMaxMergeActive];
  int8_t pad3[2];
  int32_t cached_num_groups;
};

static_assert(sizeof(HeadState) == 600, "HeadState must stay byte-identical (600 B)");
static_assert(offsetof(HeadState, cyclic_cursor) == 240, "layout");
static_assert(offsetof(HeadState, tkey_slot) == 248, "layout");
static_assert(offsetof(HeadState, tkey_count) == 440, "layout");
static_assert(offsetof(HeadState, done_slot) == 444, "layout");
static_assert(offsetof(HeadState, done_count) == 564, "layout");
static_assert(offsetof(HeadState, live_block) == 568, "layout");
static_assert(offsetof(HeadState, live_seen) == 584, "layout");
static_assert(offsetof(HeadState, cached_num_groups) == 596, "layout");

__device__ __forceinline__ void flag(int32_t* status, int32_t bits) {
  if (status != nullptr) atomicOr(status, bits);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) {
  return __uint_as_float(b << 16);
}

// Round-to-nearest-even f32 -> bf16 bits (the conversion __float2bfloat16
// performs).
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float f) {
  const __nv_bfloat16 h = __float2bfloat16_rn(f);
  return static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&h));
}

template <typename T>
__device__ __forceinline__ T ld_nc(const T* p) {
  return __ldg(p);
}

inline int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PKV_OK : PKV_ELAUNCH;
}

constexpr int kMaxDevices = 64;

// A positive value computed once per device, on the first call made with
// that device current (a kernel's shared-memory opt-in, a device attribute).
// Host threads may call concurrently; fn() returning <= 0 is not cached.
template <typename Fn>
inline int per_device_once(int (&cache)[kMaxDevices], std::mutex& mu, Fn fn) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return fn();
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] > 0) return cache[dev];
  const int v = fn();
  if (v > 0) cache[dev] = v;
  return v;
}

// Streaming multiprocessors of the current device.
inline int sm_count() {
  static std::mutex mu;
  static int cache[kMaxDevices] = {};
  return per_device_once(cache, mu, [] {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
  });
}

// Scratch arena layout used by the fused update / attend paths.  Offsets are
// computed on the host from the cache dimensions; every region is
// 256-byte aligned.
struct ScratchLayout {
  int64_t desc;        // 8 x [H * kMaxFramesPerUpdate] int32 descriptors
  int64_t copy_items;  // fused-update copy work list
  int64_t plan;        // cu + sk/sg/sl/dst + traw/tremap for max_attend_chunks
  int64_t plan_total;  // int64 packed-token total of the last plan
  int64_t attn_part;   // attention: per-CTA partial results of split units
  int64_t attn_cnt;    // attention: per-(unit, tile, warp) arrival counters
  int64_t bytes;
};

constexpr int kMaxFramesPerUpdate = 16;

// Ragged-attention workspace (pkv_attn.cu): per persistent CTA two slots x
// two query tiles of fp32 partials (130 rows of 128: O columns, m, l, plus 32
// words of headers), and an arrival counter per (unit, tile, warp).
constexpr int kAttnMaxCtas = 160;
constexpr int64_t kAttnPartFloats = 130 * 128 + 32;
constexpr int64_t kAttnPartBytes = int64_t(kAttnMaxCtas) * 4 * kAttnPartFloats * 4;
constexpr int kAttnCntPerUnit = 8;

// Attention units (segment x pair of 128-row query tiles) of the largest attend.
inline int64_t attn_units(const pkv_cache_t* c) {
  const int64_t tiles = (int64_t(c->frame_seqlen) + 127) / 128;
  return int64_t(c->max_attend_chunks) * c->num_heads * ((tiles + 1) / 2);
}

inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

inline int64_t plan_segments_per_head(const pkv_cache_t* c) {
  return int64_t(c->max_sink) + c->max_middle + c->max_recent + c->max_merge_blocks;
}

inline ScratchLayout scratch_layout(const pkv_cache_t* c) {
  ScratchLayout s{};
  const int64_t H = c->num_heads;
  int64_t off = 0;
  s.desc = off;
  off = align256(off + 8 * H * kMaxFramesPerUpdate * 4);
  s.copy_items = off;
  // sink writes + recent slots (+ committed) + middle writes, 4 int32 each
  const int64_t items = H * (kMaxFramesPerUpdate + c->max_recent + kMaxFramesPerUpdate);
  off = align256(off + items * 16 + H * 4);  // items + per-head counts
  s.plan = off;
  const int64_t C = c->max_attend_chunks;
  const int64_t N = C * H * plan_segments_per_head(c);
  off = align256(off + N * 4 * 4 + 8 + N * 8 * 2);
  s.plan_total = off;
  off = align256(off + 64);
  s.attn_part = off;
  off = align256(off + kAttnPartBytes);
  s.attn_cnt = off;
  off = align256(off + attn_units(c) * kAttnCntPerUnit * 4);
  s.bytes = off;
  return s;
}

}  // namespace pkv
