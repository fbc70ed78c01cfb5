// The AdaptiveKVCache / CppStrategyManager ops of the adahead library:
// scatter_copy, apply_pos_override, refresh_readout_layout and
// anchor_store_write_frames.  They are not on the MegaCache path; they are
// here so code that still calls them keeps working.
//
// Reference behaviour: pyramidkv/csrc/scatter_copy.cu:13-225 (kernels) and
// scatter_copy_bind.cpp:449-684 (checks, mapping-mode names).  Results are the
// same bytes; two things differ on purpose:
//   * launches go to the caller's stream (the reference's go to the legacy
//     default stream, scatter_copy.cu:244,263,296,334, which orders them
//     against nothing else on a torch stream);
//   * copies move 16 bytes per access when both ends and the length allow it
//     (4-byte words plus a byte tail otherwise), and any alignment is handled
//     (the reference casts to int32 pointers whatever the alignment).
// One CTA per segment / frame, as the reference: these ops move a handful of
// segments per call.
#include <cmath>

#include "pkv_common.cuh"

namespace pkv {
namespace {

constexpr int kLegacyThreads = 256;

// dst[0, bytes) = src[0, bytes), cooperatively by the CTA.
__device__ __forceinline__ void cta_copy(char* dst, const char* src, int64_t bytes) {
  const bool v16 = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0;
  const bool v4 = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 3) == 0;
  int64_t done = 0;
  if (v16) {
    const int64_t n = bytes / 16;
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) d[i] = s[i];
    done = n * 16;
  } else if (v4) {
    const int64_t n = bytes / 4;
    const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
    uint32_t* d = reinterpret_cast<uint32_t*>(dst);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) d[i] = s[i];
    done = n * 4;
  }
  for (int64_t i = done + threadIdx.x; i < bytes; i += blockDim.x) dst[i] = src[i];
}

__global__ void __launch_bounds__(kLegacyThreads)
    scatter_copy_kernel(const int64_t* src_ptrs, const int64_t* lengths, const int64_t* offsets,
                        char* dst, int64_t row_bytes, int n) {
  const int seg = blockIdx.x;
  if (seg >= n) return;
  const int64_t len = lengths[seg];
  if (len <= 0) return;
  cta_copy(dst + offsets[seg] * row_bytes, reinterpret_cast<const char*>(src_ptrs[seg]),
           len * row_bytes);
}

__global__ void __launch_bounds__(kLegacyThreads)
    pos_override_kernel(int64_t* pos, const int64_t* starts, const int64_t* ends,
                        const int64_t* vals, int m) {
  const int r = blockIdx.x;
  if (r >= m) return;
  const int64_t e = ends[r], v = vals[r];
  for (int64_t i = starts[r] + threadIdx.x; i < e; i += blockDim.x) pos[i * 3] = v;
}

// History time mapping of one stored time (scatter_copy.cu:138-167): mode 1
// clamps the distance to the current time at rel_max; mode 2 compresses the
// part beyond rel_max by soft_factor, rounded to nearest (llrintf of the
// float product); the result is never negative.
__device__ __forceinline__ int64_t map_history_t(int64_t src_t, int64_t current_t, int mode,
                                                 int64_t rel_max, float soft_factor) {
  if (rel_max <= 0) return src_t;
  int64_t rel = current_t - src_t;
  if (rel < 0) rel = 0;
  int64_t t = src_t;
  if (mode == 1) {
    if (rel > rel_max) rel = rel_max;
    t = current_t - rel;
  } else if (mode == 2) {
    if (rel > rel_max) rel = rel_max + llrintf(float(rel - rel_max) * soft_factor);
    t = current_t - rel;
  }
  return t < 0 ? 0 : t;
}

__global__ void __launch_bounds__(kLegacyThreads)
    refresh_readout_kernel(const int64_t* src_k, const int64_t* src_v, const int64_t* src_pos,
                           const int64_t* offsets, const int64_t* lengths, const int64_t* flags,
                           const int64_t* rope_t, char* dst_k, char* dst_v, int64_t* dst_pos,
                           int64_t* dst_frame, int64_t row_bytes, int64_t current_t, int mode,
                           int64_t rel_max, float soft_factor, int n) {
  const int seg = blockIdx.x;
  if (seg >= n) return;
  const int64_t len = lengths[seg];
  if (len <= 0) return;
  const int64_t off = offsets[seg];
  cta_copy(dst_k + off * row_bytes, reinterpret_cast<const char*>(src_k[seg]), len * row_bytes);
  cta_copy(dst_v + off * row_bytes, reinterpret_cast<const char*>(src_v[seg]), len * row_bytes);
  const int64_t fl = flags[seg];
  const bool time_map = (fl & 1) != 0, frame_physical = (fl & 2) != 0, override_t = (fl & 4) != 0;
  const int64_t rt = rope_t[seg];
  const int64_t* sp = reinterpret_cast<const int64_t*>(src_pos[seg]);
  int64_t* dp = dst_pos + off * 3;
  int64_t* df = dst_frame + off;
  for (int64_t r = threadIdx.x; r < len; r += blockDim.x) {
    const int64_t t = sp[r * 3];
    const int64_t mt =
        override_t ? rt : time_map ? map_history_t(t, current_t, mode, rel_max, soft_factor) : t;
    dp[r * 3] = mt;
    dp[r * 3 + 1] = sp[r * 3 + 1];
    dp[r * 3 + 2] = sp[r * 3 + 2];
    df[r] = frame_physical ? t : mt;
  }
}

__global__ void __launch_bounds__(kLegacyThreads)
    anchor_store_write_frames_kernel(const char* k_seq, const char* v_seq, const int64_t* pos_seq,
                                     const int64_t* frame_desc, char* store_k, char* store_v,
                                     int64_t* store_pos, int64_t frame_seqlen, int64_t row_bytes,
                                     int n) {
  const int f = blockIdx.x;
  if (f >= n) return;
  const int64_t src_frame = frame_desc[2 * f], slot = frame_desc[2 * f + 1];
  if (src_frame < 0 || slot < 0) return;
  const int64_t bytes = frame_seqlen * row_bytes;
  cta_copy(store_k + slot * bytes, k_seq + src_frame * bytes, bytes);
  cta_copy(store_v + slot * bytes, v_seq + src_frame * bytes, bytes);
  cta_copy(reinterpret_cast<char*>(store_pos + slot * frame_seqlen * 3),
           reinterpret_cast<const char*>(pos_seq + src_frame * frame_seqlen * 3),
           frame_seqlen * 3 * int64_t(sizeof(int64_t)));
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_scatter_copy(const int64_t* src_ptrs, const int64_t* lengths,
                                const int64_t* offsets, void* dst, int64_t row_bytes,
                                int num_segments, pkv_stream_t stream) {
  if (num_segments == 0) return PKV_OK;
  if (num_segments < 0 || !src_ptrs || !lengths || !offsets || !dst || row_bytes < 0)
    return PKV_EINVAL;
  scatter_copy_kernel<<<num_segments, kLegacyThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      src_ptrs, lengths, offsets, static_cast<char*>(dst), row_bytes, num_segments);
  return launch_status();
}

extern "C" int pkv_pos_override(int64_t* pos, const int64_t* starts, const int64_t* ends,
                                const int64_t* vals, int num_ranges, pkv_stream_t stream) {
  if (num_ranges == 0) return PKV_OK;
  if (num_ranges < 0 || !pos || !starts || !ends || !vals) return PKV_EINVAL;
  pos_override_kernel<<<num_ranges, kLegacyThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      pos, starts, ends, vals, num_ranges);
  return launch_status();
}

extern "C" int pkv_refresh_readout_layout(
    const int64_t* src_ptrs_k, const int64_t* src_ptrs_v, const int64_t* src_ptrs_pos,
    const int64_t* offsets, const int64_t* lengths, const int64_t* flags,
    const int64_t* dynamic_rope_t, void* dst_k, void* dst_v, int64_t* dst_rope_pos,
    int64_t* dst_frame_ids, int64_t row_bytes, int64_t current_t, int mapping_mode,
    int64_t history_relative_t_max, float history_time_soft_factor, int num_segments,
    pkv_stream_t stream) {
  if (num_segments == 0) return PKV_OK;
  if (num_segments < 0 || !src_ptrs_k || !src_ptrs_v || !src_ptrs_pos || !offsets ||
      !lengths || !flags || !dynamic_rope_t || !dst_k || !dst_v || !dst_rope_pos ||
      !dst_frame_ids || row_bytes < 0 || mapping_mode < 0 || mapping_mode > 2)
    return PKV_EINVAL;
  refresh_readout_kernel<<<num_segments, kLegacyThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      src_ptrs_k, src_ptrs_v, src_ptrs_pos, offsets, lengths, flags, dynamic_rope_t,
      static_cast<char*>(dst_k), static_cast<char*>(dst_v), dst_rope_pos, dst_frame_ids,
      row_bytes, current_t, mapping_mode, history_relative_t_max, history_time_soft_factor,
      num_segments);
  return launch_status();
}

extern "C" int pkv_anchor_store_write_frames(const void* k_seq, const void* v_seq,
                                             const int64_t* pos_seq, const int64_t* frame_desc,
                                             void* store_k, void* store_v, int64_t* store_pos,
                                             int64_t frame_seqlen, int64_t row_bytes,
                                             int num_frames, pkv_stream_t stream) {
  if (num_frames == 0) return PKV_OK;
  if (num_frames < 0 || !k_seq || !v_seq || !pos_seq || !frame_desc || !store_k || !store_v ||
      !store_pos || frame_seqlen < 0 || row_bytes < 0)
    return PKV_EINVAL;
  anchor_store_write_frames_kernel<<<num_frames, kLegacyThreads, 0,
                                     static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char*>(k_seq), static_cast<const char*>(v_seq), pos_seq, frame_desc,
      static_cast<char*>(store_k), static_cast<char*>(store_v), store_pos, frame_seqlen,
      row_bytes, num_frames);
  return launch_status();
}
