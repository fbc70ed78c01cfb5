// Layout copies around the head-parallel all-to-all.
//
// A head-parallel layer step over n ranks moves each rank's token shard of
// Q, K and V ([L/n tokens, H heads, D]) to the ranks that own the heads, and
// the attention output back.  The all-to-all itself is NCCL over NVLink; what
// this file provides is the one-pass gather into the send buffer (chunks by
// destination rank, Q/K/V interleaved per token so the receiver can read each
// of them as a strided [L, H/n, D] view without another copy) and the
// one-pass scatter of the received output into the model's [L/n, H, D]
// layout.  Both are the same operation: copy `count` sources of
// [tokens, groups, group_elems] chunks to a destination with arbitrary chunk
// strides.  The destination of each group may also be its own base pointer:
// the buffer of another GPU mapped into this process (symmetric memory), so
// the same pass writes every rank's share straight into that rank's receive
// buffer over NVLink (plain stores, no copy engine, no staging).  No
// counterpart in the reference, which runs the cache on one GPU.
#include "pkv_common.cuh"

namespace pkv {

constexpr int kMaxCopySources = 4;
constexpr int kMaxCopyGroups = 8;

struct ChunkCopy {
  const uint16_t* src[kMaxCopySources];
  int64_t src_ts[kMaxCopySources], src_gs[kMaxCopySources];
  uint16_t* dst;
  uint16_t* dst_group[kMaxCopyGroups];  // per-group bases (peer buffers), or all null
  int64_t dst_ts, dst_gs, dst_is;
  int64_t tokens;
  int groups, count, group_elems;
};

// One thread per 16-byte vector (kVec) or per element; chunk-major order so
// the threads of a warp read and write contiguous bytes.
template <bool kVec>
__global__ void __launch_bounds__(256) chunk_copy_kernel(ChunkCopy c) {
  const int per = kVec ? c.group_elems / 8 : c.group_elems;
  const int64_t chunks = c.tokens * c.groups * c.count;
  const int64_t total = chunks * per;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t chunk = idx / per;
    const int e = int(idx - chunk * per);
    // chunk order (token, group, source): a token's groups of one source are
    // neighbours in the source and a token's sources in the destination
    const int i = int(chunk % c.count);
    const int64_t tg = chunk / c.count;
    const int g = int(tg % c.groups);
    const int64_t t = tg / c.groups;
    const uint16_t* s = c.src[i] + t * c.src_ts[i] + g * c.src_gs[i];
    uint16_t* d = (c.dst_group[0] != nullptr ? c.dst_group[g] : c.dst + g * c.dst_gs) +
                  t * c.dst_ts + i * c.dst_is;
    if (kVec)
      reinterpret_cast<uint4*>(d)[e] = __ldg(reinterpret_cast<const uint4*>(s) + e);
    else
      d[e] = __ldg(s + e);
  }
}

}  // namespace pkv

using namespace pkv;

extern "C" int pkv_chunk_copy(const uint16_t* const* srcs, const int64_t* src_tok_strides,
                              const int64_t* src_group_strides, int count, uint16_t* dst,
                              int64_t dst_tok_stride, int64_t dst_group_stride,
                              int64_t dst_src_stride, int64_t tokens, int groups,
                              int group_elems, pkv_stream_t stream) {
  if (tokens == 0 || groups == 0 || count == 0 || group_elems == 0) return PKV_OK;
  if (!srcs || !src_tok_strides || !src_group_strides || !dst || count < 0 ||
      count > kMaxCopySources || tokens < 0 || groups < 0 || group_elems < 0)
    return PKV_EINVAL;
  ChunkCopy c{};
  bool vec = group_elems % 8 == 0 && reinterpret_cast<uintptr_t>(dst) % 16 == 0 &&
             dst_tok_stride % 8 == 0 && dst_group_stride % 8 == 0 && dst_src_stride % 8 == 0;
  for (int i = 0; i < count; ++i) {
    if (!srcs[i]) return PKV_EINVAL;
    c.src[i] = srcs[i];
    c.src_ts[i] = src_tok_strides[i];
    c.src_gs[i] = src_group_strides[i];
    vec = vec && reinterpret_cast<uintptr_t>(srcs[i]) % 16 == 0 && c.src_ts[i] % 8 == 0 &&
          c.src_gs[i] % 8 == 0;
  }
  c.dst = dst;
  c.dst_ts = dst_tok_stride;
  c.dst_gs = dst_group_stride;
  c.dst_is = dst_src_stride;
  c.tokens = tokens;
  c.groups = groups;
  c.count = count;
  c.group_elems = group_elems;
  const int64_t total = tokens * groups * count * (vec ? group_elems / 8 : group_elems);
  int64_t grid = (total + 255) / 256;
  const int64_t cap = int64_t(sm_count()) * 8;
  if (grid > cap) grid = cap;
  auto s = static_cast<cudaStream_t>(stream);
  if (vec)
    chunk_copy_kernel<true><<<int(grid), 256, 0, s>>>(c);
  else
    chunk_copy_kernel<false><<<int(grid), 256, 0, s>>>(c);
  return launch_status();
}

extern "C" int pkv_chunk_copy_peers(const uint16_t* const* srcs, const int64_t* src_tok_strides,
                                    const int64_t* src_group_strides, int count,
                                    uint16_t* const* dsts, int64_t dst_tok_stride,
                                    int64_t dst_src_stride, int64_t tokens, int groups,
                                    int group_elems, pkv_stream_t stream) {
  if (tokens == 0 || groups == 0 || count == 0 || group_elems == 0) return PKV_OK;
  if (!srcs || !src_tok_strides || !src_group_strides || !dsts || count < 0 ||
      count > kMaxCopySources || groups < 0 || groups > kMaxCopyGroups || tokens < 0 ||
      group_elems < 0)
    return PKV_EINVAL;
  ChunkCopy c{};
  bool vec = group_elems % 8 == 0 && dst_tok_stride % 8 == 0 && dst_src_stride % 8 == 0;
  for (int g = 0; g < groups; ++g) {
    if (!dsts[g]) return PKV_EINVAL;
    c.dst_group[g] = dsts[g];
    vec = vec && reinterpret_cast<uintptr_t>(dsts[g]) % 16 == 0;
  }
  for (int i = 0; i < count; ++i) {
    if (!srcs[i]) return PKV_EINVAL;
    c.src[i] = srcs[i];
    c.src_ts[i] = src_tok_strides[i];
    c.src_gs[i] = src_group_strides[i];
    vec = vec && reinterpret_cast<uintptr_t>(srcs[i]) % 16 == 0 && c.src_ts[i] % 8 == 0 &&
          c.src_gs[i] % 8 == 0;
  }
  c.dst = dsts[0];
  c.dst_ts = dst_tok_stride;
  c.dst_gs = 0;
  c.dst_is = dst_src_stride;
  c.tokens = tokens;
  c.groups = groups;
  c.count = count;
  c.group_elems = group_elems;
  const int64_t total = tokens * groups * count * (vec ? group_elems / 8 : group_elems);
  int64_t grid = (total + 255) / 256;
  const int64_t cap = int64_t(sm_count()) * 8;
  if (grid > cap) grid = cap;
  auto s = static_cast<cudaStream_t>(stream);
  if (vec)
    chunk_copy_kernel<true><<<int(grid), 256, 0, s>>>(c);
  else
    chunk_copy_kernel<false><<<int(grid), 256, 0, s>>>(c);
  return launch_status();
}
