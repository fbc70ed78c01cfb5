// One layer's MegaCache.attend on the device: plan -> pack (RoPE fused) ->
// ragged attention, all enqueued on one stream with no host round trip.
//
// Reference behaviour: pyramidkv/_mega_cache.py:419-569 (plan via
// mega_plan_multi, slot offsets via _layer_offset_slot_global, fused-RoPE
// pack, flash_attn_varlen_func).  The planner writes its descriptors into the
// cache's scratch arena with the layer offset already applied, and
// cu_seqlens_k into the cache's own cu_seqlens_k buffer.
#include <cstdlib>
#include <mutex>

#include "pkv_common.cuh"
#include "pkv_internal.h"
#include "pkv_plan.cuh"

using namespace pkv;

namespace {
// PKV_FUSED_PLAN_PACK=0 keeps the planner and the pack as two launches (the
// same results; for comparing the two).
bool fused_plan_pack() {
  static const bool on = [] {
    const char* e = std::getenv("PKV_FUSED_PLAN_PACK");
    return e == nullptr || e[0] != '0';
  }();
  return on;
}
}  // namespace

extern "C" int pkv_attend_pack(const pkv_cache_t* c, const uint8_t* states_layer, int layer,
                               int num_chunks, int64_t first_t, int sink_mode, int cmin,
                               int cmax, int lag, const float* ft, int ft_rows, int ft_cols,
                               const float* fy, int fy_rows, int fy_cols, const float* fx,
                               int fx_rows, int fx_cols, int64_t* token_counter,
                               pkv_stream_t stream) {
  if (!c || !states_layer || !c->scratch || !c->cu_seqlens_k) return PKV_EINVAL;
  if (num_chunks <= 0) return PKV_OK;
  if (num_chunks > c->max_attend_chunks || num_chunks > PKV_MAX_CHUNKS) return PKV_ECAPACITY;
  const ScratchLayout sl = scratch_layout(c);
  if (c->scratch_bytes < sl.bytes) return PKV_ECAPACITY;
  char* scr = static_cast<char*>(c->scratch);
  const int64_t H = c->num_heads;
  const int64_t S = plan_segments_per_head(c);
  const int64_t N = int64_t(num_chunks) * H * S;
  const int64_t NMAX = int64_t(c->max_attend_chunks) * H * S;
  int32_t* sk = reinterpret_cast<int32_t*>(scr + sl.plan);
  int32_t* sg = sk + NMAX;
  int32_t* sln = sg + NMAX;
  int32_t* dst = sln + NMAX;
  // 4 * NMAX int32 precede traw: 16-byte multiple, so traw stays 8-aligned
  int64_t* traw = reinterpret_cast<int64_t*>(dst + NMAX);
  int64_t* tremap = traw + NMAX;
  int64_t* total = reinterpret_cast<int64_t*>(scr + sl.plan_total);
  int64_t ts[PKV_MAX_CHUNKS];
  for (int i = 0; i < num_chunks; ++i) ts[i] = first_t + i;
  auto s = static_cast<cudaStream_t>(stream);
  const bool rope = ft != nullptr || fy != nullptr || fx != nullptr;
  if (!c->valid_count || !c->merge_token_count) return PKV_EINVAL;
  if (layer < 0 || layer >= c->num_layers) return PKV_EINVAL;
  {
    // one launch: each pack block derives the segment list from the staged
    // state records itself (the planner's rules), block 0 publishes cu_seqlens_k
    const PlanArgs pa = plan_args(c, states_layer, layer, ts, num_chunks, sink_mode, cmin, cmax,
                                  lag, /*check_capacity=*/1, /*add_layer_offset=*/1,
                                  c->cu_seqlens_k, total, token_counter, c->first_t_dev);
    if (fused_plan_pack() && plan_pack_fits(c, pa))
      return launch_pack_planned(c, pa, ft, ft_rows, ft_cols, fy, fy_rows, fy_cols, fx, fx_rows,
                                 fx_cols, s);
  }
  const int rc = launch_plan(c, states_layer, layer, ts, num_chunks, sink_mode, cmin, cmax, lag,
                       /*check_capacity=*/1, /*add_layer_offset=*/1, c->cu_seqlens_k, sk, sg,
                       sln, dst, traw, tremap, total, token_counter, s,
                       c->first_t_dev);
  if (rc != PKV_OK) return rc;
  return launch_pack(c, sk, sg, sln, dst, int(N), rope ? tremap : nullptr, ft, ft_rows,
                     ft_cols, fy, fy_rows, fy_cols, fx, fx_rows, fx_cols, s);
}

namespace {

// Ragged attention over the cache's last pack; with `use_scratch` the
// cache's scratch lends the attention kernel its split-unit workspace.
int attend_attention(const pkv_cache_t* c, const uint16_t* q, int64_t q_tok_stride,
                     int64_t q_head_stride, int num_chunks, float scale, uint16_t* out,
                     int64_t o_tok_stride, int64_t o_head_stride, bool use_scratch,
                     cudaStream_t stream) {
  if (!c || !q || !out || !c->cu_seqlens_k || !c->k_flat || !c->v_flat) return PKV_EINVAL;
  if (num_chunks <= 0) return PKV_OK;
  if (num_chunks > c->max_attend_chunks) return PKV_ECAPACITY;
  AttnWorkspace ws{};
  const AttnWorkspace* wsp = nullptr;
  if (use_scratch && c->scratch != nullptr) {
    const ScratchLayout sl = scratch_layout(c);
    if (c->scratch_bytes >= sl.bytes) {
      char* scr = static_cast<char*>(c->scratch);
      ws.part = reinterpret_cast<float*>(scr + sl.attn_part);
      ws.cnt = reinterpret_cast<int32_t*>(scr + sl.attn_cnt);
      ws.cnt_units = attn_units(c);
      wsp = &ws;
    }
  }
  return launch_attention(q, q_tok_stride, q_head_stride, c->k_flat, c->v_flat,
                          c->max_pack_tokens, c->cu_seqlens_k, num_chunks, c->num_heads,
                          c->frame_seqlen, c->head_dim, scale, out, o_tok_stride, o_head_stride,
                          c->status, wsp, stream);
}

}  // namespace

extern "C" int pkv_attend_attention(const pkv_cache_t* c, const uint16_t* q,
                                    int64_t q_tok_stride, int64_t q_head_stride, int num_chunks,
                                    float scale, uint16_t* out, int64_t o_tok_stride,
                                    int64_t o_head_stride, pkv_stream_t stream) {
  return attend_attention(c, q, q_tok_stride, q_head_stride, num_chunks, scale, out,
                          o_tok_stride, o_head_stride, /*use_scratch=*/true,
                          static_cast<cudaStream_t>(stream));
}

extern "C" int pkv_attend(const pkv_cache_t* c, const uint8_t* states_layer, int layer,
                          const uint16_t* q, int64_t q_tok_stride, int64_t q_head_stride,
                          int num_chunks, int64_t first_t, int sink_mode, int cmin, int cmax,
                          int lag, const float* ft, int ft_rows, int ft_cols, const float* fy,
                          int fy_rows, int fy_cols, const float* fx, int fx_rows, int fx_cols,
                          float scale, uint16_t* out, int64_t o_tok_stride,
                          int64_t o_head_stride, int64_t* token_counter, pkv_stream_t stream) {
  if (!q || !out) return PKV_EINVAL;
  const int rc = pkv_attend_pack(c, states_layer, layer, num_chunks, first_t, sink_mode, cmin,
                                 cmax, lag, ft, ft_rows, ft_cols, fy, fy_rows, fy_cols, fx,
                                 fx_rows, fx_cols, token_counter, stream);
  if (rc != PKV_OK) return rc;
  return pkv_attend_attention(c, q, q_tok_stride, q_head_stride, num_chunks, scale, out,
                              o_tok_stride, o_head_stride, stream);
}

// ---------------------------------------------------------------------------
// pkv_attend_noalloc: pkv_attend for callers that cannot allocate device
// memory.  A host runtime that owns the device's memory pool lends this
// library only the cache and each call's inputs and outputs, and a serving
// loop cannot afford a cudaMalloc, which may synchronise the device and stall
// the other streams.  The only scratch pkv_attend needs beyond the cache's own
// buffers is the planner's descriptor arrays (for shapes the self-planning
// pack does not cover; otherwise just the token total); here they live in the
// file-scope array below, which every GPU that loads libpkv.so holds until the
// process exits, and cache->scratch is not used (it may be NULL).
//
// In host code the array's name is a host-side stand-in, not its device
// address.  The address is looked up with cudaGetSymbolAddress once per
// device, with that device current, on the first call on that device; make
// that first call before any stream capture.  The planner writes every entry
// that the pack later reads, so nothing in the array needs clearing, but all
// calls share it and it keeps the last call's contents: calls whose launches
// overlap on the GPU (different streams, or several host threads on one
// device without ordering) race on it.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[PKV_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
char* g_noalloc_ptr[kNoallocMaxDevices] = {};

// Bytes of planner output for n segments: sk/sg/sl/dst (int32), traw/tremap
// (int64), one int64 total.
int64_t noalloc_plan_bytes(int64_t n) { return n * 4 * 4 + n * 8 * 2 + 8; }

// Device address of g_noalloc_scratch on the current device, nullptr on error.
char* noalloc_scratch() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoallocMaxDevices) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return nullptr;
    }
    g_noalloc_ptr[dev] = static_cast<char*>(p);
  }
  return g_noalloc_ptr[dev];
}

}  // namespace

extern "C" int pkv_attend_noalloc(const pkv_cache_t* c, const uint8_t* states_layer, int layer,
                                  const uint16_t* q, int64_t q_tok_stride,
                                  int64_t q_head_stride, int num_chunks, int64_t first_t,
                                  int sink_mode, int cmin, int cmax, int lag, const float* ft,
                                  int ft_rows, int ft_cols, const float* fy, int fy_rows,
                                  int fy_cols, const float* fx, int fx_rows, int fx_cols,
                                  float scale, uint16_t* out, int64_t o_tok_stride,
                                  int64_t o_head_stride, int64_t* token_counter,
                                  pkv_stream_t stream) {
  if (!c || !states_layer || !q || !out || !c->cu_seqlens_k) return PKV_EINVAL;
  if (num_chunks <= 0) return PKV_OK;
  if (num_chunks > c->max_attend_chunks || num_chunks > PKV_MAX_CHUNKS) return PKV_ECAPACITY;
  const int64_t n = int64_t(num_chunks) * c->num_heads * plan_segments_per_head(c);
  if (n <= 0 || noalloc_plan_bytes(n) > PKV_NOALLOC_SCRATCH_BYTES) return PKV_ENOALLOC_LIMIT;
  char* region = noalloc_scratch();
  if (region == nullptr) return PKV_ELAUNCH;
  int32_t* sk = reinterpret_cast<int32_t*>(region);
  int32_t* sg = sk + n;
  int32_t* sln = sg + n;
  int32_t* dst = sln + n;
  int64_t* traw = reinterpret_cast<int64_t*>(dst + n);  // 16n bytes in: 8-aligned
  int64_t* tremap = traw + n;
  int64_t* total = tremap + n;
  int64_t ts[PKV_MAX_CHUNKS];
  for (int i = 0; i < num_chunks; ++i) ts[i] = first_t + i;
  auto s = static_cast<cudaStream_t>(stream);
  int rc = PKV_OK;
  if (!c->valid_count || !c->merge_token_count) return PKV_EINVAL;
  if (layer < 0 || layer >= c->num_layers) return PKV_EINVAL;
  const PlanArgs pa = plan_args(c, states_layer, layer, ts, num_chunks, sink_mode, cmin, cmax,
                                lag, /*check_capacity=*/1, /*add_layer_offset=*/1,
                                c->cu_seqlens_k, total, token_counter, c->first_t_dev);
  if (fused_plan_pack() && plan_pack_fits(c, pa)) {
    // the pack plans for itself: only the token total lands in the array
    rc = launch_pack_planned(c, pa, ft, ft_rows, ft_cols, fy, fy_rows, fy_cols, fx, fx_rows,
                             fx_cols, s);
  } else {
    rc = launch_plan(c, states_layer, layer, ts, num_chunks, sink_mode, cmin, cmax, lag,
                     /*check_capacity=*/1, /*add_layer_offset=*/1, c->cu_seqlens_k, sk, sg,
                     sln, dst, traw, tremap, total, token_counter, s, c->first_t_dev);
    if (rc != PKV_OK) return rc;
    const bool rope = ft != nullptr || fy != nullptr || fx != nullptr;
    rc = launch_pack(c, sk, sg, sln, dst, int(n), rope ? tremap : nullptr, ft, ft_rows, ft_cols,
                     fy, fy_rows, fy_cols, fx, fx_rows, fx_cols, s);
  }
  if (rc != PKV_OK) return rc;
  // one CTA per attention unit: the split-unit workspace would be scratch
  return attend_attention(c, q, q_tok_stride, q_head_stride, num_chunks, scale, out,
                          o_tok_stride, o_head_stride, /*use_scratch=*/false, s);
}
