// One layer's MegaCache.attend on the device: plan -> pack (RoPE fused) ->
// ragged attention, all enqueued on one stream with no host round trip.
//
// Reference behaviour: pyramidkv/_mega_cache.py:419-569 (plan via
// mega_plan_multi, slot offsets via _layer_offset_slot_global, fused-RoPE
// pack, flash_attn_varlen_func).  The planner writes its descriptors into the
// cache's scratch arena with the layer offset already applied, and
// cu_seqlens_k into the cache's own cu_seqlens_k buffer.
#include "pkv_common.cuh"
#include "pkv_internal.h"

using namespace pkv;

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
  const int rc = launch_plan(c, states_layer, layer, ts, num_chunks, sink_mode, cmin, cmax, lag,
                       /*check_capacity=*/1, /*add_layer_offset=*/1, c->cu_seqlens_k, sk, sg,
                       sln, dst, traw, tremap, total, token_counter, s);
  if (rc != PKV_OK) return rc;
  const bool rope = ft != nullptr || fy != nullptr || fx != nullptr;
  return launch_pack(c, sk, sg, sln, dst, int(N), rope ? tremap : nullptr, ft, ft_rows,
                     ft_cols, fy, fy_rows, fy_cols, fx, fx_rows, fx_cols, s);
}

extern "C" int pkv_attend_attention(const pkv_cache_t* c, const uint16_t* q,
                                    int64_t q_tok_stride, int64_t q_head_stride, int num_chunks,
                                    float scale, uint16_t* out, int64_t o_tok_stride,
                                    int64_t o_head_stride, pkv_stream_t stream) {
  if (!c || !q || !out || !c->cu_seqlens_k || !c->k_flat || !c->v_flat) return PKV_EINVAL;
  if (num_chunks <= 0) return PKV_OK;
  if (num_chunks > c->max_attend_chunks) return PKV_ECAPACITY;
  return launch_attention(q, q_tok_stride, q_head_stride, c->k_flat, c->v_flat,
                          c->max_pack_tokens, c->cu_seqlens_k, num_chunks, c->num_heads,
                          c->frame_seqlen, c->head_dim, scale, out, o_tok_stride, o_head_stride,
                          c->status, static_cast<cudaStream_t>(stream));
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
