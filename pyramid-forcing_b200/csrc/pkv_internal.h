// Internal (non-ABI) launch descriptors shared between the library's .cu files.
#pragma once

#include <cuda_runtime.h>

#include "pkv_common.cuh"

namespace pkv {

// One layer's merge accumulation (see pkv_merge.cu).  New K/V token t of
// frame f, head h, element d is at base + f*frame_stride + h*head_stride +
// t*tok_stride + d.  new_pos == nullptr means positions are generated as
// (first_t + f, t / pos_width, t % pos_width).
struct MergeLaunch {
  const HeadState* states;
  const uint16_t* new_k;
  const uint16_t* new_v;
  int64_t frame_stride, head_stride, tok_stride;
  const int64_t* new_pos;
  int pos_width;
  int64_t first_t;
  const int64_t* t_dev;  // device first_t (nullable): replaces first_t when set
  const int32_t *dkind, *dslot, *dfin, *dnew;
  float *acc_k, *acc_v;
  int64_t* acc_pos;
  int32_t* acc_gid;
  float* acc_tpg;
  int32_t* acc_ng;
  uint16_t *mk, *mv;
  int64_t* mpos;
  int32_t* mtc;
  int H, F, FSEQ, D, MMA, MMB, MTPA;
  int32_t* status;
};

int launch_merge(const MergeLaunch& m, cudaStream_t stream);

}  // namespace pkv

namespace pkv {

int launch_plan(const pkv_cache_t* c, const uint8_t* states_layer, int layer,
                const int64_t* current_t, int num_chunks, int sink_mode, int cmin, int cmax,
                int lag, int check_capacity, int add_layer_offset, int32_t* cu, int32_t* sk,
                int32_t* sg, int32_t* sl, int32_t* dst, int64_t* traw, int64_t* tremap,
                int64_t* total, int64_t* counter, cudaStream_t stream,
                const int64_t* t_dev = nullptr);

int launch_pack(const pkv_cache_t* c, const int32_t* sk, const int32_t* sg, const int32_t* sl,
                const int32_t* dst, int n_seg, const int64_t* tremap, const float* ft,
                int ft_rows, int ft_cols, const float* fy, int fy_rows, int fy_cols,
                const float* fx, int fx_rows, int fx_cols, cudaStream_t stream);

// Ragged-attention workspace: partial-result slots and arrival counters for
// `cnt_units` units (zeroed before the first launch; each launch leaves them
// zero).  nullptr: one CTA per unit, nothing split.
struct AttnWorkspace {
  float* part;
  int32_t* cnt;
  int64_t cnt_units;
};

int launch_attention(const uint16_t* q, int64_t q_rs, int64_t q_hs, const uint16_t* k,
                     const uint16_t* v, int64_t kv_rows, const int32_t* cu, int num_chunks,
                     int H, int rows_per_chunk, int D, float scale, uint16_t* out, int64_t o_rs,
                     int64_t o_hs, int32_t* status, const AttnWorkspace* ws,
                     cudaStream_t stream);

}  // namespace pkv
