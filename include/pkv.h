/*
 * pkv.h -- C ABI of the B200 MegaCache library (libpkv.so).
 *
 * The per-step KV-cache path of Pyramid Forcing's causal Wan2.1 DiT:
 * head-aware [sink + middle + recent] cache update (cyclic / stride / lag /
 * merge middle strategies chosen per head), the plan + pack of the ragged
 * per-head caches with RoPE remapped into the training position range, and
 * the ragged-cache attention over that layout.
 *
 * Every entry point takes device pointers, sizes and a CUDA stream (as
 * `void*`, a cudaStream_t), enqueues its kernels on that stream and returns
 * a status code (PKV_OK or a PKV_E* value).  No entry point synchronises the
 * stream, reads device memory back to the host or allocates memory.  Errors a
 * kernel detects on the device (an out-of-range slot, a pack-workspace
 * overflow, a bad descriptor) are OR-ed into a caller-supplied sticky status
 * word (`int32_t *status`, PKV_ST_* bits) instead of faulting; the host reads
 * it whenever it chooses to synchronise.
 *
 * bf16 tensors travel as `uint16_t` bit patterns.
 *
 * Each declaration names the reference interface it replaces (paths are
 * inside the reference project).
 */
#ifndef PKV_H_
#define PKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes ------------------------------------------------------- */
#define PKV_OK 0
#define PKV_EINVAL 1     /* bad argument (null pointer, size out of range)   */
#define PKV_ELAUNCH 2    /* the CUDA launch itself failed                    */
#define PKV_ECAPACITY 3  /* a request cannot fit a compiled or sized bound   */
#define PKV_EUNSUPPORTED 4
#define PKV_ENOALLOC_LIMIT 5 /* plan exceeds PKV_NOALLOC_SCRATCH_BYTES        */

/* ---- sticky device status bits ----------------------------------------- */
#define PKV_ST_PACK_OVERFLOW 0x1   /* plan total > pack workspace capacity   */
#define PKV_ST_SLOT_RANGE 0x2      /* a descriptor addressed a slot outside its pool */
#define PKV_ST_STATE_RANGE 0x4     /* a PerHeadState field out of its compiled bound */
#define PKV_ST_MERGE_DUP 0x8       /* duplicate merge frame (skipped)        */
#define PKV_ST_BAD_KIND 0x10       /* unknown descriptor kind                */
#define PKV_ST_RECENT_RANGE 0x20   /* more recent writes than recent slots   */
#define PKV_ST_TIMEOUT 0x40        /* a bounded device wait expired; kernel returned */

/* Compiled bounds of the per-head strategy state
 * (pyramidkv/csrc/anchor_store.cuh:39-45,148). */
#define PKV_MAX_PHASE 6
#define PKV_MAX_BUCKET 4
#define PKV_MAX_T_KEYED 24
#define PKV_MAX_LAG_OFFSETS 4
#define PKV_MAX_MERGE_BLOCKS 6
#define PKV_MAX_MERGE_ACTIVE 2
#define PKV_MAX_MERGE_BLOCK_FRAMES 4
#define PKV_MAX_MERGE_TOKENS 420
#define PKV_MAX_CHUNKS 64

typedef void *pkv_stream_t; /* a cudaStream_t */

/*
 * The cache storage of every layer, as owned by the reference's
 * PyramidKVCacheManager (pyramidkv/csrc/pyramidkv_manager.h:62-199,
 * pyramidkv_manager.cc:36-137) plus the committed snapshot that
 * MegaCacheCtx keeps (pyramidkv/_mega_cache.py:72-89).  All pointers are
 * device pointers to contiguous arrays with the shapes noted.
 */
typedef struct pkv_cache {
    int32_t num_layers, num_heads, head_dim, frame_seqlen;   /* L, H, D, F      */
    int32_t max_sink, max_middle, max_recent;                /* slots per kind  */
    int32_t max_merge_blocks, max_merge_active, max_merge_tokens; /* MMB, MMA, MTPA */
    int32_t max_attend_chunks, spatial_width;
    int64_t max_pack_tokens;        /* rows of k_flat / v_flat / pos_flat     */

    uint16_t *sink_k, *sink_v;      /* [L, H, max_sink,   F, D] bf16          */
    uint16_t *middle_k, *middle_v;  /* [L, H, max_middle, F, D] bf16          */
    uint16_t *recent_k, *recent_v;  /* [L, H, max_recent, F, D] bf16          */
    int64_t *sink_pos, *middle_pos, *recent_pos; /* [L, H, slots, F, 3]       */
    int64_t *valid_count;           /* [L, H, 3] (sink, middle, recent)       */

    uint16_t *merge_k, *merge_v;    /* [L, H, MMB, MTPA, D] bf16              */
    int64_t *merge_pos;             /* [L, H, MMB, MTPA, 3]                   */
    int32_t *merge_token_count;     /* [L, H, MMB]                            */
    float *accum_sum_k, *accum_sum_v; /* [L, H, MMA, MTPA, D] fp32            */
    int64_t *accum_pos;             /* [L, H, MMA, MTPA, 3]                   */
    int32_t *accum_group_ids;       /* [L, H, MMA, F]                         */
    float *accum_tokens_per_group;  /* [L, H, MMA, MTPA]                      */
    int32_t *accum_num_groups;      /* [L, H, MMA]                            */

    uint16_t *k_flat, *v_flat;      /* [max_pack_tokens, D] bf16              */
    int64_t *pos_flat;              /* [max_pack_tokens, 3]                   */
    int32_t *cu_seqlens_k;          /* [max_attend_chunks * H + 1]            */

    int64_t *committed_vc;          /* [L, H, 3]                              */
    uint16_t *committed_recent_k, *committed_recent_v; /* like recent_k/v     */
    int64_t *committed_recent_pos;  /* like recent_pos                        */
    int64_t *sink_caps;             /* [L, H] per-head sink capacity          */

    void *scratch;                  /* pkv_scratch_bytes() bytes, 256-aligned */
    int64_t scratch_bytes;
    int32_t *status;                /* sticky PKV_ST_* word (nullable)        */
    /* Device int64 (nullable).  When set, pkv_cache_update, pkv_attend,
     * pkv_attend_pack and pkv_attend_noalloc read the block's first latent
     * frame from here when their kernels run, in place of their first_t
     * argument, so one captured CUDA graph of a layer step replays for every
     * block (write the frame into it before each replay).  No counterpart in
     * the reference, whose planner takes the time on the host. */
    const int64_t *first_t_dev;
} pkv_cache_t;

/* sizeof(PerHeadState), the 600-byte per-(layer, head) strategy record.
 * Replaces: torch.ops.adahead.mega_state_perhead_size
 * (pyramidkv/csrc/scatter_copy_bind.cpp:402-404). */
int64_t pkv_state_perhead_size(void);

/* Bytes of scratch the fused update / attend paths need for this cache. */
int64_t pkv_scratch_bytes(const pkv_cache_t *cache);

/* Human-readable text for a return code. */
const char *pkv_error_string(int code);

/*
 * Per-head strategy state machine over one layer's states.
 * Replaces: adahead::launch_mega_state_update
 * (pyramidkv/csrc/anchor_store_update.cu:324-374), op mega_state_update.
 * states: uint8 [num_heads * 600], mutated.  new_t_vals: int64 [frames].
 * desc_*: int32 [num_heads * frames], head-major.
 */
int pkv_mega_state_update(uint8_t *states, const int64_t *new_t_vals,
                          int32_t *desc_dst_kind, int32_t *desc_dst_slot,
                          int32_t *desc_src_frame, int32_t *desc_src_head,
                          int32_t *desc_merge_accum_slot, int32_t *desc_merge_local_idx,
                          int32_t *desc_merge_finalize_completed_idx,
                          int32_t *desc_merge_is_new_block, int num_heads,
                          int frames_in_block, int pass_kind, int32_t *status,
                          pkv_stream_t stream);

/*
 * Copy incoming frames into pool slots by descriptor.
 * Replaces: adahead::launch_pyramidkv_update
 * (pyramidkv/csrc/pyramidkv_update.cu:115-189), op pyramidkv_update.
 * new_k/new_v: bf16 [frames, H, F, D]; new_pos: int64 [frames, H, F, 3] or
 * NULL.  dst_kind 0/1/2 = sink/middle/recent, <0 = skip; dst_slot_global
 * indexes the [L*H*slots] rows of that pool.
 */
int pkv_update_frames(const pkv_cache_t *cache, const uint16_t *new_k,
                      const uint16_t *new_v, const int64_t *new_pos,
                      const int32_t *dst_kind, const int32_t *dst_slot_global,
                      const int32_t *src_frame_in_block, const int32_t *src_head,
                      int num_ops, pkv_stream_t stream);

/*
 * Merge-strategy K/V accumulation and finalize over one layer's slices.
 * Replaces: adahead::launch_mega_merge_accum
 * (pyramidkv/csrc/mega_merge_accum.cu:268-340), op mega_merge_accum.
 * new_k/new_v: bf16 [F, H, FSEQ, D]; new_pos: int64 [F, H, FSEQ, 3];
 * desc_*: int32 [H * F]; accum_* / merge_*: this layer's [H, ...] slices.
 */
int pkv_merge_accum(const uint8_t *states, const uint16_t *new_k, const uint16_t *new_v,
                    const int64_t *new_pos, const int32_t *desc_dst_kind,
                    const int32_t *desc_merge_accum_slot,
                    const int32_t *desc_merge_finalize_completed_idx,
                    const int32_t *desc_merge_is_new_block, float *accum_sum_k,
                    float *accum_sum_v, int64_t *accum_pos, int32_t *accum_group_ids,
                    float *accum_tokens_per_group, int32_t *accum_num_groups,
                    uint16_t *merge_k_pool, uint16_t *merge_v_pool, int64_t *merge_pos_pool,
                    int32_t *merge_token_count, int H, int F, int FSEQ, int D, int MMA,
                    int MMB, int MTPA, int32_t *status, pkv_stream_t stream);

/*
 * Device planner: per (chunk, head) segment list of the ragged K/V layout,
 * cu_seqlens_k by prefix scan, dst offsets and the RoPE time remap, with no
 * host round trip.  Output values are identical to the reference's host
 * planner.
 * Replaces: mega_plan / mega_plan_multi (pyramidkv/csrc/mega_plan.cc:286-407,
 * :510-654), ops mega_plan and mega_plan_multi.
 * current_t: HOST array [num_chunks] (<= PKV_MAX_CHUNKS), copied into the
 * launch parameters.  Outputs: cu [num_chunks*H+1], sk/sg/sl/dst int32 and
 * traw/tremap int64 of [num_chunks*H*(max_sink+max_middle+max_recent+MMB)].
 * check_capacity != 0 flags PKV_ST_PACK_OVERFLOW when the total exceeds
 * cache->max_pack_tokens.  add_layer_offset != 0 also applies the per-kind
 * layer offset of pyramidkv/_mega_attention.py:349-385 to sg.
 * total_tokens (device int64, nullable) receives the packed token total;
 * token_counter (device int64, nullable) accumulates it across calls.
 */
int pkv_plan(const pkv_cache_t *cache, const uint8_t *states_layer, int layer_idx,
             const int64_t *current_t, int num_chunks, int sink_mode_code,
             int sink_clamp_min, int sink_clamp_max, int decoupled_sink_lag,
             int check_capacity, int add_layer_offset, int32_t *cu_seqlens_k,
             int32_t *src_kind, int32_t *src_slot_global, int32_t *seg_lengths,
             int32_t *dst_token_offsets, int64_t *anchor_t_raw, int64_t *anchor_t_remap,
             int64_t *total_tokens, int64_t *token_counter, pkv_stream_t stream);

/*
 * Legacy all-layer plan: per (layer, head) the descriptors of its sink,
 * recent and middle segments (in that order), each from the head's slot 0
 * over valid_count[kind] frames, or kind -1 when the kind is empty; offsets
 * head-major over all layers.
 * Replaces: adahead::pyramidkv_plan (pyramidkv/csrc/pyramidkv_plan.cc:48-173),
 * op pyramidkv_plan (M1.4), which builds them on the host.
 * Outputs (device int32): cu_seqlens_k [L*H+1]; src_kind, src_slot_global,
 * seg_lengths, dst_token_offsets [L*H*3].  Segments may span several slots:
 * pkv_pack copies them whole (they stay inside the pool).
 */
int pkv_legacy_plan(const pkv_cache_t *cache, int32_t *cu_seqlens_k, int32_t *src_kind,
                    int32_t *src_slot_global, int32_t *seg_lengths,
                    int32_t *dst_token_offsets, pkv_stream_t stream);

/*
 * Gather pool segments into the flat K/V/pos workspace, rotating K by the 3D
 * RoPE at (tremap >= 0 ? tremap : stored t, stored y, stored x).
 * Replaces: adahead::launch_pyramidkv_pack
 * (pyramidkv/csrc/pyramidkv_pack.cu:189-311), op pyramidkv_pack.
 * anchor_t_remap == NULL or all tables NULL: plain copy.  Tables are fp32
 * [rows, cols*2] (re, im interleaved).
 */
int pkv_pack(const pkv_cache_t *cache, const int32_t *src_kind,
             const int32_t *src_slot_global, const int32_t *seg_lengths,
             const int32_t *dst_token_offsets, int num_segments,
             const int64_t *anchor_t_remap, const float *freqs_ft, int ft_rows, int ft_cols,
             const float *freqs_fy, int fy_rows, int fy_cols, const float *freqs_fx,
             int fx_rows, int fx_cols, pkv_stream_t stream);

/*
 * Ragged non-causal attention: for every (chunk c, head h) the
 * rows_per_chunk query rows attend the keys k[cu[c*H+h] : cu[c*H+h+1]].
 * Query row r of (c, h) is at q + (c*rows_per_chunk + r)*q_row_stride +
 * h*q_head_stride (elements); the output uses the same addressing with the
 * o_* strides.  k/v: bf16 [kv_rows, head_dim] rows.  fp32 softmax and
 * accumulation, bf16 output.
 * Replaces: flash_attn.flash_attn_varlen_func as called at
 * pyramidkv/_mega_cache.py:529-569 (including the Q/O permutes there) and
 * pyramidkv/_mega_attention.py:106-159.
 */
int pkv_attention(const uint16_t *q, int64_t q_row_stride, int64_t q_head_stride,
                  const uint16_t *k, const uint16_t *v, int64_t kv_rows,
                  const int32_t *cu_seqlens_k, int num_chunks, int num_heads,
                  int rows_per_chunk, int head_dim, float softmax_scale, uint16_t *out,
                  int64_t o_row_stride, int64_t o_head_stride, pkv_stream_t stream);

/*
 * pkv_attention with a caller-owned workspace, which lets the kernel balance
 * the work over the SMs: one persistent CTA per SM, the longest
 * (segment, query-tile pair) units run whole and the rest are cut into equal
 * per-SM shares, a unit cut between SMs being finished by whichever share
 * ends last (fp32 partials in the workspace; no SM waits for another).
 * Results match pkv_attention within the fp32-accumulation tolerance (the
 * split units sum their keys in a different order).  workspace: device
 * memory of at least pkv_attention_workspace_bytes(...) bytes, 256-byte
 * aligned, zero-filled before its first use; every launch leaves it ready for
 * the next (its counters back at zero), so it is reused without clearing.
 * Launches sharing a workspace must not overlap on the GPU.  A launch that
 * ended on a device timeout (PKV_ST_TIMEOUT) can leave counters set: zero the
 * workspace again before reuse.  workspace == NULL runs pkv_attention.
 * Replaces: flash_attn.flash_attn_varlen_func at pyramidkv/_mega_cache.py:550-559
 * (as pkv_attention; MegaCache.attend uses this path with the cache's scratch).
 */
int64_t pkv_attention_workspace_bytes(int num_chunks, int num_heads, int rows_per_chunk);
int pkv_attention_ws(const uint16_t *q, int64_t q_row_stride, int64_t q_head_stride,
                     const uint16_t *k, const uint16_t *v, int64_t kv_rows,
                     const int32_t *cu_seqlens_k, int num_chunks, int num_heads,
                     int rows_per_chunk, int head_dim, float softmax_scale, uint16_t *out,
                     int64_t o_row_stride, int64_t o_head_stride, void *workspace,
                     int64_t workspace_bytes, pkv_stream_t stream);

/*
 * One layer's MegaCache.update on the device: restore the committed
 * valid_count / recent pool, route each head's frames to sink or recent (FIFO
 * on overflow), run the strategy state machine and the middle / merge writes
 * on a clean pass, and commit.  Visible results (pools, valid_count, the
 * committed snapshot, states) equal the reference's.
 * Replaces: MegaCache.update (pyramidkv/_mega_cache.py:136-414).
 * new_k/new_v: bf16, token t of frame f, head h at
 * base + (f*F + t)*tok_stride + h*head_stride (the [1, L_in, H, D] layout).
 * states: uint8 [L, H*600].  pass_kind 0 = noisy, 1 = clean.
 */
int pkv_cache_update(const pkv_cache_t *cache, uint8_t *states, int layer_idx,
                     const uint16_t *new_k, const uint16_t *new_v, int64_t tok_stride,
                     int64_t head_stride, int frames, int64_t first_t, int pass_kind,
                     int has_merge_head, pkv_stream_t stream);

/*
 * One layer's MegaCache.attend: device plan + pack (RoPE fused) + ragged
 * attention, reading Q in the caller's [1, L_q, H, D] layout and writing O in
 * the same layout.
 * Replaces: MegaCache.attend (pyramidkv/_mega_cache.py:419-569).
 */
int pkv_attend(const pkv_cache_t *cache, const uint8_t *states_layer, int layer_idx,
               const uint16_t *q, int64_t q_tok_stride, int64_t q_head_stride, int num_chunks,
               int64_t first_t, int sink_mode_code, int sink_clamp_min, int sink_clamp_max,
               int decoupled_sink_lag, const float *freqs_ft, int ft_rows, int ft_cols,
               const float *freqs_fy, int fy_rows, int fy_cols, const float *freqs_fx,
               int fx_rows, int fx_cols, float softmax_scale, uint16_t *out,
               int64_t o_tok_stride, int64_t o_head_stride, int64_t *token_counter,
               pkv_stream_t stream);

/*
 * The two halves of pkv_attend, for callers that schedule or time them
 * separately: pkv_attend_pack runs the planner (layer offsets applied,
 * capacity checked, cu_seqlens_k written to cache->cu_seqlens_k) and the
 * RoPE-fused pack into cache->k_flat / v_flat; pkv_attend_attention runs the
 * ragged attention over what the last pkv_attend_pack on this cache wrote.
 * Replaces: the same two stages of MegaCache.attend
 * (pyramidkv/_mega_cache.py:466-523 and :525-569).
 */
int pkv_attend_pack(const pkv_cache_t *cache, const uint8_t *states_layer, int layer_idx,
                    int num_chunks, int64_t first_t, int sink_mode_code, int sink_clamp_min,
                    int sink_clamp_max, int decoupled_sink_lag, const float *freqs_ft,
                    int ft_rows, int ft_cols, const float *freqs_fy, int fy_rows, int fy_cols,
                    const float *freqs_fx, int fx_rows, int fx_cols, int64_t *token_counter,
                    pkv_stream_t stream);
int pkv_attend_attention(const pkv_cache_t *cache, const uint16_t *q, int64_t q_tok_stride,
                         int64_t q_head_stride, int num_chunks, float softmax_scale,
                         uint16_t *out, int64_t o_tok_stride, int64_t o_head_stride,
                         pkv_stream_t stream);

/*
 * pkv_attend for callers that cannot allocate device memory: a host runtime
 * that owns the device's memory pool and lends this library only the cache
 * and each call's inputs and outputs, or a serving loop where a cudaMalloc
 * could synchronise the device.  Same arguments and results as pkv_attend;
 * cache->scratch is not used (may be NULL).  The planner's scratch is a fixed
 * PKV_NOALLOC_SCRATCH_BYTES device array inside libpkv.so, held by every GPU
 * that loads the library until the process exits.  A call whose plan needs
 * more -- 32 bytes per segment plus 8, with num_chunks * num_heads *
 * (max_sink + max_middle + max_recent + max_merge_blocks) segments, i.e. more
 * than 16383 segments -- returns PKV_ENOALLOC_LIMIT before launching
 * anything.  The first call on each device looks up the array's device
 * address; make it before any stream capture.  All calls share the array:
 * calls whose launches overlap on the GPU race.  No counterpart in the
 * reference.
 */
#define PKV_NOALLOC_SCRATCH_BYTES (512 * 1024)
int pkv_attend_noalloc(const pkv_cache_t *cache, const uint8_t *states_layer, int layer_idx,
                       const uint16_t *q, int64_t q_tok_stride, int64_t q_head_stride,
                       int num_chunks, int64_t first_t, int sink_mode_code, int sink_clamp_min,
                       int sink_clamp_max, int decoupled_sink_lag, const float *freqs_ft,
                       int ft_rows, int ft_cols, const float *freqs_fy, int fy_rows, int fy_cols,
                       const float *freqs_fx, int fx_rows, int fx_cols, float softmax_scale,
                       uint16_t *out, int64_t o_tok_stride, int64_t o_head_stride,
                       int64_t *token_counter, pkv_stream_t stream);

/*
 * 3D RoPE of a query block (model side, before pkv_attend): token s of the
 * frames x grid_h x grid_w grid, head h, pair p of head_dim is multiplied in
 * complex float64 by freqs_t[start_frame + f] (p < t_cols), freqs_y[row]
 * (next y_cols pairs) or freqs_x[col] (the rest), then rounded to float32 and
 * to bf16 (torch's float64 -> bf16 cast); tokens past the grid are copied.  Tables: float64 [rows, cols, 2] (re, im).
 * x / out: bf16 at base + tok * tok_stride + h * head_stride (16-byte aligned,
 * strides multiples of 8 elements).
 * Replaces: causal_rope_apply (wan/modules/causal_model.py:30-63) for one sample.
 */
int pkv_rope_q(const uint16_t *x, int64_t x_tok_stride, int64_t x_head_stride, uint16_t *out,
               int64_t o_tok_stride, int64_t o_head_stride, int64_t tokens, int heads,
               int head_dim, int64_t start_frame, int frames, int grid_h, int grid_w,
               const double *freqs_t, int t_rows, int t_cols, const double *freqs_y, int y_rows,
               int y_cols, const double *freqs_x, int x_rows, int x_cols, pkv_stream_t stream);

/*
 * Head-parallel exchange layout copy (around the NCCL all-to-all of a layer
 * step split over ranks by heads): for each source i < count (<= 4), token
 * t < tokens and group g < groups, copy the group_elems bf16 elements at
 * srcs[i] + t*src_tok_strides[i] + g*src_group_strides[i] to
 * dst + t*dst_tok_stride + g*dst_group_stride + i*dst_src_stride (all in
 * elements).  Packs Q, K and V of a token shard into a by-destination send
 * buffer in one pass, and scatters a received attention output back into
 * the [tokens, heads, D] layout.  16-byte copies when every address and
 * stride allows.  No counterpart in the reference (it runs on one GPU).
 */
int pkv_chunk_copy(const uint16_t *const *srcs, const int64_t *src_tok_strides,
                   const int64_t *src_group_strides, int count, uint16_t *dst,
                   int64_t dst_tok_stride, int64_t dst_group_stride, int64_t dst_src_stride,
                   int64_t tokens, int groups, int group_elems, pkv_stream_t stream);

/*
 * pkv_chunk_copy with one destination base per group (groups <= 8): chunk
 * (source i, token t, group g) goes to dsts[g] + t*dst_tok_stride +
 * i*dst_src_stride.  dsts may be other GPUs' buffers mapped into this process
 * (symmetric memory): the head-parallel exchange writes each rank's share
 * straight into that rank's receive buffer over NVLink, then the ranks
 * barrier.  No counterpart in the reference.
 */
int pkv_chunk_copy_peers(const uint16_t *const *srcs, const int64_t *src_tok_strides,
                         const int64_t *src_group_strides, int count, uint16_t *const *dsts,
                         int64_t dst_tok_stride, int64_t dst_src_stride, int64_t tokens,
                         int groups, int group_elems, pkv_stream_t stream);

/* ---- AdaptiveKVCache / CppStrategyManager ops (not on the MegaCache path) ----
 * Same bytes as the reference's kernels; launched on `stream` (the
 * reference's use the legacy default stream).  One CTA per segment / frame.
 */

/* dst + offsets[s] * row_bytes <- lengths[s] rows of row_bytes bytes from the
 * device address src_ptrs[s], for each s < num_segments.
 * Replaces: scatter_copy (pyramidkv/csrc/scatter_copy.cu:13-47, :230-248). */
int pkv_scatter_copy(const int64_t *src_ptrs, const int64_t *lengths, const int64_t *offsets,
                     void *dst, int64_t row_bytes, int num_segments, pkv_stream_t stream);

/* pos[i * 3] = vals[r] for starts[r] <= i < ends[r], r < num_ranges.
 * Replaces: apply_pos_override (scatter_copy.cu:53-71, :250-267). */
int pkv_pos_override(int64_t *pos, const int64_t *starts, const int64_t *ends,
                     const int64_t *vals, int num_ranges, pkv_stream_t stream);

/* Copy segment s (lengths[s] rows, device addresses src_ptrs_k/v/pos[s]) to
 * rows offsets[s].. of dst_k / dst_v / dst_rope_pos, remapping each row's
 * time: flags bit 2 -> dynamic_rope_t[s]; else bit 0 -> history mapping
 * (mapping_mode 1 relative_clamp, 2 relative_softcap, 0 none) against
 * current_t; dst_frame_ids gets the stored time when flags bit 1 is set, else
 * the mapped one.  Replaces: refresh_readout_layout (scatter_copy.cu:77-168,
 * scatter_copy_bind.cpp:483-627). */
int pkv_refresh_readout_layout(const int64_t *src_ptrs_k, const int64_t *src_ptrs_v,
                               const int64_t *src_ptrs_pos, const int64_t *offsets,
                               const int64_t *lengths, const int64_t *flags,
                               const int64_t *dynamic_rope_t, void *dst_k, void *dst_v,
                               int64_t *dst_rope_pos, int64_t *dst_frame_ids, int64_t row_bytes,
                               int64_t current_t, int mapping_mode,
                               int64_t history_relative_t_max, float history_time_soft_factor,
                               int num_segments, pkv_stream_t stream);

/* Frame f with frame_desc[f] = (src_frame, slot), both >= 0: copy frame
 * src_frame of k_seq / v_seq / pos_seq (frame_seqlen rows) into store slot
 * `slot`.  Replaces: anchor_store_write_frames (scatter_copy.cu:170-225,
 * scatter_copy_bind.cpp:630-684). */
int pkv_anchor_store_write_frames(const void *k_seq, const void *v_seq, const int64_t *pos_seq,
                                  const int64_t *frame_desc, void *store_k, void *store_v,
                                  int64_t *store_pos, int64_t frame_seqlen, int64_t row_bytes,
                                  int num_frames, pkv_stream_t stream);

/*
 * Self-test of the kernels' bounded waits: one GPU thread waits, with the
 * attention kernel's wait helper, on a barrier that nothing completes, for
 * limit_ns (<= 4 s) nanoseconds; the wait then gives up, ORs PKV_ST_TIMEOUT
 * into *status and writes 0 to *result (1 would mean the wait completed).
 * No counterpart in the reference; it exercises the timeout path on the GPU
 * without a fault or a hang.
 */
int pkv_wait_selftest(int32_t *status, int64_t limit_ns, int32_t *result, pkv_stream_t stream);

/*
 * Evaluation order of the RoPE pair rotation in the pack kernel: 0 =
 * fma(kr, fr, -(ki*fi)) / fma(kr, fi, ki*fr) (default), 1 = fma on the second
 * product, 2 = no contraction.  Returns the previous order.  No counterpart in
 * the reference: it lets parity tests reproduce whichever order a given build
 * of the reference's pack kernel (pyramidkv/csrc/pyramidkv_pack.cu:157-160)
 * was compiled to.
 */
int pkv_set_rope_rounding(int mode);

#ifdef __cplusplus
}
#endif

#endif /* PKV_H_ */
