// torch glue: registers the `adahead` library the reference's Python calls
// (torch.classes.adahead.PyramidKVCacheManager and the torch.ops.adahead.*
// schemas of pyramidkv/csrc/scatter_copy_bind.cpp:763-982) on top of the C ABI
// in libpkv.so.  Every op here only validates tensors, builds a pkv_cache_t
// view of the manager's storage and calls one extern "C" entry point on the
// current CUDA stream; there is no compute in this file.
//
// Schemas, argument order and error messages follow the reference so callers
// (pyramidkv/_mega_cache.py, _mega_state_ops.py, _mega_attention.py, _ops.py
// and their tests) work unchanged.  Ops with names starting `pkv_` are
// additions: the fused one-layer update / attend of this library, the device
// status word and the standalone ragged attention.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGraphsC10Utils.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/custom_class.h>
#include <torch/library.h>

#include <cstring>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/pkv.h"

namespace pkv_torch {

using at::Tensor;

inline void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == PKV_OK, what, ": ", pkv_error_string(rc), " (code ", rc, ")");
}

inline void* stream_of(const Tensor& t) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

template <typename T>
inline T* ptr_or_null(const Tensor& t) {
  return (t.defined() && t.numel() > 0) ? reinterpret_cast<T*>(t.data_ptr()) : nullptr;
}

// ---------------------------------------------------------------------------
// PyramidKVCacheManager: owns every pool of the cache in one device arena.
// Shapes and dtypes of the accessors are those of
// pyramidkv/csrc/pyramidkv_manager.cc:80-137; accessors return views.
// ---------------------------------------------------------------------------
class PyramidKVCacheManager : public torch::CustomClassHolder {
 public:
  PyramidKVCacheManager(int64_t num_layers, int64_t num_heads, int64_t head_dim,
                        int64_t frame_seqlen, int64_t max_sink, int64_t max_middle,
                        int64_t max_recent, const std::string& device_str,
                        const std::string& kv_dtype_str, int64_t max_attend_chunks)
      : L_(num_layers), H_(num_heads), D_(head_dim), F_(frame_seqlen), ms_(max_sink),
        mm_(max_middle), mr_(max_recent), mac_(max_attend_chunks) {
    TORCH_CHECK(num_layers > 0 && num_heads > 0 && head_dim > 0,
                "PyramidKVCacheManager: num_layers/num_heads/head_dim must be > 0");
    TORCH_CHECK(frame_seqlen > 0, "PyramidKVCacheManager: frame_seqlen must be > 0");
    TORCH_CHECK(max_sink >= 0 && max_middle >= 0 && max_recent >= 0,
                "PyramidKVCacheManager: max_*_frames must be >= 0");
    TORCH_CHECK(max_attend_chunks > 0,
                "PyramidKVCacheManager: max_attend_chunks must be > 0 "
                "(usually = num_frame_per_block with safety margin)");
    const c10::Device device(device_str);
    at::ScalarType kv;
    if (kv_dtype_str == "bfloat16" || kv_dtype_str == "bf16") kv = at::kBFloat16;
    else if (kv_dtype_str == "float16" || kv_dtype_str == "half" || kv_dtype_str == "fp16")
      kv = at::kHalf;
    else if (kv_dtype_str == "float32" || kv_dtype_str == "float" || kv_dtype_str == "fp32")
      kv = at::kFloat;
    else TORCH_CHECK(false, "PyramidKVCacheManager: unsupported kv dtype '", kv_dtype_str, "'");

    const int64_t MMB = PKV_MAX_MERGE_BLOCKS, MMA = PKV_MAX_MERGE_ACTIVE,
                  MTPA = PKV_MAX_MERGE_TOKENS;
    const int64_t MT = ms_ + mm_ + mr_;
    const int64_t P = max_pack_tokens();
    // arena plan: (name, dtype, shape); every region 256-byte aligned
    struct Region { Tensor* t; at::ScalarType dt; std::vector<int64_t> shape; };
    std::vector<Region> plan = {
        {&sink_k_, kv, {L_, H_, ms_, F_, D_}},       {&sink_v_, kv, {L_, H_, ms_, F_, D_}},
        {&middle_k_, kv, {L_, H_, mm_, F_, D_}},     {&middle_v_, kv, {L_, H_, mm_, F_, D_}},
        {&recent_k_, kv, {L_, H_, mr_, F_, D_}},     {&recent_v_, kv, {L_, H_, mr_, F_, D_}},
        {&sink_pos_, at::kLong, {L_, H_, ms_, F_, 3}},
        {&middle_pos_, at::kLong, {L_, H_, mm_, F_, 3}},
        {&recent_pos_, at::kLong, {L_, H_, mr_, F_, 3}},
        {&head_t_, at::kLong, {L_, H_, MT}},        {&write_idx_, at::kLong, {L_, H_, 3}},
        {&valid_count_, at::kLong, {L_, H_, 3}},    {&strategy_, at::kChar, {L_, H_, 8}},
        {&k_flat_, kv, {P, 1, D_}},                 {&v_flat_, kv, {P, 1, D_}},
        {&cu_seqlens_k_, at::kInt, {mac_ * H_ + 1}}, {&pos_flat_, at::kLong, {P, 3}},
        {&merge_k_, kv, {L_, H_, MMB, MTPA, D_}},   {&merge_v_, kv, {L_, H_, MMB, MTPA, D_}},
        {&merge_pos_, at::kLong, {L_, H_, MMB, MTPA, 3}},
        {&merge_tc_, at::kInt, {L_, H_, MMB}},
        {&acc_k_, at::kFloat, {L_, H_, MMA, MTPA, D_}},
        {&acc_v_, at::kFloat, {L_, H_, MMA, MTPA, D_}},
        {&acc_pos_, at::kLong, {L_, H_, MMA, MTPA, 3}},
        {&acc_gid_, at::kInt, {L_, H_, MMA, F_}},
        {&acc_tpg_, at::kFloat, {L_, H_, MMA, MTPA}},
        {&acc_ng_, at::kInt, {L_, H_, MMA}},
        {&status_, at::kInt, {4}},
    };
    int64_t total = 0;
    std::vector<int64_t> offs;
    for (auto& r : plan) {
      int64_t n = 1;
      for (auto s : r.shape) n *= s;
      offs.push_back(total);
      total += (n * c10::elementSize(r.dt) + 255) / 256 * 256;
    }
    arena_ = at::zeros({total}, at::TensorOptions().dtype(at::kByte).device(device));
    for (size_t i = 0; i < plan.size(); ++i) {
      int64_t n = 1;
      for (auto s : plan[i].shape) n *= s;
      *plan[i].t = arena_.narrow(0, offs[i], n * c10::elementSize(plan[i].dt))
                       .view(plan[i].dt)
                       .view(plan[i].shape);
    }
    head_t_.fill_(-1);
    pkv_cache_t probe = view();
    scratch_ = at::zeros({pkv_scratch_bytes(&probe)},
                         at::TensorOptions().dtype(at::kByte).device(device));
  }

  void reset() {
    // pyramidkv_manager.cc:162-180
    write_idx_.zero_();
    valid_count_.zero_();
    head_t_.fill_(-1);
    cu_seqlens_k_.zero_();
    sink_pos_.zero_();
    middle_pos_.zero_();
    recent_pos_.zero_();
    merge_tc_.zero_();
    acc_ng_.zero_();
    // not in the reference: the attention workspace's arrival counters live
    // in the scratch; a launch that ended on a device timeout can leave them
    // set, so a reset starts them from zero again
    if (scratch_.defined()) scratch_.zero_();
  }

  void set_strategy(int64_t l, int64_t h, int64_t kind, Tensor params) {
    // pyramidkv_manager.cc:182-214
    TORCH_CHECK(l >= 0 && l < L_, "PyramidKVCacheManager::set_strategy layer_idx out of range");
    TORCH_CHECK(h >= 0 && h < H_, "PyramidKVCacheManager::set_strategy head_idx out of range");
    TORCH_CHECK(params.dtype() == at::kChar,
                "PyramidKVCacheManager::set_strategy params must be int8");
    TORCH_CHECK(params.dim() == 1, "params must be 1D");
    TORCH_CHECK(params.size(0) <= 7, "params longer than 7 (slot[0] is kind)");
    TORCH_CHECK(kind >= -128 && kind <= 127, "kind out of int8 range");
    auto cpu = params.to(at::kCPU).contiguous();
    auto buf = at::zeros({8}, at::TensorOptions().dtype(at::kChar));
    buf.data_ptr<int8_t>()[0] = static_cast<int8_t>(kind);
    if (cpu.size(0) > 0) std::memcpy(buf.data_ptr<int8_t>() + 1, cpu.data_ptr<int8_t>(), cpu.size(0));
    strategy_.index_put_({l, h}, buf.to(strategy_.device(), /*non_blocking=*/true));
  }

  // ---- accessors ----
  Tensor sink_pool() const { return sink_k_; }
  Tensor middle_pool() const { return middle_k_; }
  Tensor recent_pool() const { return recent_k_; }
  Tensor sink_k_pool() const { return sink_k_; }
  Tensor sink_v_pool() const { return sink_v_; }
  Tensor middle_k_pool() const { return middle_k_; }
  Tensor middle_v_pool() const { return middle_v_; }
  Tensor recent_k_pool() const { return recent_k_; }
  Tensor recent_v_pool() const { return recent_v_; }
  Tensor sink_pos_pool() const { return sink_pos_; }
  Tensor middle_pos_pool() const { return middle_pos_; }
  Tensor recent_pos_pool() const { return recent_pos_; }
  Tensor head_t_table() const { return head_t_; }
  Tensor write_idx() const { return write_idx_; }
  Tensor valid_count() const { return valid_count_; }
  Tensor strategy() const { return strategy_; }
  Tensor k_flat_out() const { return k_flat_; }
  Tensor v_flat_out() const { return v_flat_; }
  Tensor cu_seqlens_k() const { return cu_seqlens_k_; }
  Tensor pos_flat_out() const { return pos_flat_; }
  Tensor merge_k_pool() const { return merge_k_; }
  Tensor merge_v_pool() const { return merge_v_; }
  Tensor merge_pos_pool() const { return merge_pos_; }
  Tensor merge_token_count() const { return merge_tc_; }
  Tensor merge_accum_sum_k() const { return acc_k_; }
  Tensor merge_accum_sum_v() const { return acc_v_; }
  Tensor merge_accum_pos() const { return acc_pos_; }
  Tensor merge_accum_group_ids() const { return acc_gid_; }
  Tensor merge_accum_tokens_per_group() const { return acc_tpg_; }
  Tensor merge_accum_num_groups() const { return acc_ng_; }
  Tensor status_word() const { return status_; }
  Tensor scratch() const { return scratch_; }
  int64_t num_layers() const { return L_; }
  int64_t num_heads() const { return H_; }
  int64_t head_dim() const { return D_; }
  int64_t frame_seqlen() const { return F_; }
  int64_t max_sink() const { return ms_; }
  int64_t max_middle() const { return mm_; }
  int64_t max_recent() const { return mr_; }
  int64_t max_total() const { return ms_ + mm_ + mr_; }
  int64_t max_attend_chunks() const { return mac_; }
  int64_t max_pack_tokens() const {
    return mac_ * H_ * (max_total() + PKV_MAX_MERGE_BLOCKS) * F_;
  }
  int64_t max_total_tokens() const { return max_pack_tokens(); }
  int64_t max_merge_blocks() const { return PKV_MAX_MERGE_BLOCKS; }
  int64_t max_merge_active() const { return PKV_MAX_MERGE_ACTIVE; }
  int64_t max_merge_tokens_per_anchor() const { return PKV_MAX_MERGE_TOKENS; }

  pkv_cache_t view() const {
    pkv_cache_t c{};
    c.num_layers = int32_t(L_); c.num_heads = int32_t(H_); c.head_dim = int32_t(D_);
    c.frame_seqlen = int32_t(F_);
    c.max_sink = int32_t(ms_); c.max_middle = int32_t(mm_); c.max_recent = int32_t(mr_);
    c.max_merge_blocks = PKV_MAX_MERGE_BLOCKS; c.max_merge_active = PKV_MAX_MERGE_ACTIVE;
    c.max_merge_tokens = PKV_MAX_MERGE_TOKENS;
    c.max_attend_chunks = int32_t(mac_);
    c.spatial_width = 1;
    c.max_pack_tokens = max_pack_tokens();
    auto u16 = [](const Tensor& t) { return reinterpret_cast<uint16_t*>(t.data_ptr()); };
    c.sink_k = u16(sink_k_); c.sink_v = u16(sink_v_);
    c.middle_k = u16(middle_k_); c.middle_v = u16(middle_v_);
    c.recent_k = u16(recent_k_); c.recent_v = u16(recent_v_);
    c.sink_pos = sink_pos_.data_ptr<int64_t>(); c.middle_pos = middle_pos_.data_ptr<int64_t>();
    c.recent_pos = recent_pos_.data_ptr<int64_t>();
    c.valid_count = valid_count_.data_ptr<int64_t>();
    c.merge_k = u16(merge_k_); c.merge_v = u16(merge_v_);
    c.merge_pos = merge_pos_.data_ptr<int64_t>();
    c.merge_token_count = merge_tc_.data_ptr<int32_t>();
    c.accum_sum_k = acc_k_.data_ptr<float>(); c.accum_sum_v = acc_v_.data_ptr<float>();
    c.accum_pos = acc_pos_.data_ptr<int64_t>(); c.accum_group_ids = acc_gid_.data_ptr<int32_t>();
    c.accum_tokens_per_group = acc_tpg_.data_ptr<float>();
    c.accum_num_groups = acc_ng_.data_ptr<int32_t>();
    c.k_flat = u16(k_flat_); c.v_flat = u16(v_flat_); c.pos_flat = pos_flat_.data_ptr<int64_t>();
    c.cu_seqlens_k = cu_seqlens_k_.data_ptr<int32_t>();
    if (scratch_.defined()) {
      c.scratch = scratch_.data_ptr();
      c.scratch_bytes = scratch_.numel();
    }
    c.status = status_.data_ptr<int32_t>();
    c.first_t_dev = time_src_.defined() ? time_src_.data_ptr<int64_t>() : nullptr;
    return c;
  }

  // Not in the reference: the fused update / attend ops read the block's
  // first latent frame from `t` (a device int64 scalar) when their kernels
  // run, instead of their first_t argument, so a captured layer step replays
  // for any block.  clear_block_time() returns to the argument.
  void set_block_time(Tensor t) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kLong && t.numel() == 1 &&
                    t.device() == device(),
                "set_block_time: expected a one-element int64 tensor on the manager's device");
    time_src_ = t;
  }
  void clear_block_time() { time_src_ = Tensor(); }

  c10::Device device() const { return arena_.device(); }
  at::ScalarType kv_dtype() const { return sink_k_.scalar_type(); }

 private:
  int64_t L_, H_, D_, F_, ms_, mm_, mr_, mac_;
  Tensor arena_, scratch_;
  Tensor time_src_;  // device int64 block time read by the kernels (undefined: the argument)
  Tensor sink_k_, sink_v_, middle_k_, middle_v_, recent_k_, recent_v_;
  Tensor sink_pos_, middle_pos_, recent_pos_;
  Tensor head_t_, write_idx_, valid_count_, strategy_;
  Tensor k_flat_, v_flat_, cu_seqlens_k_, pos_flat_;
  Tensor merge_k_, merge_v_, merge_pos_, merge_tc_;
  Tensor acc_k_, acc_v_, acc_pos_, acc_gid_, acc_tpg_, acc_ng_;
  Tensor status_;
};

using Mgr = c10::intrusive_ptr<PyramidKVCacheManager>;

inline void require_cuda_bf16(const Mgr& mgr, const char* op) {
  TORCH_CHECK(mgr->device().is_cuda(), op, ": manager storage must be on CUDA");
  TORCH_CHECK(mgr->kv_dtype() == at::kBFloat16, op, " currently only implements bf16 pools");
}

// ---------------------------------------------------------------------------
// Reference-schema ops
// ---------------------------------------------------------------------------
int64_t mega_state_perhead_size() { return pkv_state_perhead_size(); }

void mega_state_update(Tensor states, Tensor new_t_vals, Tensor dk, Tensor ds, Tensor dsf,
                       Tensor dsh, Tensor dma, Tensor dml, Tensor dmf, Tensor dmn,
                       int64_t num_heads, int64_t frames, int64_t pass_kind) {
  // scatter_copy_bind.cpp:345-380 + anchor_store_update.cu:338-357
  TORCH_CHECK(states.is_cuda(), "mega_state_update: states must be CUDA");
  TORCH_CHECK(states.dtype() == at::kByte,
              "mega_state_update: states must be uint8 (raw byte buffer)");
  TORCH_CHECK(states.is_contiguous(), "mega_state_update: states must be contiguous");
  const int64_t need = num_heads * pkv_state_perhead_size();
  TORCH_CHECK(states.numel() >= need, "mega_state_update: states buffer too small (",
              states.numel(), " < ", need, ")");
  TORCH_CHECK(new_t_vals.is_cuda() && new_t_vals.dtype() == at::kLong,
              "new_t_vals must be CUDA int64");
  for (const Tensor* t : {&dk, &ds, &dsf, &dsh, &dma, &dml, &dmf, &dmn})
    TORCH_CHECK(t->dtype() == at::kInt && t->is_cuda() && t->is_contiguous() &&
                    t->numel() >= num_heads * frames,
                "all descriptor tensors must be int32");
  if (num_heads == 0 || frames == 0) return;
  const c10::cuda::CUDAGuard g(states.device());
  auto nt = new_t_vals.contiguous();
  check_rc(pkv_mega_state_update(states.data_ptr<uint8_t>(), nt.data_ptr<int64_t>(),
                                 dk.data_ptr<int32_t>(), ds.data_ptr<int32_t>(),
                                 dsf.data_ptr<int32_t>(), dsh.data_ptr<int32_t>(),
                                 dma.data_ptr<int32_t>(), dml.data_ptr<int32_t>(),
                                 dmf.data_ptr<int32_t>(), dmn.data_ptr<int32_t>(),
                                 int(num_heads), int(frames), int(pass_kind), nullptr,
                                 stream_of(states)),
           "mega_state_update");
}

void pyramidkv_update(Mgr mgr, Tensor new_k, Tensor new_v, Tensor new_pos, Tensor dst_kind,
                      Tensor dst_slot, Tensor src_frame, Tensor src_head) {
  TORCH_CHECK(mgr.get() != nullptr, "pyramidkv_update: manager is null");
  TORCH_CHECK(new_k.is_cuda() && new_v.is_cuda(), "pyramidkv_update: new_k/new_v must be on CUDA");
  TORCH_CHECK(new_k.scalar_type() == at::kBFloat16,
              "pyramidkv_update currently only implements bf16");
  TORCH_CHECK(dst_kind.dtype() == at::kInt && dst_slot.dtype() == at::kInt &&
                  src_frame.dtype() == at::kInt && src_head.dtype() == at::kInt,
              "all descriptor tensors must be int32");
  require_cuda_bf16(mgr, "pyramidkv_update");
  const int64_t n = dst_kind.numel();
  if (n == 0) return;
  const c10::cuda::CUDAGuard g(new_k.device());
  auto nk = new_k.contiguous(), nv = new_v.contiguous();
  Tensor np;
  if (new_pos.defined() && new_pos.numel() > 0) {
    TORCH_CHECK(new_pos.dtype() == at::kLong, "pyramidkv_update: new_pos must be int64");
    np = new_pos.contiguous();
  }
  auto c = mgr->view();
  auto k = dst_kind.contiguous(), s = dst_slot.contiguous(), f = src_frame.contiguous(),
       h = src_head.contiguous();
  check_rc(pkv_update_frames(&c, reinterpret_cast<const uint16_t*>(nk.data_ptr()),
                             reinterpret_cast<const uint16_t*>(nv.data_ptr()),
                             ptr_or_null<const int64_t>(np), k.data_ptr<int32_t>(),
                             s.data_ptr<int32_t>(), f.data_ptr<int32_t>(), h.data_ptr<int32_t>(),
                             int(n), stream_of(new_k)),
           "pyramidkv_update");
}

void mega_merge_accum(Tensor states, Tensor new_k, Tensor new_v, Tensor new_pos, Tensor dk,
                      Tensor dslot, Tensor dfin, Tensor dnew, Tensor acc_k, Tensor acc_v,
                      Tensor acc_pos, Tensor acc_gid, Tensor acc_tpg, Tensor acc_ng,
                      Tensor mk, Tensor mv, Tensor mpos, Tensor mtc) {
  // mega_merge_accum.cu:288-305
  TORCH_CHECK(new_k.is_cuda() && new_v.is_cuda() && new_pos.is_cuda(),
              "mega_merge_accum: new_k/v/pos must be CUDA");
  TORCH_CHECK(new_k.dtype() == at::kBFloat16, "mega_merge_accum: new_k must be bf16");
  TORCH_CHECK(new_v.dtype() == at::kBFloat16, "mega_merge_accum: new_v must be bf16");
  TORCH_CHECK(new_pos.dtype() == at::kLong, "mega_merge_accum: new_pos must be int64");
  TORCH_CHECK(acc_k.dtype() == at::kFloat && acc_v.dtype() == at::kFloat,
              "mega_merge_accum: accumulators must be fp32");
  TORCH_CHECK(mk.dtype() == at::kBFloat16 && mv.dtype() == at::kBFloat16,
              "mega_merge_accum: merge_k/v_pool must be bf16");
  for (const Tensor* t : {&acc_k, &acc_v, &acc_pos, &acc_gid, &acc_tpg, &acc_ng, &mk, &mv,
                          &mpos, &mtc})
    TORCH_CHECK(t->is_contiguous(), "mega_merge_accum: pool slices must be contiguous");
  const int F = int(new_k.size(0)), H = int(new_k.size(1)), FSEQ = int(new_k.size(2)),
            D = int(new_k.size(3));
  const int MMA = int(acc_k.size(1)), MMB = int(mk.size(1)), MTPA = int(acc_k.size(2));
  if (H == 0 || F == 0) return;
  const c10::cuda::CUDAGuard g(new_k.device());
  auto nk = new_k.contiguous(), nv = new_v.contiguous(), np = new_pos.contiguous();
  auto k = dk.contiguous(), s = dslot.contiguous(), fi = dfin.contiguous(), nw = dnew.contiguous();
  check_rc(pkv_merge_accum(states.data_ptr<uint8_t>(),
                           reinterpret_cast<const uint16_t*>(nk.data_ptr()),
                           reinterpret_cast<const uint16_t*>(nv.data_ptr()),
                           np.data_ptr<int64_t>(), k.data_ptr<int32_t>(), s.data_ptr<int32_t>(),
                           fi.data_ptr<int32_t>(), nw.data_ptr<int32_t>(), acc_k.data_ptr<float>(),
                           acc_v.data_ptr<float>(), acc_pos.data_ptr<int64_t>(),
                           acc_gid.data_ptr<int32_t>(), acc_tpg.data_ptr<float>(),
                           acc_ng.data_ptr<int32_t>(), reinterpret_cast<uint16_t*>(mk.data_ptr()),
                           reinterpret_cast<uint16_t*>(mv.data_ptr()), mpos.data_ptr<int64_t>(),
                           mtc.data_ptr<int32_t>(), H, F, FSEQ, D, MMA, MMB, MTPA, nullptr,
                           stream_of(new_k)),
           "mega_merge_accum");
}

using Plan7 = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor>;

// Reads the sticky status word (one device->host copy) and clears it.
int32_t take_status(const Mgr& mgr) {
  auto st = mgr->status_word();
  const int32_t v = st[0].item<int32_t>();
  if (v != 0) st.zero_();
  return v;
}

bool capturing(const Mgr&) {
  return c10::cuda::currentStreamCaptureStatusMayInitCtx() != c10::cuda::CaptureStatus::None;
}

// Largest token total a plan over `chunks` chunks can produce.
int64_t plan_bound(const Mgr& mgr, int64_t chunks) {
  const int64_t seg = mgr->max_total() + PKV_MAX_MERGE_BLOCKS;
  const int64_t len = std::max<int64_t>(mgr->frame_seqlen(), PKV_MAX_MERGE_TOKENS);
  return chunks * mgr->num_heads() * seg * len;
}

Plan7 plan_impl(const Mgr& mgr, const Tensor& states_bytes, int64_t layer,
                const std::vector<int64_t>& ts, int64_t sink_mode, int64_t cmin, int64_t cmax,
                int64_t lag, bool multi, const char* name) {
  TORCH_CHECK(mgr.get() != nullptr, name, ": manager is null");
  TORCH_CHECK(states_bytes.dtype() == at::kByte, name, ": states_bytes must be uint8");
  TORCH_CHECK(states_bytes.numel() >= mgr->num_heads() * pkv_state_perhead_size(), name,
              ": states_bytes too small for ", mgr->num_heads(), " heads");
  TORCH_CHECK(layer >= 0 && layer < mgr->num_layers(), name, ": layer_idx out of range");
  TORCH_CHECK(mgr->device().is_cuda(), name, ": manager storage must be on CUDA");
  const c10::cuda::CUDAGuard g(mgr->device());
  const int64_t C = int64_t(ts.size());
  const int64_t H = mgr->num_heads();
  const int64_t S = mgr->max_total() + PKV_MAX_MERGE_BLOCKS;
  auto i32 = at::TensorOptions().dtype(at::kInt).device(mgr->device());
  auto i64 = at::TensorOptions().dtype(at::kLong).device(mgr->device());
  Tensor cu = at::empty({C * H + 1}, i32), sk = at::empty({C * H * S}, i32),
         sg = at::empty({C * H * S}, i32), sl = at::empty({C * H * S}, i32),
         dst = at::empty({C * H * S}, i32), traw = at::empty({C * H * S}, i64),
         tremap = at::empty({C * H * S}, i64), total = at::empty({1}, i64);
  auto sb = states_bytes.is_cuda() ? states_bytes.contiguous()
                                   : states_bytes.to(mgr->device()).contiguous();
  auto c = mgr->view();
  check_rc(pkv_plan(&c, sb.data_ptr<uint8_t>(), int(layer), ts.data(), int(C), int(sink_mode),
                    int(cmin), int(cmax), int(lag), multi ? 1 : 0, 0, cu.data_ptr<int32_t>(),
                    sk.data_ptr<int32_t>(), sg.data_ptr<int32_t>(), sl.data_ptr<int32_t>(),
                    dst.data_ptr<int32_t>(), traw.data_ptr<int64_t>(),
                    tremap.data_ptr<int64_t>(), total.data_ptr<int64_t>(), nullptr,
                    stream_of(cu)),
           name);
  // mega_plan.cc:622-629.  The device plan flags overflow in the status
  // word; the synchronous check below runs only when the static bound says
  // an overflow is possible at all (never for the shipped configurations).
  if (multi && plan_bound(mgr, C) > mgr->max_pack_tokens() && !capturing(mgr)) {
    const int64_t tot = total.item<int64_t>();
    if (tot > mgr->max_pack_tokens()) take_status(mgr);
    TORCH_CHECK(tot <= mgr->max_pack_tokens(), "mega_plan_multi: packed tokens (", tot,
                ") exceed pack-workspace capacity (", mgr->max_pack_tokens(),
                "). Either reduce chunks (", C,
                ") or rebuild the manager with a larger max_attend_chunks (currently ",
                mgr->max_attend_chunks(), ").");
  }
  return {cu, sk, sg, sl, dst, traw, tremap};
}

Plan7 mega_plan(Mgr mgr, Tensor states_bytes, int64_t layer, int64_t current_t, int64_t,
                int64_t sink_mode, int64_t cmin, int64_t cmax, int64_t lag, int64_t, int64_t,
                double) {
  return plan_impl(mgr, states_bytes, layer, {current_t}, sink_mode, cmin, cmax, lag, false,
                   "mega_plan");
}

Plan7 mega_plan_multi(Mgr mgr, Tensor states_bytes, int64_t layer, Tensor current_t_list,
                      int64_t, int64_t sink_mode, int64_t cmin, int64_t cmax, int64_t lag,
                      int64_t, int64_t, double) {
  TORCH_CHECK(current_t_list.dtype() == at::kLong, "mega_plan_multi: current_t_list must be int64");
  TORCH_CHECK(current_t_list.dim() == 1, "mega_plan_multi: current_t_list must be 1D");
  TORCH_CHECK(current_t_list.numel() > 0, "mega_plan_multi: empty current_t_list");
  TORCH_CHECK(current_t_list.numel() <= PKV_MAX_CHUNKS, "mega_plan_multi: more than ",
              PKV_MAX_CHUNKS, " chunks");
  auto cpu = current_t_list.to(at::kCPU).contiguous();
  std::vector<int64_t> ts(cpu.data_ptr<int64_t>(), cpu.data_ptr<int64_t>() + cpu.numel());
  return plan_impl(mgr, states_bytes, layer, ts, sink_mode, cmin, cmax, lag, true,
                   "mega_plan_multi");
}

void pyramidkv_pack(Mgr mgr, Tensor sk, Tensor sg, Tensor sl, Tensor dst, Tensor tremap,
                    Tensor ft, Tensor fy, Tensor fx) {
  TORCH_CHECK(mgr.get() != nullptr, "pyramidkv_pack: manager is null");
  TORCH_CHECK(mgr->device().is_cuda(), "pools must be on CUDA");
  TORCH_CHECK(mgr->kv_dtype() == at::kBFloat16,
              "pyramidkv_pack currently only implements bf16 pools");
  TORCH_CHECK(sk.dtype() == at::kInt && sg.dtype() == at::kInt && sl.dtype() == at::kInt &&
                  dst.dtype() == at::kInt,
              "all PlanInfo descriptor tensors must be int32");
  const int64_t n = sk.numel();
  if (n == 0) return;
  const c10::cuda::CUDAGuard g(mgr->device());
  auto a = sk.contiguous(), b = sg.contiguous(), cl = sl.contiguous(), d = dst.contiguous();
  Tensor tm = (tremap.defined() && tremap.numel() > 0) ? tremap.contiguous() : Tensor();
  auto table = [](const Tensor& t, const char* nm, int& rows, int& cols) -> const float* {
    if (!t.defined() || t.numel() == 0) { rows = cols = 0; return nullptr; }
    TORCH_CHECK(t.dim() == 2 && t.dtype() == at::kFloat, nm, " must be 2D fp32");
    TORCH_CHECK(t.is_contiguous() && t.is_cuda(), nm, " must be a contiguous CUDA tensor");
    rows = int(t.size(0));
    cols = int(t.size(1) / 2);
    return t.data_ptr<float>();
  };
  int tr, tc, yr, yc, xr, xc;
  const float* pt = table(ft, "freqs_ft_flat", tr, tc);
  const float* py = table(fy, "freqs_fy_flat", yr, yc);
  const float* px = table(fx, "freqs_fx_flat", xr, xc);
  auto c = mgr->view();
  check_rc(pkv_pack(&c, a.data_ptr<int32_t>(), b.data_ptr<int32_t>(), cl.data_ptr<int32_t>(),
                    d.data_ptr<int32_t>(), int(n), ptr_or_null<const int64_t>(tm), pt, tr, tc,
                    py, yr, yc, px, xr, xc, stream_of(a)),
           "pyramidkv_pack");
}

// ---------------------------------------------------------------------------
// Additions of this library
// ---------------------------------------------------------------------------
void op_cache_update(Mgr mgr, Tensor states_all, int64_t layer, Tensor new_k, Tensor new_v,
                      int64_t first_t, int64_t pass_kind, Tensor sink_caps, Tensor committed_vc,
                      Tensor committed_k, Tensor committed_v, Tensor committed_pos,
                      int64_t spatial_width, bool has_merge_head) {
  require_cuda_bf16(mgr, "MegaCache.update");
  TORCH_CHECK(new_k.dim() == 4 && new_k.sizes() == new_v.sizes(), "K/V shapes must match");
  TORCH_CHECK(new_k.size(0) == 1, "MegaCache.update: B>1 not yet supported");
  TORCH_CHECK(new_k.size(2) == mgr->num_heads() && new_k.size(3) == mgr->head_dim(),
              "MegaCache.update: head count / head dim mismatch");
  TORCH_CHECK(new_k.size(1) % mgr->frame_seqlen() == 0, "L_in (", new_k.size(1),
              ") not multiple of FSEQ (", mgr->frame_seqlen(), ")");
  TORCH_CHECK(new_k.scalar_type() == at::kBFloat16 && new_v.scalar_type() == at::kBFloat16,
              "MegaCache.update: K/V must be bf16");
  TORCH_CHECK(states_all.dtype() == at::kByte && states_all.is_contiguous(),
              "MegaCache.update: states_bytes must be contiguous uint8");
  TORCH_CHECK(committed_vc.is_contiguous() && committed_k.is_contiguous() &&
                  committed_v.is_contiguous() && committed_pos.is_contiguous() &&
                  sink_caps.is_contiguous(),
              "MegaCache.update: committed snapshot must be contiguous");
  TORCH_CHECK(sink_caps.dtype() == at::kLong && committed_vc.dtype() == at::kLong,
              "MegaCache.update: sink caps / committed valid_count must be int64");
  const c10::cuda::CUDAGuard g(new_k.device());
  auto nk = new_k.stride(3) == 1 ? new_k : new_k.contiguous();
  auto nv = new_v.stride(3) == 1 && new_v.strides() == nk.strides() ? new_v
                                                                    : new_v.contiguous();
  if (nv.strides() != nk.strides()) nk = nk.contiguous();
  const int frames = int(new_k.size(1) / mgr->frame_seqlen());
  auto c = mgr->view();
  c.committed_vc = committed_vc.data_ptr<int64_t>();
  c.committed_recent_k = reinterpret_cast<uint16_t*>(committed_k.data_ptr());
  c.committed_recent_v = reinterpret_cast<uint16_t*>(committed_v.data_ptr());
  c.committed_recent_pos = committed_pos.data_ptr<int64_t>();
  c.sink_caps = sink_caps.data_ptr<int64_t>();
  c.spatial_width = int32_t(spatial_width);
  check_rc(pkv_cache_update(&c, states_all.data_ptr<uint8_t>(), int(layer),
                            reinterpret_cast<const uint16_t*>(nk.data_ptr()),
                            reinterpret_cast<const uint16_t*>(nv.data_ptr()), nk.stride(1),
                            nk.stride(2), frames, first_t, int(pass_kind), has_merge_head ? 1 : 0,
                            stream_of(nk)),
           "MegaCache.update");
}

int64_t attend_chunks(const Mgr& mgr, int64_t L_q) {
  TORCH_CHECK(L_q % mgr->frame_seqlen() == 0, "L_q (", L_q, ") must be a multiple of FSEQ (",
              mgr->frame_seqlen(), ")");
  const int64_t chunks = L_q / mgr->frame_seqlen();
  TORCH_CHECK(chunks <= mgr->max_attend_chunks(), "mega_plan_multi: packed tokens exceed "
              "pack-workspace capacity (", mgr->max_pack_tokens(), "). Either reduce chunks (",
              chunks, ") or rebuild the manager with a larger max_attend_chunks (currently ",
              mgr->max_attend_chunks(), ").");
  return chunks;
}

// Plan + RoPE-fused pack of one layer (first half of MegaCache.attend).
void op_attend_pack(Mgr mgr, Tensor states_layer, int64_t layer, int64_t L_q, int64_t first_t,
                    int64_t sink_mode, int64_t cmin, int64_t cmax, int64_t lag, Tensor ft,
                    Tensor fy, Tensor fx, Tensor token_counter) {
  require_cuda_bf16(mgr, "MegaCache.attend");
  const int64_t chunks = attend_chunks(mgr, L_q);
  const c10::cuda::CUDAGuard g(mgr->device());
  auto table = [](const Tensor& t, int& rows, int& cols) -> const float* {
    if (!t.defined() || t.numel() == 0) { rows = cols = 0; return nullptr; }
    TORCH_CHECK(t.dim() == 2 && t.dtype() == at::kFloat && t.is_contiguous() && t.is_cuda(),
                "freq tables must be contiguous 2D fp32 CUDA tensors");
    rows = int(t.size(0));
    cols = int(t.size(1) / 2);
    return t.data_ptr<float>();
  };
  int tr, tc, yr, yc, xr, xc;
  const float* pt = table(ft, tr, tc);
  const float* py = table(fy, yr, yc);
  const float* px = table(fx, xr, xc);
  auto c = mgr->view();
  auto sb = states_layer.contiguous();
  check_rc(pkv_attend_pack(&c, sb.data_ptr<uint8_t>(), int(layer), int(chunks), first_t,
                           int(sink_mode), int(cmin), int(cmax), int(lag), pt, tr, tc, py, yr,
                           yc, px, xr, xc, ptr_or_null<int64_t>(token_counter),
                           stream_of(sb)),
           "MegaCache.attend");
  if (plan_bound(mgr, chunks) > mgr->max_pack_tokens() && !capturing(mgr)) {
    const int32_t st = take_status(mgr);
    TORCH_CHECK((st & PKV_ST_PACK_OVERFLOW) == 0,
                "mega_plan_multi: packed tokens exceed pack-workspace capacity (",
                mgr->max_pack_tokens(), "). Either reduce chunks (", chunks,
                ") or rebuild the manager with a larger max_attend_chunks (currently ",
                mgr->max_attend_chunks(), ").");
  }
}

// Ragged attention over the last pack (second half of MegaCache.attend);
// q and the result are [1, L_q, H, D].
Tensor op_attend_attention(Mgr mgr, Tensor q, double scale) {
  require_cuda_bf16(mgr, "MegaCache.attend");
  TORCH_CHECK(q.dim() == 4 && q.size(0) == 1, "MegaCache.attend: B>1 not yet supported");
  TORCH_CHECK(q.size(2) == mgr->num_heads() && q.size(3) == mgr->head_dim(),
              "MegaCache.attend: head count / head dim mismatch");
  const int64_t chunks = attend_chunks(mgr, q.size(1));
  const c10::cuda::CUDAGuard g(q.device());
  auto qq = q.scalar_type() == at::kBFloat16 ? q : q.to(at::kBFloat16);
  if (qq.stride(3) != 1) qq = qq.contiguous();
  auto out = at::empty({1, q.size(1), q.size(2), q.size(3)}, qq.options());
  auto c = mgr->view();
  check_rc(pkv_attend_attention(&c, reinterpret_cast<const uint16_t*>(qq.data_ptr()),
                                qq.stride(1), qq.stride(2), int(chunks), float(scale),
                                reinterpret_cast<uint16_t*>(out.data_ptr()), out.stride(1),
                                out.stride(2), stream_of(qq)),
           "MegaCache.attend");
  return out;
}

Tensor op_attend(Mgr mgr, Tensor states_layer, int64_t layer, Tensor q, int64_t first_t,
                 int64_t sink_mode, int64_t cmin, int64_t cmax, int64_t lag, Tensor ft,
                 Tensor fy, Tensor fx, double scale, Tensor token_counter) {
  TORCH_CHECK(q.dim() == 4 && q.size(0) == 1, "MegaCache.attend: B>1 not yet supported");
  op_attend_pack(mgr, states_layer, layer, q.size(1), first_t, sink_mode, cmin, cmax, lag, ft,
                 fy, fx, token_counter);
  return op_attend_attention(mgr, q, scale);
}

Tensor op_attention(Tensor q, Tensor k, Tensor v, Tensor cu, int64_t num_chunks,
                     int64_t rows_per_chunk, double scale) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda() && cu.is_cuda(),
              "pkv_attention: tensors must be CUDA");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 &&
                  v.scalar_type() == at::kBFloat16,
              "pkv_attention: q/k/v must be bf16");
  TORCH_CHECK(cu.dtype() == at::kInt, "pkv_attention: cu_seqlens_k must be int32");
  TORCH_CHECK(q.dim() == 3, "pkv_attention: q must be [num_chunks*rows, H, D]");
  const int64_t H = q.size(1), D = q.size(2);
  TORCH_CHECK(q.size(0) == num_chunks * rows_per_chunk, "pkv_attention: q rows mismatch");
  TORCH_CHECK(cu.numel() >= num_chunks * H + 1, "pkv_attention: cu_seqlens_k too short");
  const c10::cuda::CUDAGuard g(q.device());
  auto qq = q.stride(2) == 1 ? q : q.contiguous();
  auto kk = k.reshape({-1, D}).contiguous(), vv = v.reshape({-1, D}).contiguous();
  auto cc = cu.contiguous();
  auto out = at::empty({q.size(0), H, D}, q.options());
  check_rc(pkv_attention(reinterpret_cast<const uint16_t*>(qq.data_ptr()), qq.stride(0),
                         qq.stride(1), reinterpret_cast<const uint16_t*>(kk.data_ptr()),
                         reinterpret_cast<const uint16_t*>(vv.data_ptr()), kk.size(0),
                         cc.data_ptr<int32_t>(), int(num_chunks), int(H), int(rows_per_chunk),
                         int(D), float(scale), reinterpret_cast<uint16_t*>(out.data_ptr()),
                         out.stride(0), out.stride(1), stream_of(qq)),
           "pkv_attention");
  return out;
}

// pkv_attention with a caller-owned workspace (uint8, zero-filled before its
// first use, at least pkv_attention_workspace_bytes): the SM-balanced path.
Tensor op_attention_ws(Tensor q, Tensor k, Tensor v, Tensor cu, int64_t num_chunks,
                       int64_t rows_per_chunk, double scale, Tensor workspace) {
  TORCH_CHECK(workspace.is_cuda() && workspace.dtype() == at::kByte &&
                  workspace.is_contiguous() && workspace.device() == q.device(),
              "pkv_attention_ws: workspace must be a contiguous uint8 tensor on q's device");
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda() && cu.is_cuda(),
              "pkv_attention: tensors must be CUDA");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 &&
                  v.scalar_type() == at::kBFloat16,
              "pkv_attention: q/k/v must be bf16");
  TORCH_CHECK(cu.dtype() == at::kInt, "pkv_attention: cu_seqlens_k must be int32");
  TORCH_CHECK(q.dim() == 3, "pkv_attention: q must be [num_chunks*rows, H, D]");
  const int64_t H = q.size(1), D = q.size(2);
  TORCH_CHECK(q.size(0) == num_chunks * rows_per_chunk, "pkv_attention: q rows mismatch");
  TORCH_CHECK(cu.numel() >= num_chunks * H + 1, "pkv_attention: cu_seqlens_k too short");
  const int64_t need = pkv_attention_workspace_bytes(int(num_chunks), int(H), int(rows_per_chunk));
  TORCH_CHECK(workspace.numel() >= need, "pkv_attention_ws: workspace needs ", need, " bytes");
  const c10::cuda::CUDAGuard g(q.device());
  auto qq = q.stride(2) == 1 ? q : q.contiguous();
  auto kk = k.reshape({-1, D}).contiguous(), vv = v.reshape({-1, D}).contiguous();
  auto cc = cu.contiguous();
  auto out = at::empty({q.size(0), H, D}, q.options());
  check_rc(pkv_attention_ws(reinterpret_cast<const uint16_t*>(qq.data_ptr()), qq.stride(0),
                            qq.stride(1), reinterpret_cast<const uint16_t*>(kk.data_ptr()),
                            reinterpret_cast<const uint16_t*>(vv.data_ptr()), kk.size(0),
                            cc.data_ptr<int32_t>(), int(num_chunks), int(H), int(rows_per_chunk),
                            int(D), float(scale), reinterpret_cast<uint16_t*>(out.data_ptr()),
                            out.stride(0), out.stride(1), workspace.data_ptr(), workspace.numel(),
                            stream_of(qq)),
           "pkv_attention_ws");
  return out;
}

int64_t op_attention_ws_bytes(int64_t num_chunks, int64_t num_heads, int64_t rows_per_chunk) {
  return pkv_attention_workspace_bytes(int(num_chunks), int(num_heads), int(rows_per_chunk));
}

// Head-parallel exchange layout copy (pkv_chunk_copy): strides in elements
// relative to each tensor's data pointer (views welcome).
void op_chunk_copy(std::vector<Tensor> srcs, std::vector<int64_t> src_ts,
                   std::vector<int64_t> src_gs, Tensor dst, int64_t dst_ts, int64_t dst_gs,
                   int64_t dst_is, int64_t tokens, int64_t groups, int64_t group_elems) {
  TORCH_CHECK(!srcs.empty() && srcs.size() <= 4 && src_ts.size() == srcs.size() &&
                  src_gs.size() == srcs.size(),
              "pkv_chunk_copy: 1-4 sources with one token and one group stride each");
  TORCH_CHECK(dst.is_cuda() && dst.scalar_type() == at::kBFloat16,
              "pkv_chunk_copy: dst must be a bf16 CUDA tensor");
  const uint16_t* ptrs[4] = {};
  for (size_t i = 0; i < srcs.size(); ++i) {
    TORCH_CHECK(srcs[i].is_cuda() && srcs[i].scalar_type() == at::kBFloat16 &&
                    srcs[i].device() == dst.device(),
                "pkv_chunk_copy: sources must be bf16 tensors on dst's device");
    ptrs[i] = reinterpret_cast<const uint16_t*>(srcs[i].data_ptr());
  }
  const c10::cuda::CUDAGuard g(dst.device());
  check_rc(pkv_chunk_copy(ptrs, src_ts.data(), src_gs.data(), int(srcs.size()),
                          reinterpret_cast<uint16_t*>(dst.data_ptr()), dst_ts, dst_gs, dst_is,
                          tokens, int(groups), int(group_elems), stream_of(dst)),
           "pkv_chunk_copy");
}

// pkv_chunk_copy_peers: dst_ptrs are device addresses (this process's
// mappings of each group's destination buffer, e.g. symmetric-memory peers).
void op_chunk_copy_peers(std::vector<Tensor> srcs, std::vector<int64_t> src_ts,
                         std::vector<int64_t> src_gs, std::vector<int64_t> dst_ptrs,
                         int64_t dst_ts, int64_t dst_is, int64_t tokens, int64_t group_elems) {
  TORCH_CHECK(!srcs.empty() && srcs.size() <= 4 && src_ts.size() == srcs.size() &&
                  src_gs.size() == srcs.size(),
              "pkv_chunk_copy_peers: 1-4 sources with one token and one group stride each");
  TORCH_CHECK(!dst_ptrs.empty() && dst_ptrs.size() <= 8,
              "pkv_chunk_copy_peers: 1-8 destination groups");
  const uint16_t* ptrs[4] = {};
  for (size_t i = 0; i < srcs.size(); ++i) {
    TORCH_CHECK(srcs[i].is_cuda() && srcs[i].scalar_type() == at::kBFloat16 &&
                    srcs[i].device() == srcs[0].device(),
                "pkv_chunk_copy_peers: sources must be bf16 tensors on one device");
    ptrs[i] = reinterpret_cast<const uint16_t*>(srcs[i].data_ptr());
  }
  uint16_t* dsts[8] = {};
  for (size_t g = 0; g < dst_ptrs.size(); ++g)
    dsts[g] = reinterpret_cast<uint16_t*>(static_cast<uintptr_t>(dst_ptrs[g]));
  const c10::cuda::CUDAGuard guard(srcs[0].device());
  check_rc(pkv_chunk_copy_peers(ptrs, src_ts.data(), src_gs.data(), int(srcs.size()), dsts,
                                dst_ts, dst_is, tokens, int(dst_ptrs.size()), int(group_elems),
                                stream_of(srcs[0])),
           "pkv_chunk_copy_peers");
}

// 3D RoPE of a query block of one sample: x [tokens, H, D] bf16 (last dim
// contiguous), tables float64 [rows, cols * 2] (re, im) for the t / y / x
// parts; returns a new [tokens, H, D] tensor (causal_model.py:30-63).
Tensor op_rope_q(Tensor x, Tensor ft, Tensor fy, Tensor fx, int64_t start_frame, int64_t frames,
                 int64_t grid_h, int64_t grid_w) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 3,
              "pkv_rope_q: x must be a [tokens, H, D] bf16 CUDA tensor");
  for (const Tensor* t : {&ft, &fy, &fx})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kDouble && t->dim() == 2 &&
                    t->is_contiguous() && t->size(1) % 2 == 0 && t->device() == x.device(),
                "pkv_rope_q: tables must be contiguous [rows, cols * 2] float64 on x's device");
  const c10::cuda::CUDAGuard g(x.device());
  auto xx = x.stride(2) == 1 ? x : x.contiguous();
  auto out = at::empty(x.sizes(), x.options());
  check_rc(pkv_rope_q(reinterpret_cast<const uint16_t*>(xx.data_ptr()), xx.stride(0),
                      xx.stride(1), reinterpret_cast<uint16_t*>(out.data_ptr()), out.stride(0),
                      out.stride(1), x.size(0), int(x.size(1)), int(x.size(2)), start_frame,
                      int(frames), int(grid_h), int(grid_w), ft.data_ptr<double>(),
                      int(ft.size(0)), int(ft.size(1) / 2), fy.data_ptr<double>(),
                      int(fy.size(0)), int(fy.size(1) / 2), fx.data_ptr<double>(),
                      int(fx.size(0)), int(fx.size(1) / 2), stream_of(xx)),
           "pkv_rope_q");
  return out;
}

int64_t op_status(Mgr mgr) { return take_status(mgr); }
int64_t op_rope_rounding(int64_t mode) { return pkv_set_rope_rounding(int(mode)); }

// ---- AdaptiveKVCache / CppStrategyManager ops (scatter_copy_bind.cpp:449-684) ----
void check_i64_1d(const Tensor& t, const char* name, int64_t n, const Tensor& like) {
  TORCH_CHECK(t.is_cuda() && t.dtype() == at::kLong && t.dim() == 1 && t.is_contiguous(),
              name, " must be a contiguous 1-D int64 CUDA tensor");
  TORCH_CHECK(t.size(0) >= n, name, " is too small");
  TORCH_CHECK(t.device() == like.device(), name, ": device mismatch");
}

void scatter_copy(Tensor src_ptrs, Tensor lengths, Tensor offsets, Tensor dst, int64_t col_dim) {
  TORCH_CHECK(dst.is_cuda() && dst.is_contiguous(), "scatter_copy: dst must be contiguous CUDA");
  const int64_t n = src_ptrs.size(0);
  if (n == 0) return;
  check_i64_1d(src_ptrs, "src_ptrs", n, dst);
  check_i64_1d(lengths, "lengths", n, dst);
  check_i64_1d(offsets, "offsets", n, dst);
  c10::cuda::CUDAGuard g(dst.device());
  check_rc(pkv_scatter_copy(src_ptrs.data_ptr<int64_t>(), lengths.data_ptr<int64_t>(),
                            offsets.data_ptr<int64_t>(), dst.data_ptr(),
                            col_dim * int64_t(dst.element_size()), int(n), stream_of(dst)),
           "scatter_copy");
}

void apply_pos_override(Tensor pos, Tensor starts, Tensor ends, Tensor vals) {
  TORCH_CHECK(pos.is_cuda() && pos.dtype() == at::kLong && pos.dim() == 2 && pos.size(1) == 3 &&
                  pos.is_contiguous(),
              "apply_pos_override: pos must be a contiguous [N, 3] int64 CUDA tensor");
  const int64_t m = starts.size(0);
  if (m == 0) return;
  check_i64_1d(starts, "starts", m, pos);
  check_i64_1d(ends, "ends", m, pos);
  check_i64_1d(vals, "vals", m, pos);
  c10::cuda::CUDAGuard g(pos.device());
  check_rc(pkv_pos_override(pos.data_ptr<int64_t>(), starts.data_ptr<int64_t>(),
                            ends.data_ptr<int64_t>(), vals.data_ptr<int64_t>(), int(m),
                            stream_of(pos)),
           "apply_pos_override");
}

// Host list of tensor addresses -> device int64 array, on the current stream.
// The host copy is staged before cudaMemcpyAsync returns (pageable source).
void copy_ptrs(const std::vector<Tensor>& ts, Tensor dst, const Tensor& like, const char* name) {
  std::vector<int64_t> host;
  host.reserve(ts.size());
  for (size_t i = 0; i < ts.size(); ++i) {
    TORCH_CHECK(ts[i].is_cuda() && ts[i].is_contiguous(), name, "[", i,
                "] must be a contiguous CUDA tensor");
    TORCH_CHECK(ts[i].device() == like.device(), name, "[", i, "] is on another device");
    host.push_back(reinterpret_cast<int64_t>(ts[i].data_ptr()));
  }
  if (host.empty()) return;
  C10_CUDA_CHECK(cudaMemcpyAsync(dst.data_ptr<int64_t>(), host.data(),
                                 host.size() * sizeof(int64_t), cudaMemcpyHostToDevice,
                                 static_cast<cudaStream_t>(stream_of(dst))));
}

int mapping_mode_code(const std::string& mode) {
  if (mode == "relative_clamp") return 1;
  if (mode == "relative_softcap") return 2;
  return 0;  // "none" and anything else (scatter_copy_bind.cpp:484-489)
}

void refresh_readout_layout(std::vector<Tensor> src_k, std::vector<Tensor> src_v,
                            std::vector<Tensor> src_pos, Tensor src_ptrs_k, Tensor src_ptrs_v,
                            Tensor src_ptrs_pos, Tensor offsets, Tensor lengths, Tensor flags,
                            Tensor dynamic_rope_t, Tensor dst_k_raw, Tensor dst_v,
                            Tensor dst_rope_pos, Tensor dst_frame_ids, int64_t head_dim,
                            int64_t current_t, std::string mode, int64_t rel_max,
                            double soft_factor) {
  const int64_t n = int64_t(src_k.size());
  TORCH_CHECK(src_v.size() == src_k.size() && src_pos.size() == src_k.size(),
              "refresh_readout_layout: src_k / src_v / src_pos lengths differ");
  if (n == 0) return;
  for (const Tensor* t : {&dst_k_raw, &dst_v, &dst_rope_pos, &dst_frame_ids})
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->device() == dst_k_raw.device(),
                "refresh_readout_layout: destinations must be contiguous on one CUDA device");
  TORCH_CHECK(dst_rope_pos.dtype() == at::kLong && dst_frame_ids.dtype() == at::kLong,
              "refresh_readout_layout: dst_rope_pos / dst_frame_ids must be int64");
  TORCH_CHECK(dst_k_raw.dtype() == dst_v.dtype(), "refresh_readout_layout: dst dtype mismatch");
  TORCH_CHECK(dst_k_raw.size(1) == head_dim && dst_v.size(1) == head_dim,
              "refresh_readout_layout: head_dim mismatch");
  TORCH_CHECK(dst_rope_pos.size(1) == 3, "refresh_readout_layout: dst_rope_pos must be [N, 3]");
  for (const auto& pr : {std::make_pair(&src_ptrs_k, "src_ptrs_k"),
                         std::make_pair(&src_ptrs_v, "src_ptrs_v"),
                         std::make_pair(&src_ptrs_pos, "src_ptrs_pos"),
                         std::make_pair(&offsets, "offsets"), std::make_pair(&lengths, "lengths"),
                         std::make_pair(&flags, "flags"),
                         std::make_pair(&dynamic_rope_t, "dynamic_rope_t")})
    check_i64_1d(*pr.first, pr.second, n, dst_k_raw);
  for (int64_t i = 0; i < n; ++i) {
    TORCH_CHECK(src_k[i].dtype() == dst_k_raw.dtype() && src_v[i].dtype() == dst_v.dtype(),
                "refresh_readout_layout: source dtype mismatch");
    TORCH_CHECK(src_pos[i].dtype() == at::kLong && src_pos[i].size(1) == 3,
                "refresh_readout_layout: src_pos must be [rows, 3] int64");
    TORCH_CHECK(src_k[i].size(1) == head_dim && src_v[i].size(1) == head_dim,
                "refresh_readout_layout: source head_dim mismatch");
  }
  c10::cuda::CUDAGuard g(dst_k_raw.device());
  copy_ptrs(src_k, src_ptrs_k, dst_k_raw, "src_k");
  copy_ptrs(src_v, src_ptrs_v, dst_k_raw, "src_v");
  copy_ptrs(src_pos, src_ptrs_pos, dst_k_raw, "src_pos");
  check_rc(pkv_refresh_readout_layout(
               src_ptrs_k.data_ptr<int64_t>(), src_ptrs_v.data_ptr<int64_t>(),
               src_ptrs_pos.data_ptr<int64_t>(), offsets.data_ptr<int64_t>(),
               lengths.data_ptr<int64_t>(), flags.data_ptr<int64_t>(),
               dynamic_rope_t.data_ptr<int64_t>(), dst_k_raw.data_ptr(), dst_v.data_ptr(),
               dst_rope_pos.data_ptr<int64_t>(), dst_frame_ids.data_ptr<int64_t>(),
               head_dim * int64_t(dst_k_raw.element_size()), current_t, mapping_mode_code(mode),
               rel_max, float(soft_factor), int(n), stream_of(dst_k_raw)),
           "refresh_readout_layout");
}

void anchor_store_write_frames(Tensor k_seq, Tensor v_seq, Tensor pos_seq, Tensor frame_desc,
                               Tensor store_k, Tensor store_v, Tensor store_pos) {
  for (const Tensor* t : {&k_seq, &v_seq, &pos_seq, &frame_desc, &store_k, &store_v, &store_pos})
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->device() == store_k.device(),
                "anchor_store_write_frames: tensors must be contiguous on one CUDA device");
  TORCH_CHECK(k_seq.dtype() == store_k.dtype() && v_seq.dtype() == store_v.dtype(),
              "anchor_store_write_frames: K/V dtype mismatch");
  TORCH_CHECK(pos_seq.dtype() == at::kLong && store_pos.dtype() == at::kLong &&
                  frame_desc.dtype() == at::kLong,
              "anchor_store_write_frames: pos / frame_desc must be int64");
  TORCH_CHECK(k_seq.dim() == 2 && v_seq.dim() == 2 && pos_seq.dim() == 2 && pos_seq.size(1) == 3,
              "anchor_store_write_frames: k_seq / v_seq [tokens, D], pos_seq [tokens, 3]");
  TORCH_CHECK(frame_desc.dim() == 2 && frame_desc.size(1) == 2,
              "anchor_store_write_frames: frame_desc must be [N, 2]");
  TORCH_CHECK(store_k.dim() == 3 && store_v.dim() == 3 && store_pos.dim() == 3 &&
                  store_pos.size(2) == 3,
              "anchor_store_write_frames: stores must be [capacity, frame_seqlen, D / 3]");
  TORCH_CHECK(store_k.size(1) == store_v.size(1) && store_k.size(2) == store_v.size(2) &&
                  store_pos.size(1) == store_k.size(1),
              "anchor_store_write_frames: store shapes disagree");
  TORCH_CHECK(k_seq.size(1) == store_k.size(2) && v_seq.size(1) == store_v.size(2),
              "anchor_store_write_frames: head_dim mismatch");
  const int64_t n = frame_desc.size(0);
  if (n == 0) return;
  c10::cuda::CUDAGuard g(store_k.device());
  check_rc(pkv_anchor_store_write_frames(
               k_seq.data_ptr(), v_seq.data_ptr(), pos_seq.data_ptr<int64_t>(),
               frame_desc.data_ptr<int64_t>(), store_k.data_ptr(), store_v.data_ptr(),
               store_pos.data_ptr<int64_t>(), store_k.size(1),
               store_k.size(2) * int64_t(store_k.element_size()), int(n), stream_of(store_k)),
           "anchor_store_write_frames");
}
// pyramidkv_plan.cc:48-173: current_t and pass_kind are accepted and unused,
// as there; the five descriptor tensors are new device tensors.
std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor> pyramidkv_plan(Mgr mgr, int64_t, int64_t) {
  TORCH_CHECK(mgr.get() != nullptr, "pyramidkv_plan: manager is null");
  const int64_t n = mgr->num_layers() * mgr->num_heads();
  auto i32 = at::TensorOptions().dtype(at::kInt).device(mgr->device());
  Tensor cu = at::empty({n + 1}, i32), sk = at::empty({n * 3}, i32), sg = at::empty({n * 3}, i32);
  Tensor sl = at::empty({n * 3}, i32), dst = at::empty({n * 3}, i32);
  c10::cuda::CUDAGuard g(mgr->device());
  auto c = mgr->view();
  check_rc(pkv_legacy_plan(&c, cu.data_ptr<int32_t>(), sk.data_ptr<int32_t>(),
                           sg.data_ptr<int32_t>(), sl.data_ptr<int32_t>(),
                           dst.data_ptr<int32_t>(), stream_of(cu)),
           "pyramidkv_plan");
  return {cu, sk, sg, sl, dst};
}

// ---- Meta kernels (shape-only) ----
Plan7 mega_plan_meta_impl(const Mgr& mgr, int64_t C) {
  const int64_t H = mgr->num_heads(), S = mgr->max_total() + PKV_MAX_MERGE_BLOCKS;
  auto i32 = at::TensorOptions().dtype(at::kInt).device(at::kMeta);
  auto i64 = at::TensorOptions().dtype(at::kLong).device(at::kMeta);
  return {at::empty({C * H + 1}, i32), at::empty({C * H * S}, i32), at::empty({C * H * S}, i32),
          at::empty({C * H * S}, i32), at::empty({C * H * S}, i32), at::empty({C * H * S}, i64),
          at::empty({C * H * S}, i64)};
}
Plan7 mega_plan_meta(Mgr mgr, Tensor, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                     int64_t, int64_t, int64_t, double) {
  return mega_plan_meta_impl(mgr, 1);
}
Plan7 mega_plan_multi_meta(Mgr mgr, Tensor, int64_t, Tensor t, int64_t, int64_t, int64_t,
                           int64_t, int64_t, int64_t, int64_t, double) {
  return mega_plan_meta_impl(mgr, t.numel());
}

}  // namespace pkv_torch

using namespace pkv_torch;

TORCH_LIBRARY(adahead, m) {
  m.class_<PyramidKVCacheManager>("PyramidKVCacheManager")
      .def(torch::init<int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                       const std::string&, const std::string&, int64_t>())
      .def("reset", &PyramidKVCacheManager::reset)
      .def("set_strategy", &PyramidKVCacheManager::set_strategy)
      .def("sink_pool", &PyramidKVCacheManager::sink_pool)
      .def("middle_pool", &PyramidKVCacheManager::middle_pool)
      .def("recent_pool", &PyramidKVCacheManager::recent_pool)
      .def("sink_k_pool", &PyramidKVCacheManager::sink_k_pool)
      .def("sink_v_pool", &PyramidKVCacheManager::sink_v_pool)
      .def("middle_k_pool", &PyramidKVCacheManager::middle_k_pool)
      .def("middle_v_pool", &PyramidKVCacheManager::middle_v_pool)
      .def("recent_k_pool", &PyramidKVCacheManager::recent_k_pool)
      .def("recent_v_pool", &PyramidKVCacheManager::recent_v_pool)
      .def("sink_pos_pool", &PyramidKVCacheManager::sink_pos_pool)
      .def("middle_pos_pool", &PyramidKVCacheManager::middle_pos_pool)
      .def("recent_pos_pool", &PyramidKVCacheManager::recent_pos_pool)
      .def("head_t_table", &PyramidKVCacheManager::head_t_table)
      .def("write_idx", &PyramidKVCacheManager::write_idx)
      .def("valid_count", &PyramidKVCacheManager::valid_count)
      .def("strategy", &PyramidKVCacheManager::strategy)
      .def("k_flat_out", &PyramidKVCacheManager::k_flat_out)
      .def("v_flat_out", &PyramidKVCacheManager::v_flat_out)
      .def("cu_seqlens_k", &PyramidKVCacheManager::cu_seqlens_k)
      .def("pos_flat_out", &PyramidKVCacheManager::pos_flat_out)
      .def("merge_k_pool", &PyramidKVCacheManager::merge_k_pool)
      .def("merge_v_pool", &PyramidKVCacheManager::merge_v_pool)
      .def("merge_pos_pool", &PyramidKVCacheManager::merge_pos_pool)
      .def("merge_token_count", &PyramidKVCacheManager::merge_token_count)
      .def("merge_accum_sum_k", &PyramidKVCacheManager::merge_accum_sum_k)
      .def("merge_accum_sum_v", &PyramidKVCacheManager::merge_accum_sum_v)
      .def("merge_accum_pos", &PyramidKVCacheManager::merge_accum_pos)
      .def("merge_accum_group_ids", &PyramidKVCacheManager::merge_accum_group_ids)
      .def("merge_accum_tokens_per_group", &PyramidKVCacheManager::merge_accum_tokens_per_group)
      .def("merge_accum_num_groups", &PyramidKVCacheManager::merge_accum_num_groups)
      .def("max_merge_blocks", &PyramidKVCacheManager::max_merge_blocks)
      .def("max_merge_active", &PyramidKVCacheManager::max_merge_active)
      .def("max_merge_tokens_per_anchor", &PyramidKVCacheManager::max_merge_tokens_per_anchor)
      .def("num_layers", &PyramidKVCacheManager::num_layers)
      .def("num_heads", &PyramidKVCacheManager::num_heads)
      .def("head_dim", &PyramidKVCacheManager::head_dim)
      .def("frame_seqlen", &PyramidKVCacheManager::frame_seqlen)
      .def("max_sink", &PyramidKVCacheManager::max_sink)
      .def("max_middle", &PyramidKVCacheManager::max_middle)
      .def("max_recent", &PyramidKVCacheManager::max_recent)
      .def("max_total", &PyramidKVCacheManager::max_total)
      .def("max_total_tokens", &PyramidKVCacheManager::max_total_tokens)
      .def("max_attend_chunks", &PyramidKVCacheManager::max_attend_chunks)
      .def("max_pack_tokens", &PyramidKVCacheManager::max_pack_tokens)
      .def("status_word", &PyramidKVCacheManager::status_word)
      .def("scratch", &PyramidKVCacheManager::scratch)
      .def("set_block_time", &PyramidKVCacheManager::set_block_time)
      .def("clear_block_time", &PyramidKVCacheManager::clear_block_time);

  m.def("scatter_copy(Tensor src_ptrs, Tensor lengths, Tensor offsets, Tensor(a!) dst, "
        "int col_dim) -> ()");
  m.def("apply_pos_override(Tensor(a!) pos, Tensor starts, Tensor ends, Tensor vals) -> ()");
  m.def("anchor_store_write_frames(Tensor k_seq, Tensor v_seq, Tensor pos_seq, "
        "Tensor frame_desc, Tensor(a!) store_k, Tensor(b!) store_v, Tensor(c!) store_pos) -> ()");
  m.def("refresh_readout_layout(Tensor[] src_k, Tensor[] src_v, Tensor[] src_pos, "
        "Tensor(a!) src_ptrs_k, Tensor(b!) src_ptrs_v, Tensor(c!) src_ptrs_pos, "
        "Tensor offsets, Tensor lengths, Tensor flags, Tensor dynamic_rope_t, "
        "Tensor(d!) dst_k_raw, Tensor(e!) dst_v, Tensor(f!) dst_rope_pos, "
        "Tensor(g!) dst_frame_ids, int head_dim, int current_t, "
        "str history_time_mapping_mode, int history_relative_t_max, "
        "float history_time_soft_factor) -> ()");
  m.def("pyramidkv_pack(__torch__.torch.classes.adahead.PyramidKVCacheManager mgr, "
        "Tensor src_kind, Tensor src_slot_global, Tensor seg_lengths, Tensor dst_token_offsets, "
        "Tensor anchor_t_remap, Tensor freqs_ft_flat, Tensor freqs_fy_flat, "
        "Tensor freqs_fx_flat) -> ()");
  m.def("pyramidkv_plan(__torch__.torch.classes.adahead.PyramidKVCacheManager mgr, "
        "int current_t, int pass_kind) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def("pyramidkv_update(__torch__.torch.classes.adahead.PyramidKVCacheManager mgr, "
        "Tensor new_k, Tensor new_v, Tensor new_pos, Tensor dst_kind, Tensor dst_slot_global, "
        "Tensor src_frame_in_block, Tensor src_head) -> ()");
  m.def("mega_state_update(Tensor(a!) states, Tensor new_t_vals, Tensor(b!) desc_dst_kind, "
        "Tensor(c!) desc_dst_slot, Tensor(d!) desc_src_frame, Tensor(e!) desc_src_head, "
        "Tensor(f!) desc_merge_accum_slot, Tensor(g!) desc_merge_local_idx, "
        "Tensor(h!) desc_merge_finalize_completed_idx, Tensor(i!) desc_merge_is_new_block, "
        "int num_heads, int frames_in_block, int pass_kind) -> ()");
  m.def("mega_plan(__torch__.torch.classes.adahead.PyramidKVCacheManager mgr, "
        "Tensor states_bytes, int layer_idx, int current_t, int pass_kind, "
        "int sink_mode_code, int sink_clamp_min, int sink_clamp_max, int decoupled_sink_lag, "
        "int hist_mode_code, int hist_relative_t_max, float hist_soft_factor) "
        "-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def("mega_plan_multi(__torch__.torch.classes.adahead.PyramidKVCacheManager mgr, "
        "Tensor states_bytes, int layer_idx, Tensor current_t_list, int pass_kind, "
        "int sink_mode_code, int sink_clamp_min, int sink_clamp_max, int decoupled_sink_lag, "
        "int hist_mode_code, int hist_relative_t_max, float hist_soft_factor) "
        "-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def("mega_state_perhead_size() -> int");
  m.def("mega_merge_accum(Tensor states, Tensor new_k, Tensor new_v, Tensor new_pos, "
        "Tensor desc_dst_kind, Tensor desc_merge_accum_slot, "
        "Tensor desc_merge_finalize_completed_idx, Tensor desc_merge_is_new_block, "
        "Tensor(a!) accum_sum_k, Tensor(b!) accum_sum_v, Tensor(c!) accum_pos, "
        "Tensor(d!) accum_group_ids, Tensor(e!) accum_tokens_per_group, "
        "Tensor(f!) accum_num_groups, Tensor(g!) merge_k_pool, Tensor(h!) merge_v_pool, "
        "Tensor(i!) merge_pos_pool, Tensor(j!) merge_token_count) -> ()");

  // additions
  m.def("pkv_cache_update(__torch__.torch.classes.adahead.PyramidKVCacheManager mgr, "
        "Tensor(a!) states_bytes, int layer_idx, Tensor new_k, Tensor new_v, int first_t, "
        "int pass_kind, Tensor sink_caps, Tensor(b!) committed_vc, Tensor(c!) committed_k, "
        "Tensor(d!) committed_v, Tensor(e!) committed_pos, int spatial_width, "
        "bool has_merge_head) -> ()");
  m.def("pkv_attend(__torch__.torch.classes.adahead.PyramidKVCacheManager mgr, "
        "Tensor states_layer, int layer_idx, Tensor q, int first_t, int sink_mode_code, "
        "int sink_clamp_min, int sink_clamp_max, int decoupled_sink_lag, Tensor freqs_ft_flat, "
        "Tensor freqs_fy_flat, Tensor freqs_fx_flat, float softmax_scale, "
        "Tensor(a!) token_counter) -> Tensor");
  m.def("pkv_attend_pack(__torch__.torch.classes.adahead.PyramidKVCacheManager mgr, "
        "Tensor states_layer, int layer_idx, int L_q, int first_t, int sink_mode_code, "
        "int sink_clamp_min, int sink_clamp_max, int decoupled_sink_lag, Tensor freqs_ft_flat, "
        "Tensor freqs_fy_flat, Tensor freqs_fx_flat, Tensor(a!) token_counter) -> ()");
  m.def("pkv_attend_attention(__torch__.torch.classes.adahead.PyramidKVCacheManager mgr, "
        "Tensor q, float softmax_scale) -> Tensor");
  m.def("pkv_attention(Tensor q, Tensor k, Tensor v, Tensor cu_seqlens_k, int num_chunks, "
        "int rows_per_chunk, float softmax_scale) -> Tensor");
  m.def("pkv_attention_ws(Tensor q, Tensor k, Tensor v, Tensor cu_seqlens_k, int num_chunks, "
        "int rows_per_chunk, float softmax_scale, Tensor(a!) workspace) -> Tensor");
  m.def("pkv_attention_ws_bytes(int num_chunks, int num_heads, int rows_per_chunk) -> int");
  m.def("pkv_chunk_copy(Tensor[] srcs, int[] src_tok_strides, int[] src_group_strides, "
        "Tensor(a!) dst, int dst_tok_stride, int dst_group_stride, int dst_src_stride, "
        "int tokens, int groups, int group_elems) -> ()");
  m.def("pkv_chunk_copy_peers(Tensor[] srcs, int[] src_tok_strides, int[] src_group_strides, "
        "int[] dst_ptrs, int dst_tok_stride, int dst_src_stride, int tokens, "
        "int group_elems) -> ()");
  m.def("pkv_status(__torch__.torch.classes.adahead.PyramidKVCacheManager mgr) -> int");
  m.def("pkv_rope_rounding(int mode) -> int");
  m.def("pkv_rope_q(Tensor x, Tensor ft, Tensor fy, Tensor fx, int start_frame, int frames, "
        "int grid_h, int grid_w) -> Tensor");
}

TORCH_LIBRARY_IMPL(adahead, CUDA, m) {
  m.impl("scatter_copy", scatter_copy);
  m.impl("apply_pos_override", apply_pos_override);
  m.impl("anchor_store_write_frames", anchor_store_write_frames);
  m.impl("refresh_readout_layout", refresh_readout_layout);
  m.impl("pyramidkv_pack", pyramidkv_pack);
  m.impl("pyramidkv_update", pyramidkv_update);
  m.impl("mega_state_update", mega_state_update);
  m.impl("mega_merge_accum", mega_merge_accum);
  m.impl("pkv_cache_update", op_cache_update);
  m.impl("pkv_attend", op_attend);
  m.impl("pkv_rope_q", op_rope_q);
  m.impl("pkv_attend_pack", op_attend_pack);
  m.impl("pkv_attend_attention", op_attend_attention);
  m.impl("pkv_attention", op_attention);
  m.impl("pkv_attention_ws", op_attention_ws);
  m.impl("pkv_chunk_copy", op_chunk_copy);
  m.impl("pkv_chunk_copy_peers", op_chunk_copy_peers);
}

TORCH_LIBRARY_IMPL(adahead, CompositeExplicitAutograd, m) {
  m.impl("pyramidkv_plan", pyramidkv_plan);
  m.impl("mega_state_perhead_size", mega_state_perhead_size);
  m.impl("mega_plan", mega_plan);
  m.impl("mega_plan_multi", mega_plan_multi);
  m.impl("pkv_status", op_status);
  m.impl("pkv_attention_ws_bytes", op_attention_ws_bytes);
  m.impl("pkv_rope_rounding", op_rope_rounding);
}

TORCH_LIBRARY_IMPL(adahead, Meta, m) {
  m.impl("scatter_copy", [](Tensor, Tensor, Tensor, Tensor, int64_t) {});
  m.impl("apply_pos_override", [](Tensor, Tensor, Tensor, Tensor) {});
  m.impl("anchor_store_write_frames", [](Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor) {});
  m.impl("refresh_readout_layout",
         [](std::vector<Tensor>, std::vector<Tensor>, std::vector<Tensor>, Tensor, Tensor, Tensor,
            Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, int64_t, int64_t,
            std::string, int64_t, double) {});
  m.impl("pyramidkv_pack", [](Mgr, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor) {});
  m.impl("pyramidkv_update", [](Mgr, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor) {});
  m.impl("mega_state_update", [](Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor,
                                 Tensor, Tensor, int64_t, int64_t, int64_t) {});
  m.impl("mega_merge_accum", [](Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor,
                                Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor,
                                Tensor, Tensor) {});
  m.impl("mega_plan", mega_plan_meta);
  m.impl("mega_plan_multi", mega_plan_multi_meta);
  m.impl("pkv_attention", [](Tensor q, Tensor, Tensor, Tensor, int64_t, int64_t, double) {
    return at::empty_like(q);
  });
}
