// Pack: gather the planned segments of the sink / middle / recent / merge
// pools into the flat K/V/pos workspace that the attention kernel reads,
// rotating K by the 3D RoPE at the remapped time.
//
// Reference behaviour: pyramidkv/csrc/pyramidkv_pack.cu:28-185.  For a
// segment with t_remap >= 0 the time row of every token is t_remap, else the
// token's stored t; y / x rows come from the stored position; rows are
// clamped into each table; pair p of the 64 complex pairs of head_dim 128
// uses the t table for p < ft_cols, the y table for the next fy_cols and the
// x table for the rest.  V and pos are copied unchanged.
//
// B200 design: a persistent grid walks (segment, 32-token tile) units; every
// thread owns one 16-byte chunk (8 bf16 = 4 complex pairs) of a token row, so
// each warp reads and writes whole 512-byte row pairs with 128-bit accesses.
// The rotation of a pair is evaluated as fma(kr, fr, -(ki*fi)) /
// fma(kr, fi, ki*fr) (kRopeFmaFirst); the reference's compiled kernel is the
// authority on which order nvcc's contraction picks, and the GPU parity tests
// pin this choice against it.
#include "pkv_common.cuh"

namespace pkv {

constexpr int kPackTile = 32;
enum RopeMode : int { kRopeFmaFirst = 0, kRopeFmaSecond = 1, kRopeNoFma = 2 };

// Process-wide rotation order (see file comment); tests may switch it to
// compare against the reference's build.
static int g_rope_mode = kRopeFmaFirst;

struct PackArgs {
  const uint16_t* k[4];
  const uint16_t* v[4];
  const int64_t* pos[4];
  int64_t rows[4];  // slot rows per pool
  uint16_t* k_out;
  uint16_t* v_out;
  int64_t* pos_out;
  int64_t out_rows;
  const int32_t *sk, *sg, *sl, *dst;
  int n_seg;
  const int64_t* tremap;
  const float *ft, *fy, *fx;
  int ft_rows, ft_cols, fy_rows, fy_cols, fx_rows, fx_cols;
  int F, MTPA, D;
  int rope;         // fused RoPE enabled
  int rope_mode;
  int32_t* status;
};

__device__ __forceinline__ void rotate(float kr, float ki, float fr, float fi, int mode,
                                       float& nr, float& ni) {
  if (mode == kRopeFmaFirst) {
    nr = __fmaf_rn(kr, fr, -__fmul_rn(ki, fi));
    ni = __fmaf_rn(kr, fi, __fmul_rn(ki, fr));
  } else if (mode == kRopeFmaSecond) {
    nr = __fmaf_rn(-ki, fi, __fmul_rn(kr, fr));
    ni = __fmaf_rn(ki, fr, __fmul_rn(kr, fi));
  } else {
    nr = __fsub_rn(__fmul_rn(kr, fr), __fmul_rn(ki, fi));
    ni = __fadd_rn(__fmul_rn(kr, fi), __fmul_rn(ki, fr));
  }
}

__device__ __forceinline__ float2 freq_of(const PackArgs& a, int p, int64_t t, int64_t y,
                                          int64_t x) {
  const float* tab;
  int rows, cols, col;
  int64_t r;
  if (p < a.ft_cols) {
    tab = a.ft; rows = a.ft_rows; cols = a.ft_cols; col = p; r = t;
  } else if (p < a.ft_cols + a.fy_cols) {
    tab = a.fy; rows = a.fy_rows; cols = a.fy_cols; col = p - a.ft_cols; r = y;
  } else {
    tab = a.fx; rows = a.fx_rows; cols = a.fx_cols; col = p - a.ft_cols - a.fy_cols; r = x;
  }
  if (tab == nullptr) return make_float2(1.0f, 0.0f);
  int row = static_cast<int>(r);
  if (row < 0) row = 0;
  if (row >= rows) row = rows - 1;
  return __ldg(reinterpret_cast<const float2*>(tab + (int64_t(row) * cols + col) * 2));
}

template <bool kVec>
__global__ void __launch_bounds__(256) pack_kernel(PackArgs a) {
  const int max_len = a.F > a.MTPA ? a.F : a.MTPA;
  const int tiles = (max_len + kPackTile - 1) / kPackTile;
  const int64_t units = int64_t(a.n_seg) * tiles;
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    const int seg = int(u / tiles);
    const int tile = int(u - int64_t(seg) * tiles);
    const int kind = a.sk[seg];
    if (kind < 0) continue;
    const int len = a.sl[seg];
    const int tok0 = tile * kPackTile;
    if (len <= 0 || tok0 >= len) continue;
    if (kind > 3) {
      if (tile == 0 && threadIdx.x == 0) flag(a.status, PKV_ST_BAD_KIND);
      continue;
    }
    const int64_t slot = a.sg[seg];
    const int64_t dst0 = a.dst[seg];
    const int stride_tok = kind == kSrcMerge ? a.MTPA : a.F;
    if (slot < 0 || slot >= a.rows[kind] || len > stride_tok || dst0 < 0 ||
        dst0 + len > a.out_rows || a.k[kind] == nullptr) {
      if (tile == 0 && threadIdx.x == 0)
        flag(a.status, dst0 + len > a.out_rows ? PKV_ST_PACK_OVERFLOW : PKV_ST_SLOT_RANGE);
      continue;
    }
    const int ntok = min(kPackTile, len - tok0);
    const int D = a.D;
    const uint16_t* sk = a.k[kind] + slot * stride_tok * D;
    const uint16_t* sv = a.v[kind] + slot * stride_tok * D;
    const int64_t* sp = a.pos[kind] ? a.pos[kind] + slot * stride_tok * 3 : nullptr;
    uint16_t* dk = a.k_out + dst0 * D;
    uint16_t* dv = a.v_out + dst0 * D;
    const bool rope = a.rope && sp != nullptr;
    const int64_t tm = rope ? a.tremap[seg] : -1;

    if (kVec) {
      const int cpr = D / 8;
      for (int i = threadIdx.x; i < ntok * cpr; i += blockDim.x) {
        const int r = i / cpr, ch = i - r * cpr;
        const int64_t e = int64_t(tok0 + r) * D + ch * 8;
        uint4 kk = *reinterpret_cast<const uint4*>(sk + e);
        const uint4 vv = *reinterpret_cast<const uint4*>(sv + e);
        if (rope) {
          const int64_t* pp = sp + int64_t(tok0 + r) * 3;
          const int64_t pt = tm >= 0 ? tm : pp[0];
          const int64_t py = pp[1], px = pp[2];
          uint32_t w[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 fq = freq_of(a, ch * 4 + j, pt, py, px);
            const float kr = bf16_bits_to_f32(w[j] & 0xffffu);
            const float ki = bf16_bits_to_f32(w[j] >> 16);
            float nr, ni;
            rotate(kr, ki, fq.x, fq.y, a.rope_mode, nr, ni);
            w[j] = f32_to_bf16_bits(nr) | (f32_to_bf16_bits(ni) << 16);
          }
          kk = make_uint4(w[0], w[1], w[2], w[3]);
        }
        *reinterpret_cast<uint4*>(dk + e) = kk;
        *reinterpret_cast<uint4*>(dv + e) = vv;
      }
    } else {
      const int ppr = D / 2;
      for (int i = threadIdx.x; i < ntok * ppr; i += blockDim.x) {
        const int r = i / ppr, p = i - r * ppr;
        const int64_t e = int64_t(tok0 + r) * D + p * 2;
        uint16_t k0 = sk[e], k1 = sk[e + 1];
        if (rope) {
          const int64_t* pp = sp + int64_t(tok0 + r) * 3;
          const int64_t pt = tm >= 0 ? tm : pp[0];
          const float2 fq = freq_of(a, p, pt, pp[1], pp[2]);
          float nr, ni;
          rotate(bf16_bits_to_f32(k0), bf16_bits_to_f32(k1), fq.x, fq.y, a.rope_mode, nr, ni);
          k0 = static_cast<uint16_t>(f32_to_bf16_bits(nr));
          k1 = static_cast<uint16_t>(f32_to_bf16_bits(ni));
        }
        dk[e] = k0;
        dk[e + 1] = k1;
        dv[e] = sv[e];
        dv[e + 1] = sv[e + 1];
      }
    }
    if (a.pos_out != nullptr && sp != nullptr) {
      int64_t* dp = a.pos_out + dst0 * 3;
      for (int e = threadIdx.x; e < ntok * 3; e += blockDim.x)
        dp[int64_t(tok0) * 3 + e] = sp[int64_t(tok0) * 3 + e];
    }
  }
}

int launch_pack(const pkv_cache_t* c, const int32_t* sk, const int32_t* sg, const int32_t* sl,
                const int32_t* dst, int n_seg, const int64_t* tremap, const float* ft,
                int ft_rows, int ft_cols, const float* fy, int fy_rows, int fy_cols,
                const float* fx, int fx_rows, int fx_cols, cudaStream_t stream) {
  if (n_seg == 0) return PKV_OK;
  if (!c || !sk || !sg || !sl || !dst || n_seg < 0 || !c->k_flat || !c->v_flat)
    return PKV_EINVAL;
  PackArgs a{};
  const int64_t lh = int64_t(c->num_layers) * c->num_heads;
  a.k[0] = c->sink_k; a.v[0] = c->sink_v; a.pos[0] = c->sink_pos; a.rows[0] = lh * c->max_sink;
  a.k[1] = c->middle_k; a.v[1] = c->middle_v; a.pos[1] = c->middle_pos;
  a.rows[1] = lh * c->max_middle;
  a.k[2] = c->recent_k; a.v[2] = c->recent_v; a.pos[2] = c->recent_pos;
  a.rows[2] = lh * c->max_recent;
  a.k[3] = c->merge_k; a.v[3] = c->merge_v; a.pos[3] = c->merge_pos;
  a.rows[3] = lh * c->max_merge_blocks;
  // pos packing needs every pool's pos (pyramidkv_pack.cu:37-42)
  a.k_out = c->k_flat;
  a.v_out = c->v_flat;
  a.pos_out = c->pos_flat;
  a.out_rows = c->max_pack_tokens;
  a.sk = sk; a.sg = sg; a.sl = sl; a.dst = dst;
  a.n_seg = n_seg;
  a.tremap = tremap;
  a.ft = ft; a.fy = fy; a.fx = fx;
  a.ft_rows = ft ? ft_rows : 0; a.ft_cols = ft ? ft_cols : 0;
  a.fy_rows = fy ? fy_rows : 0; a.fy_cols = fy ? fy_cols : 0;
  a.fx_rows = fx ? fx_rows : 0; a.fx_cols = fx ? fx_cols : 0;
  a.F = c->frame_seqlen;
  a.MTPA = c->max_merge_tokens;
  a.D = c->head_dim;
  a.rope = tremap != nullptr && (ft != nullptr || fy != nullptr || fx != nullptr);
  a.rope_mode = g_rope_mode;
  a.status = c->status;
  const int max_len = a.F > a.MTPA ? a.F : a.MTPA;
  const int64_t units = int64_t(n_seg) * ((max_len + kPackTile - 1) / kPackTile);
  int64_t grid = int64_t(sm_count()) * 8;
  if (units < grid) grid = units;
  if (grid < 1) grid = 1;
  bool vec = (a.D % 8 == 0);
  for (int i = 0; i < 4; ++i)
    vec = vec && ((reinterpret_cast<uintptr_t>(a.k[i]) | reinterpret_cast<uintptr_t>(a.v[i])) % 16 == 0);
  if (vec) pack_kernel<true><<<int(grid), 256, 0, stream>>>(a);
  else pack_kernel<false><<<int(grid), 256, 0, stream>>>(a);
  return launch_status();
}

}  // namespace pkv

using namespace pkv;

extern "C" int pkv_pack(const pkv_cache_t* c, const int32_t* src_kind,
                        const int32_t* src_slot_global, const int32_t* seg_lengths,
                        const int32_t* dst_token_offsets, int num_segments,
                        const int64_t* anchor_t_remap, const float* ft, int ft_rows,
                        int ft_cols, const float* fy, int fy_rows, int fy_cols, const float* fx,
                        int fx_rows, int fx_cols, pkv_stream_t stream) {
  return launch_pack(c, src_kind, src_slot_global, seg_lengths, dst_token_offsets,
                     num_segments, anchor_t_remap, ft, ft_rows, ft_cols, fy, fy_rows, fy_cols,
                     fx, fx_rows, fx_cols, static_cast<cudaStream_t>(stream));
}

// Select the evaluation order of the RoPE pair rotation (0: fma on the first
// product, 1: fma on the second, 2: no contraction).  Returns the previous
// order.  Not part of the reference interface; used by the parity tests.
extern "C" int pkv_set_rope_rounding(int mode) {
  const int prev = g_rope_mode;
  if (mode >= 0 && mode <= 2) g_rope_mode = mode;
  return prev;
}
