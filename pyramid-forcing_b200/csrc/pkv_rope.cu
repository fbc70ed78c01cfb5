// 3D RoPE of the query block, fused: the model-side step before attend.
//
// Reference behaviour: causal_rope_apply, wan/modules/causal_model.py:30-63:
// x (bf16) is widened to float64, pairs (2i, 2i+1) of head_dim are complex
// numbers, token s = (f, h, w) of the block's F x Hg x Wg grid is multiplied by
// freqs_t[start_frame + f] (pairs [0, ct)), freqs_y[h] (the next cy pairs) and
// freqs_x[w] (the rest), in complex128, and the result is cast back to bf16
// the way torch casts float64 to bf16: to float32, then to bf16, each to
// nearest even.  Tokens past F * Hg * Wg pass through.
//
// B200 design: the op is a pure streaming pass (16 bytes in, 16 bytes out per
// 4 complex pairs), so one thread owns a 16-byte chunk of a (token, head) row;
// the frequency tables (about 1 MB of float64) stay in L2.  The products are
// evaluated as a*c - b*d and a*d + b*c without contraction, each operation
// rounded to float64.
#include "pkv_common.cuh"

namespace pkv {
namespace {

__global__ void __launch_bounds__(256)
    rope_q_kernel(const uint16_t* x, int64_t x_tok, int64_t x_head, uint16_t* out,
                  int64_t o_tok, int64_t o_head, int64_t tokens, int heads, int chunks,
                  int64_t start_frame, int F, int Hg, int Wg, const double* ft, int ct,
                  const double* fy, int cy, const double* fx, int cx) {
  const int64_t n = tokens * heads * chunks;
  const int64_t grid_tok = int64_t(F) * Hg * Wg;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int ch = int(i % chunks);
    const int64_t th = i / chunks;
    const int h = int(th % heads);
    const int64_t tok = th / heads;
    const uint4 w = *reinterpret_cast<const uint4*>(x + tok * x_tok + h * x_head + ch * 8);
    uint4 r = w;
    if (tok < grid_tok) {
      const int f = int(tok / (int64_t(Hg) * Wg));
      const int rem = int(tok - int64_t(f) * Hg * Wg);
      const int hh = rem / Wg, ww = rem - (rem / Wg) * Wg;
      uint32_t in[4] = {w.x, w.y, w.z, w.w}, o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int p = ch * 4 + j;
        const double* tab;
        if (p < ct) tab = ft + ((start_frame + f) * ct + p) * 2;
        else if (p < ct + cy) tab = fy + (int64_t(hh) * cy + (p - ct)) * 2;
        else tab = fx + (int64_t(ww) * cx + (p - ct - cy)) * 2;
        const double c = __ldg(tab), d = __ldg(tab + 1);
        const double a = double(bf16_bits_to_f32(in[j] & 0xffffu));
        const double b = double(bf16_bits_to_f32(in[j] >> 16));
        const double re = __dsub_rn(__dmul_rn(a, c), __dmul_rn(b, d));
        const double im = __dadd_rn(__dmul_rn(a, d), __dmul_rn(b, c));
        // float64 -> float32 -> bf16, each to nearest even: torch's cast
        o[j] = f32_to_bf16_bits(__double2float_rn(re)) |
               (f32_to_bf16_bits(__double2float_rn(im)) << 16);
      }
      r = make_uint4(o[0], o[1], o[2], o[3]);
    }
    *reinterpret_cast<uint4*>(out + tok * o_tok + h * o_head + ch * 8) = r;
  }
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_rope_q(const uint16_t* x, int64_t x_tok_stride, int64_t x_head_stride,
                          uint16_t* out, int64_t o_tok_stride, int64_t o_head_stride,
                          int64_t tokens, int heads, int head_dim, int64_t start_frame,
                          int frames, int grid_h, int grid_w, const double* freqs_t,
                          int t_rows, int t_cols, const double* freqs_y, int y_rows,
                          int y_cols, const double* freqs_x, int x_rows, int x_cols,
                          pkv_stream_t stream) {
  if (tokens == 0 || heads == 0) return PKV_OK;
  if (!x || !out || !freqs_t || !freqs_y || !freqs_x || tokens < 0 || heads < 0 ||
      frames < 0 || grid_h <= 0 || grid_w <= 0 || start_frame < 0)
    return PKV_EINVAL;
  if (head_dim % 8 != 0 || t_cols + y_cols + x_cols != head_dim / 2) return PKV_EUNSUPPORTED;
  // every token of the grid must find its rows (the reference slices the same
  // rows and fails on a shorter table)
  if (start_frame + frames > t_rows || grid_h > y_rows || grid_w > x_rows) return PKV_ECAPACITY;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) % 16 != 0 ||
      x_tok_stride % 8 || x_head_stride % 8 || o_tok_stride % 8 || o_head_stride % 8)
    return PKV_EUNSUPPORTED;
  const int chunks = head_dim / 8;
  const int64_t n = tokens * heads * chunks;
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = int64_t(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  rope_q_kernel<<<int(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, x_tok_stride, x_head_stride, out, o_tok_stride, o_head_stride, tokens, heads, chunks,
      start_frame, frames, grid_h, grid_w, freqs_t, t_cols, freqs_y, y_cols, freqs_x, x_cols);
  return launch_status();
}
