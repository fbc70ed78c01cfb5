"""Causal Wan2.1 DiT forward for one block of latent frames, random init.

Architecture (Wan2.1-T2V-1.3B, the reference's ``wan/modules/model.py`` and
``causal_model.py``): patch embedding (Conv3d 16 -> 1536, kernel = stride =
(1, 2, 2)), sinusoidal time embedding (256) -> MLP -> 6 x 1536 modulation,
text embedding MLP (4096 -> 1536 -> 1536), 30 blocks of

    x = x + gate_msa * SelfAttn(LN(x) * (1 + scale_msa) + shift_msa)
    x = x + CrossAttn(LN_affine(x), text)
    x = x + gate_mlp * FFN(LN(x) * (1 + scale_mlp) + shift_mlp)

with RMSNorm on q and k (over the full 1536 channels), 12 heads x 128, FFN
8960 with tanh-GELU, and a modulated head (1536 -> 16 x 1 x 2 x 2).  In the
self-attention, K is stored raw and V as is in the block's MegaCache
(``update``), Q is rotated by the 3D RoPE at the block's frame offset
(``causal_rope_apply`` -> ``pkv_rope_q``) and attends the cache (``attend``):
the reference's call order at causal_model.py:213-227.  The cross-attention
K/V of the 512 text tokens are computed once per video per layer (the
reference's ``crossattn_cache``, causal_inference.py:909-922) and stored
head-major, so every block's cross-attention is one launch of the library's
ragged attention kernel (12 segments of 512 keys).

Weights are seeded N(0, 0.02) (modulation N(0, 1/1536), as the reference
initialises it), bf16.  The modulation arithmetic runs in bf16 here (the
reference promotes it to fp32); the DiT is timed, not checked for numerics.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class WanConfig:
    dim: int = 1536
    ffn_dim: int = 8960
    freq_dim: int = 256
    text_dim: int = 4096
    in_dim: int = 16
    out_dim: int = 16
    num_heads: int = 12
    num_layers: int = 30
    patch: tuple = (1, 2, 2)
    eps: float = 1e-6
    text_len: int = 512


def rope_table(head_dim: int, max_len: int = 1024) -> torch.Tensor:
    """complex128 [max_len, head_dim / 2]: the model's t / y / x RoPE parts
    (rope_params of sizes d - 4(d//6), 2(d//6), 2(d//6); causal_model.py:586-591)."""
    def part(dim):
        inv = 1.0 / torch.pow(10000, torch.arange(0, dim, 2).to(torch.float64).div(dim))
        ang = torch.outer(torch.arange(max_len), inv)
        return torch.polar(torch.ones_like(ang), ang)
    d = head_dim
    return torch.cat([part(d - 4 * (d // 6)), part(2 * (d // 6)), part(2 * (d // 6))], dim=1)


def sinusoidal(dim: int, t: torch.Tensor) -> torch.Tensor:
    """The reference's sinusoidal_embedding_1d (model.py:15-25)."""
    half = dim // 2
    pos = t.to(torch.float64)
    s = torch.outer(pos, torch.pow(10000, -torch.arange(half, device=t.device).to(pos).div(half)))
    return torch.cat([torch.cos(s), torch.sin(s)], dim=1)


class CausalWanDiT:
    """Weights as plain tensors on one device; ``forward`` runs one block."""

    def __init__(self, cfg: WanConfig, device, seed: int = 0):
        self.cfg = cfg
        self.device = torch.device(device)
        g = torch.Generator(device=self.device).manual_seed(seed)
        bf = torch.bfloat16
        d, ff = cfg.dim, cfg.ffn_dim

        def w(*shape, std=0.02):
            return (torch.randn(*shape, generator=g, device=self.device) * std).to(bf)

        def z(*shape):
            return torch.zeros(*shape, device=self.device, dtype=bf)
        pdim = cfg.in_dim * math.prod(cfg.patch)
        self.patch_w, self.patch_b = w(d, pdim), z(d)
        self.time_w1, self.time_b1 = w(d, cfg.freq_dim), z(d)
        self.time_w2, self.time_b2 = w(d, d), z(d)
        self.proj_w, self.proj_b = w(6 * d, d), z(6 * d)
        self.text_w1, self.text_b1 = w(d, cfg.text_dim), z(d)
        self.text_w2, self.text_b2 = w(d, d), z(d)
        self.layers = []
        for _ in range(cfg.num_layers):
            self.layers.append({
                "qkv_w": w(3 * d, d), "qkv_b": z(3 * d),
                "o_w": w(d, d), "o_b": z(d),
                "nq": torch.ones(d, device=self.device, dtype=bf),
                "nk": torch.ones(d, device=self.device, dtype=bf),
                "n3_w": torch.ones(d, device=self.device, dtype=bf), "n3_b": z(d),
                "cq_w": w(d, d), "cq_b": z(d), "ckv_w": w(2 * d, d), "ckv_b": z(2 * d),
                "co_w": w(d, d), "co_b": z(d),
                "cnq": torch.ones(d, device=self.device, dtype=bf),
                "cnk": torch.ones(d, device=self.device, dtype=bf),
                "f1_w": w(ff, d), "f1_b": z(ff), "f2_w": w(d, ff), "f2_b": z(d),
                "mod": w(1, 6, d, std=1.0 / math.sqrt(d)),
            })
        self.head_w, self.head_b = w(pdim, d), z(pdim)
        self.head_mod = w(1, 2, d, std=1.0 / math.sqrt(d))
        self.freqs = rope_table(d // cfg.num_heads).to(self.device)
        self.cross = None

    # -- per video ---------------------------------------------------------------
    def set_text(self, context: torch.Tensor) -> None:
        """Text embedding and every layer's cross-attention K/V of the 512
        context tokens, head-major [H * 512, 128] with cu_seqlens."""
        c = self.cfg
        H, hd = c.num_heads, c.dim // c.num_heads
        ctx = F.linear(context[0].to(torch.bfloat16), self.text_w1, self.text_b1)
        ctx = F.linear(F.gelu(ctx, approximate="tanh"), self.text_w2, self.text_b2)
        n = ctx.shape[0]
        self.cross = []
        for p in self.layers:
            kv = F.linear(ctx, p["ckv_w"], p["ckv_b"])
            k = _rms(kv[:, :c.dim], p["cnk"], c.eps)
            v = kv[:, c.dim:]
            kh = k.view(n, H, hd).transpose(0, 1).contiguous().view(H * n, hd)
            vh = v.contiguous().view(n, H, hd).transpose(0, 1).contiguous().view(H * n, hd)
            self.cross.append((kh, vh))
        self.cross_cu = torch.arange(0, (H + 1) * n, n, dtype=torch.int32, device=self.device)

    # -- one block ---------------------------------------------------------------
    def forward(self, latent: torch.Tensor, t: float, caches, current_start: int,
                mode: str) -> torch.Tensor:
        """latent [1, 16, F, 60, 104] bf16 at timestep t -> the flow prediction
        of the same shape; caches: the 30 MegaCache layers."""
        from pyramidkv import _ops
        from pyramidkv.rope import causal_rope_apply
        c = self.cfg
        d, H = c.dim, c.num_heads
        hd = d // H
        _, C, Fr, Hh, Ww = latent.shape
        gh, gw = Hh // c.patch[1], Ww // c.patch[2]
        L = Fr * gh * gw
        # patch embedding as a GEMM over (c, 1, 2, 2) patches
        pt = latent[0].view(C, Fr, gh, 2, gw, 2).permute(1, 2, 4, 0, 3, 5).reshape(L, C * 4)
        x = F.linear(pt, self.patch_w, self.patch_b)
        # time embedding (one timestep for the block's frames) -> 6 modulations
        tt = torch.full((1,), float(t), device=self.device)
        e = F.linear(sinusoidal(c.freq_dim, tt).to(torch.bfloat16), self.time_w1, self.time_b1)
        e = F.linear(F.silu(e), self.time_w2, self.time_b2)
        e0 = F.linear(F.silu(e), self.proj_w, self.proj_b).view(1, 6, d)
        grid = ((Fr, gh, gw),)
        ops = _ops.ops()
        scale = hd ** -0.5
        for li, p in enumerate(self.layers):
            m = (p["mod"] + e0)[0]                      # [6, d]
            y = F.layer_norm(x, (d,), eps=c.eps) * (1 + m[1]) + m[0]
            qkv = F.linear(y, p["qkv_w"], p["qkv_b"])
            q = _rms(qkv[:, :d], p["nq"], c.eps).view(1, L, H, hd)
            k = _rms(qkv[:, d:2 * d], p["nk"], c.eps).view(1, L, H, hd)
            v = qkv[:, 2 * d:].view(1, L, H, hd)
            rq = causal_rope_apply(q, None, self.freqs, start_frame=current_start // (gh * gw),
                                   grid_int=grid)
            caches[li].update(k, v, current_start, cache_update_mode=mode)
            a = caches[li].attend(rq, current_start)
            x = x + F.linear(a.view(L, d), p["o_w"], p["o_b"]) * m[2]
            # cross-attention over the cached text K/V
            y = F.layer_norm(x, (d,), p["n3_w"], p["n3_b"], eps=c.eps)
            cq = _rms(F.linear(y, p["cq_w"], p["cq_b"]), p["cnq"], c.eps).view(L, H, hd)
            kh, vh = self.cross[li]
            ca = ops.pkv_attention(cq, kh, vh, self.cross_cu, 1, L, scale)
            x = x + F.linear(ca.view(L, d), p["co_w"], p["co_b"])
            # feed-forward
            y = F.layer_norm(x, (d,), eps=c.eps) * (1 + m[4]) + m[3]
            h1 = F.gelu(F.linear(y, p["f1_w"], p["f1_b"]), approximate="tanh")
            x = x + F.linear(h1, p["f2_w"], p["f2_b"]) * m[5]
        hm = (self.head_mod + e.view(1, 1, d))[0]
        y = F.layer_norm(x, (d,), eps=c.eps) * (1 + hm[1]) + hm[0]
        out = F.linear(y, self.head_w, self.head_b)       # [L, C * 4]
        return out.view(Fr, gh, gw, C, 2, 2).permute(3, 0, 1, 4, 2, 5).reshape(1, C, Fr, Hh, Ww)


def _rms(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """WanRMSNorm (model.py:70-86): fp32 normalisation, back to x's dtype, times weight."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)).to(x.dtype) * weight
