"""3D RoPE of the query block, one fused kernel per sample.

``causal_rope_apply`` has the signature and results of the reference's
wan/modules/causal_model.py:30-63 (the model rotates Q with it before
``MegaCache.attend``; K is stored raw and rotated by the pack): pairs of
head_dim are complex numbers multiplied in float64 by the time / row / column
frequencies of each token's (frame, h, w) position and cast back to bf16 as
torch casts float64 (through float32).
The reference builds a float64 copy of the block and a broadcast frequency
tensor per call; here ``adahead.pkv_rope_q`` reads bf16 and writes bf16.
"""
from __future__ import annotations

import torch

from . import _ops

_TABLES: dict = {}


def _tables(freqs: torch.Tensor, c: int, device) -> tuple:
    """float64 (re, im) tables of the t / y / x parts of a complex128 [rows, c]
    frequency tensor, cached per tensor."""
    key = (freqs.data_ptr(), tuple(freqs.shape), str(device))
    t = _TABLES.get(key)
    if t is None:
        parts = freqs.split([c - 2 * (c // 3), c // 3, c // 3], dim=1)
        t = tuple(torch.view_as_real(p.to(device=device, dtype=torch.complex128))
                  .reshape(p.shape[0], -1).contiguous() for p in parts)
        _TABLES.clear()
        _TABLES[key] = t
    return t


def causal_rope_apply(x: torch.Tensor, grid_sizes, freqs: torch.Tensor, start_frame: int = 0,
                      grid_int=None) -> torch.Tensor:
    """x [B, L, n, 2c] bf16 on CUDA, grid_sizes [B, 3] (f, h, w), freqs
    complex128 [rows, c]; returns x rotated, same dtype (the reference's)."""
    if not x.is_cuda or x.dtype != torch.bfloat16:
        raise ValueError("causal_rope_apply: x must be a bf16 CUDA tensor")
    c = x.size(3) // 2
    ft, fy, fx = _tables(freqs, c, x.device)
    grid = grid_int if grid_int is not None else grid_sizes.tolist()
    ops = _ops.ops()
    out = [ops.pkv_rope_q(x[i], ft, fy, fx, int(start_frame), int(f), int(h), int(w))
           for i, (f, h, w) in enumerate(grid)]
    return torch.stack(out)
