"""Fused query RoPE (adahead.pkv_rope_q via pyramidkv.rope.causal_rope_apply)
against the reference's own outputs (golden vectors) and the oracle, bit for
bit, including tokens past the grid, the last rows of the tables and a
strided (non-contiguous head) input."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import pkv_oracle as O

pytestmark = pytest.mark.gpu


def _bf(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)


def _u16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def test_fused_rope_matches_reference_golden(cuda):
    from pyramidkv import rope
    g = np.load(os.path.join(GOLDEN, "rope_q.npz"))
    _, full = O.rope_freq_tables(128)
    for i in range(int(g["n_cases"])):
        F, Hg, Wg, start, heads, pad = (int(v) for v in g[f"c{i}_dims"])
        x = _bf(g[f"c{i}_x"], cuda)
        y = rope.causal_rope_apply(x, torch.tensor([[F, Hg, Wg]]), full, start_frame=start)
        np.testing.assert_array_equal(_u16(y), g[f"c{i}_y"], err_msg=f"case {i}")


def test_fused_rope_strided_input_matches_oracle(cuda):
    from pyramidkv import rope
    rng = np.random.default_rng(2)
    _, full = O.rope_freq_tables(128)
    F, Hg, Wg, start = 3, 30, 52, 12
    L, n = F * Hg * Wg, 12
    qkv = O.f32_to_bf16(rng.standard_normal((1, L, 3 * n, 128)).astype(np.float32) * 3)
    x = _bf(qkv, cuda)[:, :, n:2 * n]               # a head slice: token stride 3 n D
    y = rope.causal_rope_apply(x, None, full, start_frame=start, grid_int=[(F, Hg, Wg)])
    want = O.rope_q(qkv[0, :, n:2 * n], full, start, F, Hg, Wg)
    np.testing.assert_array_equal(_u16(y)[0], want)
