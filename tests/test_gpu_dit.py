"""The random-init causal DiT driving the MegaCache (small configuration).

Two layers, dim 256 (2 heads x 128), FFN 512, a 4 x 8 token grid (16 x 8 x 16
latents), 2 blocks of 3 frames through the few-step loop (4 noisy passes and
a clean pass per block).  Checks that the video is finite, the cache's device
status stays clear, the cache holds what the clean passes committed (sink +
recent valid counts of 6 frames per head), and that a second run from a reset
cache and the same seeds is bit-identical.  The DiT's own arithmetic is torch;
the cache path and the cross-attention kernel inside it are pinned by the
other GPU tests.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(cuda):
    from causal_dit import CausalWanDiT, WanConfig, generate_video
    from pyramidkv import _mega_cache, policy
    cfg = WanConfig(dim=256, ffn_dim=512, freq_dim=32, text_dim=64, num_heads=2,
                    num_layers=2, text_len=16)
    model = CausalWanDiT(cfg, cuda, seed=3)
    labels = np.array([[-1, 1], [2, -1]])
    caches = _mega_cache.build_mega_caches(
        2, 2, 128, 32, 3, 24, 4, policy.compositions_from_labels(labels), device="cuda:0",
        sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18, sink_time_clamp_max=21,
        spatial_width=8, spatial_height=4, freqs=model.freqs)
    g = torch.Generator(device=cuda).manual_seed(5)
    text = torch.randn(1, cfg.text_len, cfg.text_dim, generator=g, device=cuda)
    noise = torch.randn(1, 16, 6, 8, 16, generator=g, device=cuda, dtype=torch.bfloat16)
    out = generate_video(model, caches, noise, text, generator=g)
    torch.cuda.synchronize()
    return out, caches[0].ctx


def test_dit_generates_through_megacache(cuda):
    out, ctx = _run(cuda)
    assert out.shape == (1, 16, 6, 8, 16)
    assert torch.isfinite(out.float()).all()
    assert ctx.check_status() == 0
    vc = ctx.mgr.valid_count().cpu().numpy()
    # 6 committed frames per head: sink up to its capacity, the rest in recent (<= 4)
    assert ((vc[:, :, 0] + vc[:, :, 2]) == np.minimum(6, vc[:, :, 0] + 4)).all(), vc
    out2, _ = _run(cuda)
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))
