"""Few-step block-causal generation loop (the reference's
pipeline/causal_inference.py:445-502): per block of 3 latent frames, the
denoising timesteps 1000 / 750 / 500 / 250 run the DiT on the noisy block
with the cache in ``noisy`` mode (the prediction re-noised to the next
timestep in between), then one pass at timestep 0 on the denoised block
commits it to the cache (``clean``).  Flow matching with the shifted sigma
schedule of the reference's scheduler: sigma(t) = shift*s / (1 + (shift-1)*s),
s = t / 1000, x0 = x_t - sigma * flow, x_t' = (1 - sigma') x0 + sigma' noise.
"""
from __future__ import annotations

import torch

STEPS = (1000, 750, 500, 250)


def sigma(t: float, shift: float = 5.0) -> float:
    s = t / 1000.0
    return shift * s / (1.0 + (shift - 1.0) * s)


def generate_video(model, caches, noise: torch.Tensor, text: torch.Tensor,
                   steps=STEPS, frames_per_block: int = 3, generator=None,
                   hooks=None) -> torch.Tensor:
    """noise [1, 16, F, H, W] bf16 -> denoised latents of the same shape.
    ``hooks(block, pass_index)`` (optional) runs before every DiT pass."""
    model.set_text(text)
    out = torch.empty_like(noise)
    _, _, n_frames, hh, ww = noise.shape
    tokens_per_frame = (hh // model.cfg.patch[1]) * (ww // model.cfg.patch[2])
    for blk in range(n_frames // frames_per_block):
        f0 = blk * frames_per_block
        start = f0 * tokens_per_frame
        x = noise[:, :, f0:f0 + frames_per_block]
        x0 = x
        for i, t in enumerate(steps):
            if hooks:
                hooks(blk, i)
            flow = model.forward(x, float(t), caches, start, "noisy")
            x0 = x - sigma(t) * flow
            if i + 1 < len(steps):
                sn = sigma(steps[i + 1])
                nz = torch.randn(x0.shape, generator=generator, device=x0.device,
                                 dtype=x0.dtype)
                x = (1.0 - sn) * x0 + sn * nz
        out[:, :, f0:f0 + frames_per_block] = x0
        if hooks:
            hooks(blk, len(steps))
        model.forward(x0, 0.0, caches, start, "clean")
    return out
