"""The cache path at the benchmark's full sizes, through size-independent checks.

One layer with the benchmark's shape (12 heads x 128, 1560-token frames on a
52 x 30 grid, 3-frame blocks, sink 3 / middle 24 / recent 4 frames, window-clamp
RoPE remap, seeded labels) runs 14 blocks of two noisy and one clean pass, so
the middle pools and merge anchors reach their steady state.  On the last attend:
* every planned segment is whole frames plus 390-token merge anchors, the
  offsets are non-decreasing, and their total equals the device token counter;
* the attention output of sampled (chunk, head) segments matches a torch fp32
  softmax over the packed K/V that the kernel read, within the bf16 tolerance
  (max abs 2e-2, mean abs 2e-3);
* a second attend on the same cache gives the same bits;
* the device status word stays clear.
The bit-exact comparisons with the oracle run on smaller head counts in
test_gpu_megacache.py.
"""
from __future__ import annotations

import pytest
import torch

from oracle import pkv_oracle as O

pytestmark = pytest.mark.gpu

H, D, W, HG, F = 12, 128, 52, 30, 3
FSEQ = W * HG
BLOCKS = 14


def test_full_size_layer_properties(cuda):
    from pyramidkv import _mega_cache, policy
    labels = policy.random_labels(1, H, seed=0)
    _, full = O.rope_freq_tables(D)
    caches = _mega_cache.build_mega_caches(
        1, H, D, FSEQ, 3, 24, 4, policy.compositions_from_labels(labels, "baseline"),
        max_attend_chunks=8, device=str(cuda), sink_time_mapping_mode="window_clamp",
        sink_time_clamp_min=18, sink_time_clamp_max=21, spatial_width=W, spatial_height=HG,
        freqs=full)
    c = caches[0]
    c.ctx.token_counter = torch.zeros(1, dtype=torch.int64, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(5)
    rnd = lambda: torch.randn(1, F * FSEQ, H, D, generator=g, device=cuda).to(torch.bfloat16)  # noqa
    for blk in range(BLOCKS):
        start = blk * F * FSEQ
        for mode in ("noisy", "noisy", "clean"):
            c.update(rnd(), rnd(), start, cache_update_mode=mode)
            c.attend(rnd(), start)
    start = BLOCKS * F * FSEQ
    c.update(rnd(), rnd(), start, cache_update_mode="noisy")
    q = rnd()
    before = int(c.ctx.token_counter.item())
    out = c.attend(q, start)
    torch.cuda.synchronize()
    mgr = c.ctx.mgr
    cu = mgr.cu_seqlens_k()[:F * H + 1].cpu().to(torch.int64)
    lens = cu[1:] - cu[:-1]
    assert int(cu[0]) == 0 and bool((lens >= 0).all())
    assert bool((lens % 390 == 0).all()), lens
    assert int(cu[-1]) == int(c.ctx.token_counter.item()) - before
    assert int(lens.min()) >= FSEQ  # every head attends at least its recent frames

    kf = mgr.k_flat_out()[:int(cu[-1])].reshape(-1, D).float()
    vf = mgr.v_flat_out()[:int(cu[-1])].reshape(-1, D).float()
    order = torch.argsort(lens)
    picks = {int(order[0]), int(order[-1]), int(order[len(order) // 2])}
    scale = D ** -0.5
    for i in sorted(picks):
        ch, h = divmod(i, H)
        a, b = int(cu[i]), int(cu[i + 1])
        qh = q[0, ch * FSEQ:(ch + 1) * FSEQ, h].float()
        ref = torch.softmax((qh @ kf[a:b].T) * scale, dim=-1) @ vf[a:b]
        err = (out[0, ch * FSEQ:(ch + 1) * FSEQ, h].float() - ref).abs()
        assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3, (i, err.max().item())

    again = c.attend(q, start)
    assert torch.equal(again.view(torch.int16), out.view(torch.int16))
    assert c.ctx.check_status() == 0
