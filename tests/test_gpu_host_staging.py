"""Layer-steps fed from pinned host memory through ``HostStaging``.

Two identical cache sets run the same blocks: one with device-resident Q/K/V,
the other with host Q/K/V staged by ``pyramidkv.host_staging.HostStaging``
(copy-in of layer-step i+1 while layer-step i runs, copy-out of every output).
The host outputs must equal the device outputs bit for bit, and the helper
must refuse calls out of order.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import pkv_oracle as O

pytestmark = pytest.mark.gpu

L, H, D, W, HG, F = 2, 4, 128, 13, 8, 3
FSEQ = W * HG


def _caches():
    from pyramidkv import _mega_cache, policy
    _, full = O.rope_freq_tables(D)
    labels = np.array([[-1, 1, 2, 2], [2, 1, -1, 1]])
    return _mega_cache.build_mega_caches(
        L, H, D, FSEQ, 3, 24, 4, policy.compositions_from_labels(labels), device="cuda:0",
        sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18, sink_time_clamp_max=21,
        spatial_width=W, spatial_height=HG, freqs=full)


def test_staged_layer_steps_match_device_inputs(cuda):
    from pyramidkv.host_staging import HostStaging
    g = torch.Generator(device="cpu").manual_seed(17)
    rnd = lambda: torch.randn(1, F * FSEQ, H, D, generator=g).to(torch.bfloat16)  # noqa: E731
    steps = []
    for blk in range(4):
        for mode in ("noisy", "clean"):
            for layer in range(L):
                steps.append((blk * F * FSEQ, mode, layer, (rnd(), rnd(), rnd())))

    ref = _caches()
    want = []
    for start, mode, layer, (q, k, v) in steps:
        ref[layer].update(k.to(cuda), v.to(cuda), start, cache_update_mode=mode)
        want.append(ref[layer].attend(q.to(cuda), start).cpu())

    caches = _caches()
    host = [tuple(x.pin_memory() for x in s[3]) for s in steps]
    outs = [torch.empty(1, F * FSEQ, H, D, dtype=torch.bfloat16).pin_memory() for _ in steps]
    stage = HostStaging(host[0], cuda, depth=2)
    stage.put(host[0])
    fins = []
    for i, (start, mode, layer, _) in enumerate(steps):
        if i + 1 < len(steps):
            stage.put(host[i + 1])
        q, k, v = stage.get()
        caches[layer].update(k, v, start, cache_update_mode=mode)
        fins.append(stage.done(caches[layer].attend(q, start), outs[i]))
    for f in fins:
        f.synchronize()
    for i, w in enumerate(want):
        assert torch.equal(outs[i].view(torch.int16), w.view(torch.int16)), i
    assert caches[0].ctx.check_status() == 0


def test_staging_refuses_out_of_order_calls(cuda):
    from pyramidkv.host_staging import HostStaging
    x = torch.zeros(4, 8, dtype=torch.bfloat16).pin_memory()
    stage = HostStaging([x], cuda, depth=2)
    with pytest.raises(RuntimeError):
        stage.get()
    stage.put([x])
    stage.put([x])
    with pytest.raises(RuntimeError):
        stage.put([x])                     # both slots wait for done()
    (d,) = stage.get()
    with pytest.raises(RuntimeError):
        stage.get()                        # the previous get() is not done
    stage.done(d * 2, torch.empty(4, 8, dtype=torch.bfloat16).pin_memory()).synchronize()
    with pytest.raises(RuntimeError):
        stage.done(d, x)
    stage.synchronize()
