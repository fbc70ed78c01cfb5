"""The device MegaCache against the reference's own MegaCache.update, at full size.

``tests/golden/megacache_c1.npz`` records digests of every pool, the valid
counts, the per-head state bytes and the committed snapshot after each
update call of the reference's ``pyramidkv/_mega_cache.py``
(``MegaCache.update`` :136-414, driven by
``tests/golden/make_megacache_golden.py``) at the benchmark's layer shape:
12 heads x 128, 1560-token frames (30 x 52), pools 3 / 24 / 4 frames, 20
blocks of a noisy and a clean update, for a uniform label row (``c1``) and a
merge-heavy one (``merge``: six merge heads, whose merge FIFO evicts -- quirks
Q2/Q3).  Here the device path (``MegaCache.update`` -> ``pkv_cache_update``)
runs the same calls on the same seeded inputs and must match every digest
after every call (bit-exact); then ``attend`` on the final state must
reproduce the recorded ``cu_seqlens_k`` and the digests of every packed K, V
and position segment (bit-exact), and its output must match a torch fp32
softmax over the packed K/V for all 36 (chunk, head) segments within the
attention tolerance (max abs 2e-2, mean abs 2e-3).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN

sys.path.insert(0, GOLDEN)
import make_megacache_golden as G   # noqa: E402
import megacache_digest as MD       # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", list(G.CONFIGS))
def test_device_megacache_matches_reference_update(cuda, name):
    from oracle import pkv_oracle as O
    from pyramidkv import _mega_cache, policy
    gold = np.load(os.path.join(GOLDEN, "megacache_c1.npz"))
    cfg = G.CONFIGS[name]
    labels = gold[f"{name}_labels"]
    _, full = O.rope_freq_tables(G.D)
    caches = _mega_cache.build_mega_caches(
        G.L, G.H, G.D, G.FSEQ, G.SINK, G.MIDDLE, G.RECENT,
        policy.compositions_from_labels(labels, "baseline"), device="cuda:0",
        sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18, sink_time_clamp_max=21,
        spatial_width=G.W, spatial_height=G.HG, freqs=full)
    cache, ctx = caches[0], caches[0].ctx
    assert np.array_equal(ctx.states_bytes.cpu().numpy(), gold[f"{name}_states0"])
    kv, q = G.inputs(cfg["seed"])
    dev = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(cuda)  # noqa
    i = 0
    for blk in range(G.BLOCKS):
        for p, mode in enumerate(G.PASSES):
            k, v = kv[blk][p]
            cache.update(dev(k), dev(v), blk * G.F * G.FSEQ, cache_update_mode=mode)
            committed = {"committed_vc": ctx.committed_vc,
                         "committed_recent_k": ctx.committed_recent_k,
                         "committed_recent_v": ctx.committed_recent_v,
                         "committed_recent_pos": ctx.committed_recent_pos}
            got = MD.state_digests(ctx.mgr, ctx.states_bytes, committed)
            for key, val in got.items():
                want = gold[f"{name}_{key}"][i]
                assert np.array_equal(val, want), (name, blk, mode, key,
                                                   np.nonzero(val != want)[0][:8])
            i += 1
    assert ctx.check_status() == 0
    # attend on the final state: plan + RoPE pack bit-exact, attention within tolerance
    start = G.BLOCKS * G.F * G.FSEQ
    qd = dev(q)
    out = cache.attend(qd, start)
    torch.cuda.synchronize()
    mgr = ctx.mgr
    cu = mgr.cu_seqlens_k()[:G.F * G.H + 1].cpu().numpy()
    assert np.array_equal(cu, gold[f"{name}_plan_cu"])
    kf, vf, pf = mgr.k_flat_out(), mgr.v_flat_out(), mgr.pos_flat_out()
    for s_, (a_, b_) in enumerate(zip(cu[:-1], cu[1:])):
        got = [MD.blob_digest(kf[a_:b_]), MD.blob_digest(vf[a_:b_]), MD.blob_digest(pf[a_:b_])]
        assert got == gold[f"{name}_plan_seg_digests"][s_].tolist(), (name, s_)
    scale = G.D ** -0.5
    worst_max, tot_err, n = 0.0, 0.0, 0
    for s_, (a_, b_) in enumerate(zip(cu[:-1], cu[1:])):
        c, h = divmod(s_, G.H)
        qs = qd[0, c * G.FSEQ:(c + 1) * G.FSEQ, h].float()
        kk = kf[a_:b_].reshape(-1, G.D).float()
        vv = vf[a_:b_].reshape(-1, G.D).float()
        ref = torch.softmax((qs @ kk.T) * scale, dim=-1) @ vv
        err = (out[0, c * G.FSEQ:(c + 1) * G.FSEQ, h].float() - ref).abs()
        worst_max = max(worst_max, err.max().item())
        tot_err += err.sum().item()
        n += err.numel()
    assert worst_max <= 2e-2 and tot_err / n <= 2e-3, (worst_max, tot_err / n)
    assert ctx.check_status() == 0
