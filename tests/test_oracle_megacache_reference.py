"""The oracle's MegaCache restatement against the reference's own MegaCache.update.

``tests/golden/megacache_c1.npz`` holds digests of every pool, the valid
counts, the state bytes and the committed snapshot after each update call of
the reference's ``pyramidkv/_mega_cache.py`` (``MegaCache.update`` :136-414,
run on CPU by ``tests/golden/make_megacache_golden.py``) at the benchmark's
layer shape: 12 heads x 128, 1560-token frames, 20 blocks of a noisy and a
clean update, for a uniform label row and a merge-heavy one.  Here
``oracle.pkv_oracle.OracleMegaCache`` runs the same calls; its state must
match after every clean pass, and its plan + pack of the final state must
match the recorded cu_seqlens_k and packed-segment digests.
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
from oracle import pkv_oracle as O  # noqa: E402


class _OracleManager(G.StandInManager):
    pass


@pytest.mark.parametrize("name", list(G.CONFIGS))
def test_oracle_megacache_matches_reference_update(name):
    gold = np.load(os.path.join(GOLDEN, "megacache_c1.npz"))
    cfg = G.CONFIGS[name]
    labels = gold[f"{name}_labels"]
    from pyramidkv import policy
    states, caps = policy.states_from_labels(labels, "baseline")
    assert np.array_equal(states, gold[f"{name}_states0"])
    assert np.array_equal(caps, gold[f"{name}_sink_caps"])
    tables, _ = O.rope_freq_tables(G.D)
    orc = O.OracleMegaCache(G.L, G.H, G.D, G.FSEQ, G.SINK, G.MIDDLE, G.RECENT, states, caps,
                            spatial_width=G.W, sink_time_mapping_mode="window_clamp",
                            sink_time_clamp_min=18, sink_time_clamp_max=21, freq_tables=tables)
    mgr = _OracleManager(orc)
    kv, _ = G.inputs(cfg["seed"])
    i = 0
    for blk in range(G.BLOCKS):
        for p, mode in enumerate(G.PASSES):
            k, v = kv[blk][p]
            orc.update(0, k, v, blk * G.F * G.FSEQ, mode)
            if mode == "clean":
                committed = {
                    "committed_vc": torch.from_numpy(orc.committed_vc),
                    "committed_recent_k": torch.from_numpy(orc.committed_rec_k.view(np.int16)),
                    "committed_recent_v": torch.from_numpy(orc.committed_rec_v.view(np.int16)),
                    "committed_recent_pos": torch.from_numpy(orc.committed_rec_pos)}
                got = MD.state_digests(mgr, torch.from_numpy(orc.states), committed)
                for key, val in got.items():
                    want = gold[f"{name}_{key}"][i]
                    assert np.array_equal(val, want), (name, blk, mode, key,
                                                       np.nonzero(val != want)[0][:8])
            i += 1
    pk = orc.plan_and_pack(0, G.BLOCKS * G.F * G.FSEQ, G.F)
    assert np.array_equal(pk["cu"].astype(np.int32), gold[f"{name}_plan_cu"])
    bf = lambda a: torch.from_numpy(a.view(np.int16))  # noqa: E731
    cu = pk["cu"]
    for s_, (a_, b_) in enumerate(zip(cu[:-1], cu[1:])):
        got = [MD.blob_digest(bf(pk["k"][a_:b_].copy())), MD.blob_digest(bf(pk["v"][a_:b_].copy())),
               MD.blob_digest(torch.from_numpy(pk["pos"][a_:b_].copy()))]
        assert got == gold[f"{name}_plan_seg_digests"][s_].tolist(), (name, s_)
