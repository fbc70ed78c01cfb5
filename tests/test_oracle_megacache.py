"""The oracle's MegaCache restatement against the reference's known answers.

Expectations are those the reference's own tests assert for its MegaCache
(tests/test_mega_cache_update_attend.py:45-120 and
tests/test_mega_cache_noisy_clean.py:41-120): sink fill, recent FIFO, stride
key times, noisy passes not advancing committed counters, clean commits.  A
mixed-strategy run then exercises every oracle wrapper (plan, pack with RoPE,
merge) on CPU.
"""
from __future__ import annotations

import numpy as np

from oracle import pkv_oracle as O


def _stride_cache(H=1, D=16, FSEQ=4, capacity=12, max_middle=12):
    st = O.make_states([{"kind": O.SK_STRIDE, "interval": 1, "capacity": capacity,
                         "sink_capacity": 3}] * H)
    return O.OracleMegaCache(1, H, D, FSEQ, 3, max_middle, 4, st, [[3] * H], spatial_width=2)


def _rand(rng, shape):
    return O.f32_to_bf16(rng.standard_normal(shape).astype(np.float32))


def _tkeys(c, h=0):
    raw = c.states[0].reshape(-1, 600)[h]
    i32 = raw[4:].view(np.int32)
    count = int(raw[440].view(np.int8))
    return count, [int(x) for x in raw[344:344 + 96].view(np.int32)[:count]]


def test_three_blocks_sink_recent_stride():
    c = _stride_cache()
    rng = np.random.default_rng(3)
    F, FSEQ, H, D = 3, 4, 1, 16
    blocks = [(_rand(rng, (1, F * FSEQ, H, D)), _rand(rng, (1, F * FSEQ, H, D))) for _ in range(3)]
    c.update(0, *blocks[0], 0)
    assert c.vc[0, 0, 0] == 3 and c.vc[0, 0, 2] == 0
    assert _tkeys(c) == (3, [0, 1, 2])
    c.update(0, *blocks[1], 3 * FSEQ)
    assert c.vc[0, 0, 0] == 3 and c.vc[0, 0, 2] == 3
    assert _tkeys(c) == (6, [0, 1, 2, 3, 4, 5])
    c.update(0, *blocks[2], 6 * FSEQ)
    assert c.vc[0, 0, 2] == 4
    # recent holds frames t=5,6,7,8 after evicting 3,4 (FIFO shift-left)
    np.testing.assert_array_equal(c.rec_pos[0, 0, :, 0, 0], [5, 6, 7, 8])
    k2 = blocks[1][0].reshape(F, FSEQ, H, D)
    np.testing.assert_array_equal(c.rec_k[0, 0, 0], k2[2, :, 0])   # t=5 shifted to slot 0
    out, pk = c.attend(0, _rand(rng, (1, F * FSEQ, H, D)), 6 * FSEQ)
    # 3 sink + 4 recent + 6 stride frames (keys t=3..8, t >= sink_capacity)
    assert pk["cu"][1] == (3 + 4 + 6) * FSEQ
    assert np.isfinite(out).all()


def test_noisy_passes_do_not_commit():
    c = _stride_cache(capacity=8, max_middle=8)
    rng = np.random.default_rng(7)
    F, FSEQ, H, D = 3, 4, 1, 16
    for _ in range(4):
        c.update(0, _rand(rng, (1, 12, H, D)), _rand(rng, (1, 12, H, D)), 0, "noisy")
        assert c.vc[0, 0, 0] == F and c.committed_vc[0, 0, 0] == 0
    assert _tkeys(c)[0] == 0
    ck = _rand(rng, (1, 12, H, D))
    c.update(0, ck, _rand(rng, (1, 12, H, D)), 0, "clean")
    assert c.committed_vc[0, 0, 0] == F and _tkeys(c)[0] == F
    np.testing.assert_array_equal(c.sink_k[0, 0, 0], ck.reshape(F, FSEQ, H, D)[0, :, 0])
    # block 2 noisy restores the block-1 commit
    c.update(0, _rand(rng, (1, 12, H, D)), _rand(rng, (1, 12, H, D)), 12, "noisy")
    assert c.vc[0, 0, 2] == 3 and c.committed_vc[0, 0, 2] == 0
    c.update(0, _rand(rng, (1, 12, H, D)), _rand(rng, (1, 12, H, D)), 12, "noisy")
    assert c.vc[0, 0, 2] == 3


def test_mixed_strategies_run_through_every_wrapper():
    from pyramidkv import policy
    labels = np.array([[-1, 1, 2, 1], [2, -1, -1, 1]])
    states, caps = policy.states_from_labels(labels, "baseline")
    tables, _ = O.rope_freq_tables(64)
    W, Hg, D = 6, 4, 64
    c = O.OracleMegaCache(2, 4, D, W * Hg, 3, 24, 4, states, caps, spatial_width=W,
                          sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18,
                          sink_time_clamp_max=21, freq_tables=tables)
    rng = np.random.default_rng(1)
    FSEQ = W * Hg
    for blk in range(12):
        for mode in ("noisy", "clean"):
            for layer in range(2):
                k, v, q = (_rand(rng, (1, 3 * FSEQ, 4, D)) for _ in range(3))
                c.update(layer, k, v, blk * 3 * FSEQ, mode)
                out, pk = c.attend(layer, q, blk * 3 * FSEQ)
                assert np.isfinite(out).all()
                assert pk["total"] == pk["cu"][-1] == pk["sl"][pk["sk"] >= 0].sum()
    assert c.mtc.max() > 0                       # merge anchors finalized
    assert (c.mtc[c.mtc > 0] == (W // 2) * (Hg // 2)).all()
    # merge anchors appear in the plan with the block's median time
    kinds = pk["sk"][pk["sk"] >= 0]
    assert (kinds == 3).any()
