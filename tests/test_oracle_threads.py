"""The oracle's pack gives the same bytes on one thread and on several.

The timed CPU baseline runs the C pack over all host cores (segments handed
out from a shared counter, each writing its own output range); the tests use
one thread.  A steady-state cache with merge heads and the RoPE remap is
packed both ways and compared bit for bit.
"""
from __future__ import annotations

import numpy as np

from oracle import pkv_oracle as O


def test_threaded_pack_is_bit_identical():
    from pyramidkv import policy
    H, D, W, HG, F = 6, 32, 13, 8, 3
    FSEQ = W * HG
    labels = np.array([[-1, 1, 2, -1, 2, 1]])
    states, caps = policy.states_from_labels(labels, "baseline")
    tables, _ = O.rope_freq_tables(D)
    orc = O.OracleMegaCache(1, H, D, FSEQ, 3, 24, 4, states, caps, spatial_width=W,
                            sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18,
                            sink_time_clamp_max=21, freq_tables=tables)
    rng = np.random.default_rng(3)
    for blk in range(10):
        k, v = (O.f32_to_bf16(rng.standard_normal((1, F * FSEQ, H, D)).astype(np.float32))
                for _ in range(2))
        orc.update(0, k, v, blk * F * FSEQ, "clean")
    start = 10 * F * FSEQ
    try:
        O.set_threads(1)
        one = orc.plan_and_pack(0, start, F)
        O.set_threads(7)
        many = orc.plan_and_pack(0, start, F)
    finally:
        O.set_threads(1)
    assert one["total"] == many["total"] > 0
    for key in ("k", "v", "pos", "cu"):
        np.testing.assert_array_equal(one[key], many[key], err_msg=key)
