"""Oracle restatement of the AdaptiveKVCache / CppStrategyManager ops.

Known answers of the history time mapping of ``refresh_readout_layout``
(pyramidkv/csrc/scatter_copy.cu:138-163), worked out by hand from its
definition: relative_clamp (mode 1) caps current_t - t at rel_max;
relative_softcap (mode 2) keeps rel_max and scales the excess by the soft
factor, rounding the float32 product to nearest even (llrintf); the mapped
time is never negative; rel_max <= 0 leaves t unchanged.
"""
from __future__ import annotations

import numpy as np

from oracle import pkv_oracle as O


def test_history_time_mapping_known_answers():
    m = O.legacy_map_t
    assert m(5, 30, 1, 21, 1.0) == 9          # rel 25 -> 21
    assert m(20, 30, 1, 21, 1.0) == 20        # inside the window
    assert m(35, 30, 1, 21, 1.0) == 30        # future time: rel clamps to 0
    assert m(5, 30, 2, 21, 0.5) == 7          # over 4 * 0.5 = 2 -> rel 23
    assert m(4, 30, 2, 21, 0.5) == 7          # over 5 * 0.5 = 2.5 -> 2 (even): rel 23
    assert m(2, 30, 2, 21, 0.5) == 5          # over 7 * 0.5 = 3.5 -> 4 (even): rel 25
    assert m(0, 10, 1, 21, 1.0) == 0
    assert m(-3, 10, 0, 21, 1.0) == 0         # mode none still clamps at 0
    assert m(-3, 10, 1, 0, 1.0) == -3         # rel_max <= 0: untouched


def test_refresh_layout_flags():
    rng = np.random.default_rng(0)
    D, n0, n1 = 8, 5, 3
    sk = [rng.integers(0, 2 ** 16, (n, D), dtype=np.uint16) for n in (n0, n1)]
    sv = [rng.integers(0, 2 ** 16, (n, D), dtype=np.uint16) for n in (n0, n1)]
    sp = [np.stack([np.arange(n) * 3, np.arange(n) + 100, np.arange(n) + 200], 1).astype(np.int64)
          for n in (n0, n1)]
    dk = np.zeros((10, D), np.uint16); dv = np.zeros_like(dk)
    dp = np.full((10, 3), -7, np.int64); df = np.full(10, -7, np.int64)
    O.legacy_refresh(sk, sv, sp, [0, 6], [n0, n1], [1 | 2, 4], [0, 42], dk, dv, dp, df,
                     current_t=12, mode=1, rel_max=4, soft=1.0)
    assert (dk[:n0] == sk[0]).all() and (dv[6:9] == sv[1]).all()
    assert dp[:n0, 0].tolist() == [8, 8, 8, 9, 12]      # t = 0, 3, 6, 9, 12 clamped to 12 - 4
    assert df[:n0].tolist() == [0, 3, 6, 9, 12]         # physical frame ids (bit 1)
    assert dp[6:9, 0].tolist() == [42, 42, 42] and df[6:9].tolist() == [42, 42, 42]
    assert dp[5].tolist() == [-7, -7, -7]               # untouched row
