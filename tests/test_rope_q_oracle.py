"""The oracle's query RoPE against golden vectors of the reference's own
``causal_rope_apply`` (tests/golden/make_rope_q_golden.py), bit for bit."""
from __future__ import annotations

import os

import numpy as np

from conftest import GOLDEN
from oracle import pkv_oracle as O


def test_oracle_rope_q_matches_reference_golden():
    g = np.load(os.path.join(GOLDEN, "rope_q.npz"))
    _, full = O.rope_freq_tables(128)
    for i in range(int(g["n_cases"])):
        F, Hg, Wg, start, heads, pad = (int(v) for v in g[f"c{i}_dims"])
        got = O.rope_q(g[f"c{i}_x"][0], full, start, F, Hg, Wg)
        np.testing.assert_array_equal(got, g[f"c{i}_y"][0], err_msg=f"case {i}")
