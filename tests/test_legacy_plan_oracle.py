"""The legacy all-layer plan (op pyramidkv_plan, M1.4) restated in the
oracle, against the known answers of the reference's own tests
(tests/test_pyramidkv_plan.py:35-137): per-head totals of (ms + mm + mr) * F
with every slot valid, kinds ordered sink / recent / middle, inactive kinds
-1, offsets head-major over all layers."""
from __future__ import annotations

import numpy as np

from oracle import pkv_oracle as O


def test_all_kinds_full():
    L, H, F, ms, mm, mr = 2, 4, 8, 2, 4, 2
    vc = np.zeros((L, H, 3), np.int64)
    vc[..., 0], vc[..., 1], vc[..., 2] = ms, mm, mr
    cu, sk, sg, sl, dst = O.legacy_plan(vc, F, ms, mm, mr)
    n = L * H
    assert cu.shape == (n + 1,) and sk.shape == (n * 3,) and cu.dtype == np.int32
    assert (np.diff(cu) == (ms + mm + mr) * F).all()
    assert (sk.reshape(n, 3) == [0, 2, 1]).all()
    assert (sl.reshape(n, 3) == [ms * F, mr * F, mm * F]).all()
    # slot 0 of each (layer, head) in each pool
    assert (sg.reshape(n, 3) == np.arange(n)[:, None] * [ms, mr, mm]).all()
    # segments tile the packed rows in order
    assert (dst == np.concatenate([[0], np.cumsum(sl)[:-1]])).all()


def test_inactive_kinds():
    L, H, F, ms, mm, mr = 1, 2, 4, 2, 2, 2
    vc = np.zeros((L, H, 3), np.int64)
    vc[..., 1] = mm
    cu, sk, sg, sl, dst = O.legacy_plan(vc, F, ms, mm, mr)
    assert (sk.reshape(-1, 3) == [-1, -1, 1]).all()
    assert (np.diff(cu) == mm * F).all()
    inactive = sk == -1
    assert (sg[inactive] == 0).all() and (sl[inactive] == 0).all() and (dst[inactive] == 0).all()
