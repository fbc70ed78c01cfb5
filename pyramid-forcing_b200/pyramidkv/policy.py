"""Per-head label matrix -> PerHeadState records for the MegaCache path.

The reference builds these through ``pyramidkv/factory.py:build_compositions``
(:220-407) and ``_mega_cache._composition_to_perhead_state`` (:572-628) from a
labels CSV and the yaml maps.  This module produces the same records directly
from a label matrix for the two routings the benchmark configurations use:

* ``"yaml"``      -- configs/pyramid-forcing.yaml:112-131: label -1 -> cyclic
  (period 6, 4 buckets, 1 sink frame), 1 -> stride (interval 6, capacity 4,
  3 sink frames), 2 -> merge (patch 2, capacity 4, 3 sink frames);
* ``"baseline"``  -- stride for label 1, periodic (cyclic) for 2, merge for -1,
  with the yaml's parameters and per-label sink frames.

The output equals the reference factory's for the same labels (pinned by a
golden fixture).
"""
from __future__ import annotations

import numpy as np

from . import _mega_state_ops
from . import _mega_state_ref as ref

ROUTINGS = {
    "yaml": {-1: "cyclic", 1: "stride", 2: "merge"},
    "baseline": {1: "stride", 2: "cyclic", -1: "merge"},
}
SINK_FRAMES = {-1: 1, 1: 3, 2: 3}


def head_state(label: int, routing: str = "baseline", *, period: int = 6, bucket_cap: int = 4,
               stride_interval: int = 6, stride_capacity: int = 4, merge_patch: int = 2,
               merge_capacity: int = 4, sink_frames: dict | None = None) -> ref.PerHeadState:
    kind = ROUTINGS[routing][int(label)]
    if kind == "cyclic":
        s = ref.make_cyclic(period=period, bucket_cap=bucket_cap)
    elif kind == "stride":
        cap = stride_capacity if 0 < stride_capacity <= ref.MAX_T_KEYED else ref.MAX_T_KEYED
        s = ref.make_stride(interval=stride_interval, capacity=cap)
    else:
        s = ref.make_merge(patch_size=merge_patch, capacity=merge_capacity)
    s.sink_capacity = int((sink_frames or SINK_FRAMES)[int(label)])
    return s


def states_from_labels(labels, routing: str = "baseline", **kw):
    """labels [L, H] -> (uint8 [L, H*600] state bytes, int64 [L, H] sink caps)."""
    labels = np.asarray(labels)
    L, H = labels.shape
    out = np.zeros((L, H * _mega_state_ops.PER_HEAD_STATE_DTYPE.itemsize), np.uint8)
    caps = np.zeros((L, H), np.int64)
    for l in range(L):
        states = [head_state(int(x), routing, **kw) for x in labels[l]]
        out[l] = _mega_state_ops.pack_states(states).view(np.uint8).reshape(-1)
        caps[l] = [s.sink_capacity for s in states]
    return out, caps


def random_labels(L: int, H: int, seed: int = 0, merge_fraction: float | None = None):
    """Seeded label matrix over {-1, 1, 2}: uniform, or with an exact share of
    merge (-1) heads and the rest split evenly between 1 and 2."""
    rng = np.random.default_rng(seed)
    if merge_fraction is None:
        return rng.choice(np.asarray([-1, 1, 2]), size=(L, H))
    n = L * H
    n_merge = int(round(n * merge_fraction))
    rest = n - n_merge
    flat = np.array([-1] * n_merge + [1] * (rest // 2) + [2] * (rest - rest // 2))
    rng.shuffle(flat)
    return flat.reshape(L, H)


class _Strategy:
    """Attribute holder standing in for a reference middle-strategy object;
    ``_composition_to_perhead_state`` dispatches on the class name."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


class CyclicStrategy(_Strategy):
    pass


class StrideStrategy(_Strategy):
    pass


class MergeStrategy(_Strategy):
    pass


class LabelComposition:
    """Minimal HeadComposition (sink_frames + middle_strategies) for one head."""

    def __init__(self, label: int, routing: str = "baseline", **kw):
        st = head_state(label, routing, **kw)
        self.label = int(label)
        self.sink_frames = st.sink_capacity
        if st.kind == ref.SK_CYCLIC:
            self.middle_strategies = [CyclicStrategy(period=st.period, bucket_cap=st.bucket_cap)]
        elif st.kind == ref.SK_STRIDE:
            self.middle_strategies = [StrideStrategy(interval=st.interval, capacity=st.capacity)]
        else:
            self.middle_strategies = [MergeStrategy(patch_size=st.patch_size,
                                                    capacity=st.capacity)]


def compositions_from_labels(labels, routing: str = "baseline", **kw):
    """[L][H] compositions for ``_mega_cache.build_mega_caches``."""
    return [[LabelComposition(int(x), routing, **kw) for x in row] for row in np.asarray(labels)]
