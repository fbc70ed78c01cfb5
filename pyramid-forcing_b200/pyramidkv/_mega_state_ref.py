"""Host-side mirror of the per-(layer, head) strategy record ``PerHeadState``.

Same names, constants and constructor defaults as the reference's
pyramidkv/_mega_state_ref.py:23-113 (the dataclass and the ``make_*``
builders callers use to describe a head), so compositions built against the
reference build identical state bytes here.  The record additionally carries
the merge bookkeeping fields of the C++ struct (``merge_completed_start_t``,
``_end_t``, ``_median_t``, ``merge_active_slot``) that the reference's mirror
omits; their defaults pack to the same zero bytes.

The state machine itself runs only on the GPU (``mega_state_update``).
"""
from __future__ import annotations

from dataclasses import dataclass, field

SK_RECENT = 0
SK_CYCLIC = 1
SK_STRIDE = 2
SK_LAG = 3
SK_MERGE = 4

MAX_PHASE = 6
MAX_BUCKET = 4
MAX_T_KEYED = 24
MAX_LAG_OFFSETS = 4
MAX_MERGE_BLOCKS = 6
MAX_MERGE_ACTIVE = 2
MAX_MERGE_BLOCK_FRAMES = 4
MAX_MERGE_TOKENS = 420

DST_KIND_SINK = 0
DST_KIND_MIDDLE = 1
DST_KIND_RECENT = 2
DST_KIND_SKIP = -1
DST_KIND_MERGE_ACCUM = 5


class MergeDuplicateError(ValueError):
    """A merge block saw the same local frame twice (the device skips it)."""


def _filled(n: int, v: int):
    return field(default_factory=lambda: [v] * n)


@dataclass
class PerHeadState:
    kind: int = SK_RECENT
    sink_capacity: int = 0
    period: int = 0
    bucket_cap: int = 0
    interval: int = 0
    capacity: int = 0
    patch_size: int = 0
    block_frames: int = 0
    lag_offsets: list[int] = _filled(MAX_LAG_OFFSETS, 0)
    lag_offset_count: int = 0
    cyclic_slot: list[int] = _filled(MAX_PHASE * MAX_BUCKET, -1)
    cyclic_t: list[int] = _filled(MAX_PHASE * MAX_BUCKET, 0)
    cyclic_cursor: list[int] = _filled(MAX_PHASE, 0)
    tkey_slot: list[int] = _filled(MAX_T_KEYED, -1)
    tkey_t: list[int] = _filled(MAX_T_KEYED, 0)
    tkey_count: int = 0
    tkey_head: int = 0
    merge_completed_slot: list[int] = _filled(MAX_MERGE_BLOCKS, -1)
    merge_completed_block_id: list[int] = _filled(MAX_MERGE_BLOCKS, -1)
    merge_completed_count: int = 0
    merge_active_block_id: list[int] = _filled(MAX_MERGE_ACTIVE, -1)
    merge_active_seen: list[list[bool]] = field(
        default_factory=lambda: [[False] * MAX_MERGE_BLOCK_FRAMES
                                 for _ in range(MAX_MERGE_ACTIVE)])
    merge_active_complete_count: list[int] = _filled(MAX_MERGE_ACTIVE, 0)
    cached_num_groups: int = 0
    # fields of the C++ record the reference mirror does not carry
    merge_completed_start_t: list[int] = _filled(MAX_MERGE_BLOCKS, 0)
    merge_completed_end_t: list[int] = _filled(MAX_MERGE_BLOCKS, 0)
    merge_completed_median_t: list[int] = _filled(MAX_MERGE_BLOCKS, 0)
    merge_active_slot: list[int] = _filled(MAX_MERGE_ACTIVE, 0)


def make_cyclic(period: int, bucket_cap: int) -> PerHeadState:
    return PerHeadState(kind=SK_CYCLIC, period=period, bucket_cap=bucket_cap)


def make_stride(interval: int, capacity: int) -> PerHeadState:
    return PerHeadState(kind=SK_STRIDE, interval=interval, capacity=capacity)


def make_lag(history_frames: int, offsets: list[int] | None = None) -> PerHeadState:
    s = PerHeadState(kind=SK_LAG, capacity=history_frames)
    if offsets:
        used = list(offsets)[:MAX_LAG_OFFSETS]
        s.lag_offsets[:len(used)] = used
        s.lag_offset_count = len(used)
    return s


def make_recent() -> PerHeadState:
    return PerHeadState(kind=SK_RECENT)


def make_merge(patch_size: int = 2, capacity: int = 6) -> PerHeadState:
    return PerHeadState(kind=SK_MERGE, patch_size=patch_size, capacity=capacity,
                        block_frames=patch_size * patch_size)
