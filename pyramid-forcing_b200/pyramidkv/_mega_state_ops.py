"""Python <-> device bridge for the per-head state and the plan ops.

Same API as the reference's pyramidkv/_mega_state_ops.py:36-411:
``PER_HEAD_STATE_DTYPE``, ``pack_states``, ``unpack_states``,
``mega_plan_cuda``, ``mega_plan_multi_cuda``, ``mega_merge_accum_cuda``,
``mega_state_update_cuda``.

``PER_HEAD_STATE_DTYPE`` spells the 600-byte record with explicit byte offsets
(the record is an ABI shared with every producer of state bytes; the layout is
pyramidkv/csrc/anchor_store.cuh:62-132), and ``_check_abi`` compares its size
with the library's ``mega_state_perhead_size``.
"""
from __future__ import annotations

from typing import Iterable, Sequence

import numpy as np
import torch

from . import _mega_state_ref as _ref
from . import _ops

_I8, _I32 = np.int8, np.int32
# (name, numpy type, shape, byte offset)
_FIELDS = [
    ("kind", _I8, (), 0),
    ("sink_capacity", _I8, (), 1),
    ("_pad0", _I8, (2,), 2),
    ("period", _I32, (), 4),
    ("bucket_cap", _I32, (), 8),
    ("interval", _I32, (), 12),
    ("capacity", _I32, (), 16),
    ("patch_size", _I32, (), 20),
    ("block_frames", _I32, (), 24),
    ("lag_offsets", _I32, (_ref.MAX_LAG_OFFSETS,), 28),
    ("lag_offset_count", _I32, (), 44),
    ("cyclic_slot", _I32, (_ref.MAX_PHASE * _ref.MAX_BUCKET,), 48),
    ("cyclic_t", _I32, (_ref.MAX_PHASE * _ref.MAX_BUCKET,), 144),
    ("cyclic_cursor", _I8, (_ref.MAX_PHASE,), 240),
    ("tkey_slot", _I32, (_ref.MAX_T_KEYED,), 248),
    ("tkey_t", _I32, (_ref.MAX_T_KEYED,), 344),
    ("tkey_count", _I8, (), 440),
    ("tkey_head", _I8, (), 441),
    ("_pad1", _I8, (2,), 442),
    ("merge_completed_slot", _I32, (_ref.MAX_MERGE_BLOCKS,), 444),
    ("merge_completed_block_id", _I32, (_ref.MAX_MERGE_BLOCKS,), 468),
    ("merge_completed_start_t", _I32, (_ref.MAX_MERGE_BLOCKS,), 492),
    ("merge_completed_end_t", _I32, (_ref.MAX_MERGE_BLOCKS,), 516),
    ("merge_completed_median_t", _I32, (_ref.MAX_MERGE_BLOCKS,), 540),
    ("merge_completed_count", _I8, (), 564),
    ("_pad2", _I8, (3,), 565),
    ("merge_active_block_id", _I32, (_ref.MAX_MERGE_ACTIVE,), 568),
    ("merge_active_slot", _I32, (_ref.MAX_MERGE_ACTIVE,), 576),
    ("merge_active_seen", _I8, (_ref.MAX_MERGE_ACTIVE, _ref.MAX_MERGE_BLOCK_FRAMES), 584),
    ("merge_active_complete_count", _I8, (_ref.MAX_MERGE_ACTIVE,), 592),
    ("_pad3", _I8, (2,), 594),
    ("cached_num_groups", _I32, (), 596),
]
PER_HEAD_STATE_DTYPE = np.dtype({
    "names": [f[0] for f in _FIELDS],
    "formats": [(f[1], f[2]) if f[2] else f[1] for f in _FIELDS],
    "offsets": [f[3] for f in _FIELDS],
    "itemsize": 600,
})

_SCALARS = ("kind", "sink_capacity", "period", "bucket_cap", "interval", "capacity",
            "patch_size", "block_frames", "lag_offset_count", "tkey_count", "tkey_head",
            "merge_completed_count", "cached_num_groups")
_ARRAYS = ("lag_offsets", "cyclic_slot", "cyclic_t", "cyclic_cursor", "tkey_slot", "tkey_t",
           "merge_completed_slot", "merge_completed_block_id", "merge_completed_start_t",
           "merge_completed_end_t", "merge_completed_median_t", "merge_active_block_id",
           "merge_active_slot", "merge_active_complete_count")

_ABI_CHECKED = False


def _check_abi() -> None:
    global _ABI_CHECKED
    if _ABI_CHECKED:
        return
    lib_size = int(_ops.ops().mega_state_perhead_size())
    if lib_size != PER_HEAD_STATE_DTYPE.itemsize:
        raise RuntimeError(
            f"PerHeadState ABI mismatch: numpy dtype itemsize={PER_HEAD_STATE_DTYPE.itemsize}, "
            f"sizeof(PerHeadState)={lib_size}.")
    _ABI_CHECKED = True


def pack_states(states: Sequence[_ref.PerHeadState]) -> np.ndarray:
    arr = np.zeros(len(states), dtype=PER_HEAD_STATE_DTYPE)
    for i, s in enumerate(states):
        rec = arr[i]
        for name in _SCALARS:
            rec[name] = getattr(s, name)
        for name in _ARRAYS:
            rec[name][:] = getattr(s, name, rec[name])
        rec["merge_active_seen"][:] = [[int(bool(b)) for b in row] for row in s.merge_active_seen]
    return arr


def unpack_states(arr: np.ndarray) -> list[_ref.PerHeadState]:
    out = []
    for i in range(arr.shape[0]):
        rec = arr[i]
        kw = {name: int(rec[name]) for name in _SCALARS}
        for name in _ARRAYS:
            kw[name] = [int(x) for x in rec[name]]
        kw["merge_active_seen"] = [[bool(b) for b in row] for row in rec["merge_active_seen"]]
        out.append(_ref.PerHeadState(**kw))
    return out


def _to_bytes_tensor(arr: np.ndarray, device) -> torch.Tensor:
    flat = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
    return torch.from_numpy(flat).clone().to(device=device, non_blocking=False)


_SINK_MODE = {"lag": 0, "window_clamp": 1}
_HIST_MODE = {"none": 0, "relative_clamp": 1, "relative_softcap": 2}


def mega_plan_cuda(mgr, states_bytes, layer_idx: int, current_t: int, pass_kind: int = 1,
                   sink_time_mapping_mode: str = "lag", sink_time_clamp_min: int = 0,
                   sink_time_clamp_max: int = 21, decoupled_sink_time_lag: int = 0,
                   history_time_mapping_mode: str = "none", history_relative_t_max: int = 21,
                   history_time_soft_factor: float = 1.0):
    """One-chunk plan: (cu_seqlens_k, src_kind, src_slot_global, seg_lengths,
    dst_token_offsets, anchor_t_raw, anchor_t_remap), all device tensors."""
    return _ops.ops().mega_plan(
        mgr, states_bytes, int(layer_idx), int(current_t), int(pass_kind),
        int(_SINK_MODE.get(sink_time_mapping_mode, 0)), int(sink_time_clamp_min),
        int(sink_time_clamp_max), int(decoupled_sink_time_lag),
        int(_HIST_MODE.get(history_time_mapping_mode, 0)), int(history_relative_t_max),
        float(history_time_soft_factor))


def mega_plan_multi_cuda(mgr, states_bytes, layer_idx: int, current_t_list, pass_kind: int = 1,
                         sink_time_mapping_mode: str = "lag", sink_time_clamp_min: int = 0,
                         sink_time_clamp_max: int = 21, decoupled_sink_time_lag: int = 0,
                         history_time_mapping_mode: str = "none",
                         history_relative_t_max: int = 21,
                         history_time_soft_factor: float = 1.0):
    """Multi-chunk plan with chunk-offset dst_token_offsets (7 device tensors)."""
    if not isinstance(current_t_list, torch.Tensor):
        current_t_list = torch.tensor(list(current_t_list), dtype=torch.int64)
    elif current_t_list.dtype != torch.int64:
        current_t_list = current_t_list.to(torch.int64)
    if current_t_list.dim() == 0:
        current_t_list = current_t_list.view(1)
    if current_t_list.device.type != "cpu":
        current_t_list = current_t_list.cpu()
    return _ops.ops().mega_plan_multi(
        mgr, states_bytes, int(layer_idx), current_t_list, int(pass_kind),
        int(_SINK_MODE.get(sink_time_mapping_mode, 0)), int(sink_time_clamp_min),
        int(sink_time_clamp_max), int(decoupled_sink_time_lag),
        int(_HIST_MODE.get(history_time_mapping_mode, 0)), int(history_relative_t_max),
        float(history_time_soft_factor))


def mega_merge_accum_cuda(mgr, layer_idx: int, states_bytes, new_k, new_v, new_pos,
                          descriptors) -> None:
    """Merge accumulation + finalize for one layer's slices of the manager pools."""
    desc_kind, desc_slot, desc_finalize, desc_new = descriptors
    _ops.ops().mega_merge_accum(
        states_bytes, new_k, new_v, new_pos, desc_kind, desc_slot, desc_finalize, desc_new,
        mgr.merge_accum_sum_k()[layer_idx], mgr.merge_accum_sum_v()[layer_idx],
        mgr.merge_accum_pos()[layer_idx], mgr.merge_accum_group_ids()[layer_idx],
        mgr.merge_accum_tokens_per_group()[layer_idx], mgr.merge_accum_num_groups()[layer_idx],
        mgr.merge_k_pool()[layer_idx], mgr.merge_v_pool()[layer_idx],
        mgr.merge_pos_pool()[layer_idx], mgr.merge_token_count()[layer_idx])


def mega_state_update_cuda(states: Sequence[_ref.PerHeadState], new_t_vals: Iterable[int],
                           pass_kind: int, device="cuda"):
    """pack -> device state machine -> unpack.

    Returns (8 descriptor lists..., mutated_states) like the reference.
    """
    _check_abi()
    dev = torch.device(device)
    H = len(states)
    t = list(new_t_vals)
    N = H * len(t)
    buf = _to_bytes_tensor(pack_states(states), dev)
    tt = torch.tensor(t, dtype=torch.int64, device=dev)
    descs = [torch.full((N,), -1, dtype=torch.int32, device=dev) for _ in range(8)]
    _ops.ops().mega_state_update(buf, tt, *descs, int(H), int(len(t)), int(pass_kind))
    back = buf.cpu().numpy().view(PER_HEAD_STATE_DTYPE).reshape(H).copy()
    return tuple(d.cpu().tolist() for d in descs) + (unpack_states(back),)
