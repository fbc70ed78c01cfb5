"""``torch.ops.adahead`` access, same API as the reference's pyramidkv/_ops.py.

``ops()`` returns the namespace after loading the prebuilt library and raises
when it is unavailable; the wrappers forward to the registered ops (whose
schemas carry the reference's mutable-argument annotations and Meta kernels).
"""
from __future__ import annotations

import torch

from . import _scatter_ext


def _ensure_loaded() -> bool:
    return _scatter_ext._try_load()


def available() -> bool:
    if not _ensure_loaded():
        return False
    return hasattr(torch.ops, "adahead") and hasattr(torch.ops.adahead, "scatter_copy")


def ops():
    if not _ensure_loaded():
        raise RuntimeError("CUDA scatter extension not available")
    return torch.ops.adahead


def scatter_copy(src_ptrs, lengths, offsets, dst, col_dim: int) -> None:
    ops().scatter_copy(src_ptrs, lengths, offsets, dst, int(col_dim))


_EMPTY: dict = {}


def _empty(device: torch.device, dtype: torch.dtype) -> torch.Tensor:
    key = (str(device), dtype)
    t = _EMPTY.get(key)
    if t is None:
        t = torch.empty(0, dtype=dtype, device=device)
        _EMPTY[key] = t
    return t


def pyramidkv_pack(mgr, src_kind, src_slot_global, seg_lengths, dst_token_offsets, *,
                   anchor_t_remap=None, freqs_ft_flat=None, freqs_fy_flat=None,
                   freqs_fx_flat=None) -> None:
    """Pack with optional fused RoPE; omitted tensors become zero-sized."""
    dev = src_kind.device
    ops().pyramidkv_pack(
        mgr, src_kind, src_slot_global, seg_lengths, dst_token_offsets,
        anchor_t_remap if anchor_t_remap is not None else _empty(dev, torch.int64),
        freqs_ft_flat if freqs_ft_flat is not None else _empty(dev, torch.float32),
        freqs_fy_flat if freqs_fy_flat is not None else _empty(dev, torch.float32),
        freqs_fx_flat if freqs_fx_flat is not None else _empty(dev, torch.float32),
    )


def apply_pos_override(pos, starts, ends, vals) -> None:
    ops().apply_pos_override(pos, starts, ends, vals)


def anchor_store_write_frames(k_seq, v_seq, pos_seq, frame_desc, store_k, store_v,
                              store_pos) -> None:
    ops().anchor_store_write_frames(k_seq, v_seq, pos_seq, frame_desc, store_k, store_v,
                                    store_pos)


def refresh_readout_layout(src_k, src_v, src_pos, src_ptrs_k, src_ptrs_v, src_ptrs_pos,
                           offsets, lengths, flags, dynamic_rope_t, dst_k_raw, dst_v,
                           dst_rope_pos, dst_frame_ids, head_dim, current_t,
                           history_time_mapping_mode, history_relative_t_max,
                           history_time_soft_factor) -> None:
    ops().refresh_readout_layout(
        src_k, src_v, src_pos, src_ptrs_k, src_ptrs_v, src_ptrs_pos, offsets, lengths, flags,
        dynamic_rope_t, dst_k_raw, dst_v, dst_rope_pos, dst_frame_ids, int(head_dim),
        int(current_t), str(history_time_mapping_mode), int(history_relative_t_max),
        float(history_time_soft_factor))
