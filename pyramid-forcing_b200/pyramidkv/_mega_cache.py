"""MegaCache: the per-layer KV cache of Pyramid Forcing on the B200 library.

Same API as the reference's pyramidkv/_mega_cache.py:42-756 --
``MegaCacheCtx``, ``MegaCache`` (``update`` / ``attend``),
``_composition_to_perhead_state`` and ``build_mega_caches`` -- so
``wan/modules/causal_model.py:216-227`` (``isinstance(kv_cache, MegaCache)``,
``update``, ``attend``) and ``pipeline/causal_inference.py:766-805`` work
unchanged.

What differs is where the work runs.  The reference's update reads three
per-head counters back to the host, loops over heads in Python issuing about a
hundred small copies, and snapshot-copies the whole recent pool twice per
call; its attend plans on the host (three blocking device-to-host copies and
seven host-to-device copies per call).  Here ``update`` is one op
(``adahead.pkv_cache_update``: device routing + state machine + vectorised
frame copies + merge accumulation + commit) and ``attend`` is one op
(``adahead.pkv_attend``: device plan + RoPE-fused pack + tcgen05 attention),
neither of which synchronises with the host, so a layer step can be captured
in a CUDA graph.  The visible state (pools, ``valid_count``, the committed
snapshot on the ctx, the state bytes) evolves exactly as the reference's.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np
import torch

from . import _mega_state_ops
from . import _mega_state_ref as ref
from . import _ops

_STRATEGY_NAME_TO_KIND = {
    "RecentStrategy": ref.SK_RECENT,
    "CyclicStrategy": ref.SK_CYCLIC,
    "StrideStrategy": ref.SK_STRIDE,
    "LagStrategy": ref.SK_LAG,
    "MergeStrategy": ref.SK_MERGE,
}
_SINK_MODE = {"lag": 0, "window_clamp": 1}


@dataclass
class MegaCacheCtx:
    """State shared by all per-layer MegaCache views (fields as the reference)."""
    mgr: object
    states_bytes: torch.Tensor
    num_layers: int
    num_heads: int
    head_dim: int
    frame_seqlen: int
    sink_time_mapping_mode: str = "lag"
    sink_time_clamp_min: int = 0
    sink_time_clamp_max: int = 21
    decoupled_sink_time_lag: int = 0
    history_time_mapping_mode: str = "none"
    history_relative_t_max: int = 21
    history_time_soft_factor: float = 1.0
    spatial_width: int = 52
    spatial_height: int = 30
    has_merge_head: bool = False
    sink_caps_per_head: torch.Tensor = None
    committed_vc: torch.Tensor = None
    committed_recent_k: torch.Tensor = None
    committed_recent_v: torch.Tensor = None
    committed_recent_pos: torch.Tensor = None
    freqs: torch.Tensor = None
    freq_parts: tuple = None
    freq_parts_flat: tuple = None
    # device int64 counter of packed K/V tokens over all attend calls (the
    # attention FLOP / pack byte accounting of the benchmark); None disables
    token_counter: torch.Tensor = None
    # optional callable invoked between the pack and the attention launches of
    # attend() (used to place CUDA events around the attention kernel)
    on_stage: object = None

    def device_block_time(self) -> torch.Tensor:
        """Make the kernels read the block's first latent frame from a device
        int64 scalar (returned) instead of ``current_start``: write
        ``current_start // frame_seqlen`` into it before each layer step, and
        one captured CUDA graph of a layer step replays for every block.  Not
        in the reference (whose planner takes the time on the host)."""
        if getattr(self, "_block_time", None) is None:
            self._block_time = torch.zeros(1, dtype=torch.int64,
                                           device=self.states_bytes.device)
            self.mgr.set_block_time(self._block_time)
        return self._block_time

    def check_status(self) -> int:
        """Synchronise, read and clear the device status word; raise on errors."""
        st = int(_ops.ops().pkv_status(self.mgr))
        if st:
            raise RuntimeError(f"pyramidkv device status 0x{st:x} "
                               "(see PKV_ST_* in include/pkv.h)")
        return st


class MegaCache:
    """Per-layer view onto the shared MegaCacheCtx."""

    def __init__(self, ctx: MegaCacheCtx, layer_idx: int):
        self.ctx = ctx
        self.layer_idx = layer_idx
        self._frame_seqlen = ctx.frame_seqlen
        self.frame_seq_length = ctx.frame_seqlen
        self.num_heads = ctx.num_heads
        self.head_dim = ctx.head_dim
        self.batch_size = 1

    @property
    def states_bytes_for_layer(self) -> torch.Tensor:
        return self.ctx.states_bytes[self.layer_idx]

    def _ensure_snapshot(self) -> None:
        ctx = self.ctx
        mgr = ctx.mgr
        if ctx.committed_vc is None:
            ctx.committed_vc = mgr.valid_count().clone()
        if ctx.committed_recent_k is None:
            ctx.committed_recent_k = mgr.recent_k_pool().clone()
            ctx.committed_recent_v = mgr.recent_v_pool().clone()
            ctx.committed_recent_pos = mgr.recent_pos_pool().clone()

    def update(self, new_k: torch.Tensor, new_v: torch.Tensor, current_start: int, *,
               cache_update_mode: str = "clean", freqs=None) -> None:
        """Insert the incoming frames (raw K) of this layer (reference :136-414)."""
        if cache_update_mode == "default":
            cache_update_mode = "clean"
        if cache_update_mode not in ("noisy", "clean"):
            return
        ctx = self.ctx
        FSEQ, H, D = int(ctx.frame_seqlen), int(ctx.num_heads), int(ctx.head_dim)
        assert new_k.shape == new_v.shape, "K/V shapes must match"
        B, L_in, Hk, Dk = new_k.shape
        assert B == 1, "MegaCache.update: B>1 not yet supported"
        assert Hk == H and Dk == D
        assert L_in % FSEQ == 0, f"L_in ({L_in}) not multiple of FSEQ ({FSEQ})"
        self._ensure_snapshot()
        _ops.ops().pkv_cache_update(
            ctx.mgr, ctx.states_bytes, int(self.layer_idx), new_k, new_v,
            int(current_start // FSEQ), 1 if cache_update_mode == "clean" else 0,
            ctx.sink_caps_per_head, ctx.committed_vc, ctx.committed_recent_k,
            ctx.committed_recent_v, ctx.committed_recent_pos, int(ctx.spatial_width),
            bool(ctx.has_merge_head))

    def attend(self, q: torch.Tensor, current_start: int, *, freqs=None, softmax_scale=None,
               causal: bool = False, max_seqlen_k=None) -> torch.Tensor:
        """Attention output [B, L_q, H, D] from the current cache (reference :419-569)."""
        ctx = self.ctx
        FSEQ = int(ctx.frame_seqlen)
        B, L_q, H, D = q.shape
        assert B == 1, "MegaCache.attend: B>1 not yet supported"
        assert L_q % FSEQ == 0, f"L_q ({L_q}) must be a multiple of FSEQ ({FSEQ})"
        if causal:
            raise NotImplementedError("MegaCache.attend: the ragged cache attention is non-causal")
        eff_freqs = ctx.freqs if ctx.freqs is not None else freqs
        tables = ctx.freq_parts_flat
        if tables is None and eff_freqs is not None:
            tables = _flat_parts(eff_freqs.to(q.device), D)[1]
            ctx.freq_parts_flat = tables
        if eff_freqs is None:
            tables = None
        dev = q.device
        empty = _empty_f32(dev)
        ft, fy, fx = tables if tables is not None else (empty, empty, empty)
        if softmax_scale is None:
            softmax_scale = D ** -0.5
        counter = ctx.token_counter if ctx.token_counter is not None else _empty_i64(dev)
        args = (int(current_start // FSEQ), int(_SINK_MODE.get(ctx.sink_time_mapping_mode, 0)),
                int(ctx.sink_time_clamp_min), int(ctx.sink_time_clamp_max),
                int(ctx.decoupled_sink_time_lag), ft, fy, fx)
        ops = _ops.ops()
        if ctx.on_stage is None:
            out = ops.pkv_attend(ctx.mgr, self.states_bytes_for_layer, int(self.layer_idx), q,
                                 *args, float(softmax_scale), counter)
        else:
            ops.pkv_attend_pack(ctx.mgr, self.states_bytes_for_layer, int(self.layer_idx),
                                int(L_q), *args, counter)
            ctx.on_stage("packed")
            out = ops.pkv_attend_attention(ctx.mgr, q, float(softmax_scale))
        return out if out.dtype == q.dtype else out.to(q.dtype)


_EMPTY: dict = {}


def _empty_f32(dev):
    key = ("f32", str(dev))
    if key not in _EMPTY:
        _EMPTY[key] = torch.empty(0, dtype=torch.float32, device=dev)
    return _EMPTY[key]


def _empty_i64(dev):
    key = ("i64", str(dev))
    if key not in _EMPTY:
        _EMPTY[key] = torch.empty(0, dtype=torch.int64, device=dev)
    return _EMPTY[key]


def _flat_parts(freqs: torch.Tensor, head_dim: int):
    """Split the [max_t, head_dim/2] complex table into (t, y, x) parts and
    their fp32 (re, im)-interleaved [max_t, cols*2] copies for the kernels."""
    c = head_dim // 2
    parts = tuple(p.contiguous() for p in freqs.split([c - 2 * (c // 3), c // 3, c // 3], dim=1))
    flat = tuple(torch.view_as_real(p.to(torch.complex64)).contiguous().view(p.shape[0], -1)
                 for p in parts)
    return parts, flat


def _composition_to_perhead_state(composition) -> ref.PerHeadState:
    """HeadComposition -> PerHeadState (reference :572-628): the first middle
    strategy picks the kind; composition.sink_frames is the sink capacity."""
    sink_cap = int(getattr(composition, "sink_frames", 0))
    middles = list(getattr(composition, "middle_strategies", []) or [])
    if not middles:
        state = ref.make_recent()
    else:
        m = middles[0]
        name = type(m).__name__
        if name == "CyclicStrategy":
            state = ref.make_cyclic(period=int(m.period), bucket_cap=int(m.bucket_cap))
        elif name == "StrideStrategy":
            cap = int(m.capacity)
            state = ref.make_stride(interval=int(m.interval),
                                    capacity=ref.MAX_T_KEYED if cap <= 0 or cap > ref.MAX_T_KEYED
                                    else cap)
        elif name == "LagStrategy":
            hist = min(int(getattr(m, "history_frames", ref.MAX_T_KEYED)), ref.MAX_T_KEYED)
            state = ref.make_lag(history_frames=hist,
                                 offsets=list(getattr(m, "offsets", []) or []))
        elif name == "MergeStrategy":
            state = ref.make_merge(patch_size=int(getattr(m, "patch_size", 2)),
                                   capacity=int(getattr(m, "capacity", ref.MAX_MERGE_BLOCKS)))
        else:
            state = ref.make_recent()
    state.sink_capacity = sink_cap
    return state


def _states_from_compositions(compositions, num_layers: int, num_heads: int):
    """[L][H] compositions -> (uint8 [L, H*600] state bytes, int64 [L, H] sink caps,
    any merge head)."""
    size = _mega_state_ops.PER_HEAD_STATE_DTYPE.itemsize
    raw = np.zeros((num_layers, num_heads * size), dtype=np.uint8)
    caps = np.zeros((num_layers, num_heads), dtype=np.int64)
    any_merge = False
    for l in range(num_layers):
        if len(compositions[l]) != num_heads:
            raise ValueError(f"compositions[{l}] has {len(compositions[l])} heads, "
                             f"expected {num_heads}")
        states = [_composition_to_perhead_state(c) for c in compositions[l]]
        any_merge = any_merge or any(s.kind == ref.SK_MERGE for s in states)
        caps[l] = [int(s.sink_capacity) for s in states]
        raw[l] = _mega_state_ops.pack_states(states).view(np.uint8).reshape(-1)
    return raw, caps, any_merge


def build_mega_caches(num_layers: int, num_heads: int, head_dim: int, frame_seqlen: int,
                      max_sink_frames: int, max_middle_frames: int, max_recent_frames: int,
                      compositions: Sequence[Sequence], *, max_attend_chunks: int = 8,
                      device: str = "cuda:0", kv_dtype: str = "bfloat16",
                      sink_time_mapping_mode: str = "lag", sink_time_clamp_min: int = 0,
                      sink_time_clamp_max: int = 21, decoupled_sink_time_lag: int = 0,
                      history_time_mapping_mode: str = "none", history_relative_t_max: int = 21,
                      history_time_soft_factor: float = 1.0, spatial_width: int = 52,
                      spatial_height: int = 30, freqs=None) -> list[MegaCache]:
    """(manager, state bytes, MegaCache x L) from an [L][H] composition matrix."""
    if len(compositions) != num_layers:
        raise ValueError(f"compositions has {len(compositions)} layers, expected {num_layers}")
    if not _ops._ensure_loaded():
        raise RuntimeError("CUDA scatter extension not available")
    mgr = torch.classes.adahead.PyramidKVCacheManager(
        num_layers, num_heads, head_dim, frame_seqlen, max_sink_frames, max_middle_frames,
        max_recent_frames, device, kv_dtype, int(max_attend_chunks))
    raw, caps, any_merge = _states_from_compositions(compositions, num_layers, num_heads)
    states_bytes = torch.from_numpy(raw).to(device=device).contiguous()
    parts = flat = None
    if freqs is not None:
        freqs = freqs.to(device=device)
        parts, flat = _flat_parts(freqs, head_dim)
    ctx = MegaCacheCtx(
        mgr=mgr, states_bytes=states_bytes, num_layers=num_layers, num_heads=num_heads,
        head_dim=head_dim, frame_seqlen=frame_seqlen,
        sink_time_mapping_mode=sink_time_mapping_mode, sink_time_clamp_min=sink_time_clamp_min,
        sink_time_clamp_max=sink_time_clamp_max, decoupled_sink_time_lag=decoupled_sink_time_lag,
        history_time_mapping_mode=history_time_mapping_mode,
        history_relative_t_max=history_relative_t_max,
        history_time_soft_factor=history_time_soft_factor, spatial_width=spatial_width,
        spatial_height=spatial_height, has_merge_head=any_merge,
        sink_caps_per_head=torch.from_numpy(caps).to(device=device).contiguous(), freqs=freqs,
        freq_parts=parts, freq_parts_flat=flat)
    return [MegaCache(ctx, layer_idx=l) for l in range(num_layers)]
