"""Per-layer readout helpers, same API as the reference's pyramidkv/_mega_attention.py.

``mega_readout_kv_only`` (plan + pack with fused RoPE, cloned K/V),
``mega_readout`` (+ ragged attention), ``mega_attention_step`` (state update +
middle writes + readout), ``_layer_offset_slot_global`` and
``_flash_attn_varlen``.  Attention runs on this library's tcgen05 kernel
(``torch.ops.adahead.pkv_attention``); ``_flash_attn_varlen()`` returns a
function with ``flash_attn_varlen_func``'s signature over the same kernel for
callers that hold flattened (segment-major) queries.
"""
from __future__ import annotations

import torch

from . import _mega_state_ops, _ops


def _flash_attn_varlen():
    """A ``flash_attn_varlen_func``-compatible callable on the pkv kernel.

    Supports the form the MegaCache path uses: every query sequence has the
    same length (``cu_seqlens_q`` = arange * max_seqlen_q), one head per
    packed row, non-causal, no dropout.
    """

    def varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
               dropout_p=0.0, softmax_scale=None, causal=False, **_unused):
        if causal:
            raise NotImplementedError("pkv ragged attention is non-causal")
        if dropout_p:
            raise NotImplementedError("pkv ragged attention has no dropout")
        D = q.shape[-1]
        n_seg = int(cu_seqlens_q.numel()) - 1
        rows = int(max_seqlen_q)
        if q.shape[0] != n_seg * rows:
            raise ValueError("cu_seqlens_q must describe equal-length query sequences")
        scale = D ** -0.5 if softmax_scale is None else float(softmax_scale)
        out = _ops.ops().pkv_attention(q.reshape(n_seg * rows, 1, D), k.reshape(-1, D),
                                       v.reshape(-1, D), cu_seqlens_k.to(torch.int32),
                                       n_seg, rows, scale)
        return out.view(q.shape)

    return varlen


def _flat_tables(freqs, freq_parts, head_dim: int, device):
    """fp32 [rows, cols*2] (re, im) tables of the (t, y, x) RoPE parts."""
    if freq_parts is None:
        c = head_dim // 2
        freq_parts = freqs.to(device=device).split([c - 2 * (c // 3), c // 3, c // 3], dim=1)
    return tuple(torch.view_as_real(p.to(device=device, dtype=torch.complex64))
                 .reshape(p.shape[0], -1).contiguous() for p in freq_parts)


def mega_readout_kv_only(mgr, per_head_states_bytes, layer_idx: int, current_t: int, H: int,
                         D: int, *, freqs=None, freq_parts=None, pass_kind: int = 1,
                         sink_time_mapping_mode: str = "lag", sink_time_clamp_min: int = 0,
                         sink_time_clamp_max: int = 21, decoupled_sink_time_lag: int = 0,
                         history_time_mapping_mode: str = "none",
                         history_relative_t_max: int = 21,
                         history_time_soft_factor: float = 1.0):
    """Plan + pack (+ RoPE) for one query chunk; returns cloned (k, v, cu_seqlens_k)."""
    (cu, sk, sg, sl, dst, _traw, tremap) = _mega_state_ops.mega_plan_cuda(
        mgr, per_head_states_bytes, layer_idx=layer_idx, current_t=current_t,
        pass_kind=pass_kind, sink_time_mapping_mode=sink_time_mapping_mode,
        sink_time_clamp_min=sink_time_clamp_min, sink_time_clamp_max=sink_time_clamp_max,
        decoupled_sink_time_lag=decoupled_sink_time_lag,
        history_time_mapping_mode=history_time_mapping_mode,
        history_relative_t_max=history_relative_t_max,
        history_time_soft_factor=history_time_soft_factor)
    sga = _layer_offset_slot_global(sg, sk, layer_idx, max_sink=int(mgr.max_sink()),
                                    max_middle=int(mgr.max_middle()),
                                    max_recent=int(mgr.max_recent()), num_heads=H,
                                    max_merge_blocks=int(mgr.max_merge_blocks()))
    if freqs is not None or freq_parts is not None:
        ft, fy, fx = _flat_tables(freqs, freq_parts, D, sk.device)
        _ops.pyramidkv_pack(mgr, sk, sga, sl, dst, anchor_t_remap=tremap, freqs_ft_flat=ft,
                            freqs_fy_flat=fy, freqs_fx_flat=fx)
    else:
        _ops.pyramidkv_pack(mgr, sk, sga, sl, dst)
    n_active = int(cu[-1].item())
    return (mgr.k_flat_out()[:n_active].clone(), mgr.v_flat_out()[:n_active].clone(),
            cu.clone())


def _attend_one_chunk(q, k_flat, v_flat, cu_seqlens_k, *, softmax_scale, causal,
                      max_seqlen_k: int):
    """Attention of one query chunk [B=1, L_q, H, D] over per-head ragged K/V."""
    if causal:
        raise NotImplementedError("pkv ragged attention is non-causal")
    B, L_q, H, D = q.shape
    qq = q[0] if q.dtype == torch.bfloat16 else q[0].to(torch.bfloat16)
    scale = D ** -0.5 if softmax_scale is None else float(softmax_scale)
    out = _ops.ops().pkv_attention(qq, k_flat.reshape(-1, D), v_flat.reshape(-1, D),
                                   cu_seqlens_k.to(torch.int32), 1, L_q, scale)
    return out.view(B, L_q, H, D).to(q.dtype)


def mega_readout(mgr, per_head_states_bytes, q, layer_idx: int, current_t: int, *, freqs=None,
                 freq_parts=None, pass_kind: int = 1, softmax_scale=None, causal: bool = False,
                 max_seqlen_k=None, sink_time_mapping_mode: str = "lag",
                 sink_time_clamp_min: int = 0, sink_time_clamp_max: int = 21,
                 decoupled_sink_time_lag: int = 0, history_time_mapping_mode: str = "none",
                 history_relative_t_max: int = 21, history_time_soft_factor: float = 1.0):
    """Single-chunk attention readout; returns [B, L_q, H, D] in q's dtype."""
    assert q.dim() == 4, f"q must be [B, L_q, H, D], got {tuple(q.shape)}"
    B, L_q, H, D = q.shape
    assert B == 1, "mega_readout: B>1 not yet supported"
    k, v, cu = mega_readout_kv_only(
        mgr=mgr, per_head_states_bytes=per_head_states_bytes, layer_idx=layer_idx,
        current_t=current_t, H=H, D=D, freqs=freqs, freq_parts=freq_parts,
        pass_kind=pass_kind, sink_time_mapping_mode=sink_time_mapping_mode,
        sink_time_clamp_min=sink_time_clamp_min, sink_time_clamp_max=sink_time_clamp_max,
        decoupled_sink_time_lag=decoupled_sink_time_lag,
        history_time_mapping_mode=history_time_mapping_mode,
        history_relative_t_max=history_relative_t_max,
        history_time_soft_factor=history_time_soft_factor)
    if max_seqlen_k is None:
        max_seqlen_k = int(mgr.max_total()) * int(mgr.frame_seqlen())
    return _attend_one_chunk(q, k, v, cu, softmax_scale=softmax_scale, causal=causal,
                             max_seqlen_k=max_seqlen_k)


def mega_attention_step(mgr, per_head_states_bytes, q, k_new, v_new, new_t_vals,
                        layer_idx: int, current_t: int, *, pass_kind: int = 1,
                        softmax_scale=None, causal: bool = False, max_seqlen_k=None,
                        sink_time_mapping_mode: str = "lag", sink_time_clamp_min: int = 0,
                        sink_time_clamp_max: int = 21, decoupled_sink_time_lag: int = 0,
                        history_time_mapping_mode: str = "none",
                        history_relative_t_max: int = 21,
                        history_time_soft_factor: float = 1.0):
    """State update + middle writes + readout (reference _mega_attention.py:224-346)."""
    assert q.shape == k_new.shape == v_new.shape, "q, k_new, v_new must agree"
    B, L_q, H, D = q.shape
    F = int(new_t_vals.shape[0])
    FSEQ = int(mgr.frame_seqlen())
    assert L_q == F * FSEQ, f"L_q ({L_q}) must equal F ({F}) * FSEQ ({FSEQ})"
    assert B == 1, "mega_attention_step: B>1 not yet supported"
    dev = q.device
    N = H * F
    d = [torch.full((N,), -1, dtype=torch.int32, device=dev) for _ in range(8)]
    _ops.ops().mega_state_update(per_head_states_bytes, new_t_vals, *d, int(H), int(F),
                                 int(pass_kind))
    kind, slot_local, src_frame, src_head = d[0], d[1], d[2], d[3]
    slot_global = (slot_local.long() + (layer_idx * H + src_head.long())
                   * int(mgr.max_middle())).to(torch.int32)
    nk = k_new.view(B, F, FSEQ, H, D).permute(0, 1, 3, 2, 4).reshape(F, H, FSEQ, D).contiguous()
    nv = v_new.view(B, F, FSEQ, H, D).permute(0, 1, 3, 2, 4).reshape(F, H, FSEQ, D).contiguous()
    _ops.ops().pyramidkv_update(mgr, nk, nv, torch.empty(0, dtype=torch.int64, device=dev),
                                kind, slot_global, src_frame, src_head)
    return mega_readout(
        mgr=mgr, per_head_states_bytes=per_head_states_bytes, q=q, layer_idx=layer_idx,
        current_t=current_t, pass_kind=pass_kind, softmax_scale=softmax_scale, causal=causal,
        max_seqlen_k=max_seqlen_k, sink_time_mapping_mode=sink_time_mapping_mode,
        sink_time_clamp_min=sink_time_clamp_min, sink_time_clamp_max=sink_time_clamp_max,
        decoupled_sink_time_lag=decoupled_sink_time_lag,
        history_time_mapping_mode=history_time_mapping_mode,
        history_relative_t_max=history_relative_t_max,
        history_time_soft_factor=history_time_soft_factor)


def _layer_offset_slot_global(src_slot_global, src_kind, layer_idx: int, max_sink: int,
                              max_middle: int, max_recent: int, num_heads: int,
                              max_merge_blocks: int = 0):
    """Add layer_idx * H * max_slots[kind] to every active segment's slot id."""
    if layer_idx == 0:
        return src_slot_global
    per_kind = torch.tensor([max_sink, max_middle, max_recent, max_merge_blocks],
                            dtype=torch.int32, device=src_slot_global.device)
    per_kind = per_kind * int(layer_idx * num_heads)
    active = src_kind >= 0
    offset = per_kind[src_kind.clamp(min=0).long()] * active.to(torch.int32)
    return src_slot_global + offset
