"""Row digests of MegaCache state, shared by the fixture generator
(``make_megacache_golden.py``) and the GPU test that checks against it.

A digest is an exact integer: the row's bytes read as int16 words, times
seeded weights in [1, 2^15), summed in int64 (|sum| < 2^15 * 2^15 * 2^18, no
overflow), so it is the same on any device and any summation order, and any
change of a row's bytes changes it except with negligible probability.
"""
from __future__ import annotations

import numpy as np
import torch

# Every pool of the manager that MegaCache.update writes, with the number of
# leading dims that index one digest row ([L, H, slot] for the per-slot pools,
# [L, H] for the per-head counters).
POOLS = [
    ("sink_k_pool", 3), ("sink_v_pool", 3), ("sink_pos_pool", 3),
    ("middle_k_pool", 3), ("middle_v_pool", 3), ("middle_pos_pool", 3),
    ("recent_k_pool", 3), ("recent_v_pool", 3), ("recent_pos_pool", 3),
    ("merge_k_pool", 3), ("merge_v_pool", 3), ("merge_pos_pool", 3),
    ("merge_token_count", 2),
    ("merge_accum_sum_k", 3), ("merge_accum_sum_v", 3), ("merge_accum_pos", 3),
    ("merge_accum_group_ids", 3), ("merge_accum_tokens_per_group", 3),
    ("merge_accum_num_groups", 2),
]
# int16 words of the longest row digested: a bf16 [1560, 128] frame is 199,680
_MAX_WORDS = 1 << 18
_W: dict = {}


def _weights(n: int, device) -> torch.Tensor:
    if n > _MAX_WORDS:
        raise ValueError(f"row of {n} int16 words exceeds the digest's {_MAX_WORDS}")
    key = str(device)
    if key not in _W:
        w = np.random.default_rng(20261202).integers(1, 1 << 15, size=_MAX_WORDS, dtype=np.int64)
        _W[key] = torch.from_numpy(w).to(device)
    return _W[key]


def row_digests(x: torch.Tensor, n_lead: int) -> np.ndarray:
    """int64 digest of each row of ``x`` (rows = its first ``n_lead`` dims)."""
    rows = int(np.prod(x.shape[:n_lead])) if n_lead else 1
    b = x.contiguous().view(torch.uint8).reshape(rows, -1)
    if b.shape[1] % 2:
        b = torch.nn.functional.pad(b, (0, 1))
    words = b.view(torch.int16)
    w = _weights(words.shape[1], x.device)[:words.shape[1]]
    out = torch.empty(rows, dtype=torch.int64, device=x.device)
    step = max(1, (1 << 26) // max(1, words.shape[1]))   # bound the int64 temporary
    for r0 in range(0, rows, step):
        out[r0:r0 + step] = (words[r0:r0 + step].to(torch.int64) * w).sum(dim=1)
    return out.cpu().numpy()


def blob_digest(x: torch.Tensor) -> int:
    """One digest of a tensor of any size: row digests of its int16 words in
    blocks of 2^17, combined as a polynomial modulo 2^61 - 1 (exact)."""
    b = x.contiguous().view(torch.uint8).reshape(-1)
    if b.numel() == 0:
        return 0
    blk = 1 << 18                                   # bytes per block (2^17 words)
    pad = (-b.numel()) % blk
    if pad:
        b = torch.nn.functional.pad(b, (0, pad))
    rows = row_digests(b.view(-1, blk), 1)
    h, mod = 0, (1 << 61) - 1
    for d in rows.tolist():
        h = (h * 1000003 + d) % mod
    return h


def state_digests(mgr, states_bytes: torch.Tensor, committed: dict) -> dict:
    """Digests of the manager's pools, valid_count, the state bytes (per head)
    and the committed snapshot (``committed``: name -> tensor)."""
    d = {name: row_digests(getattr(mgr, name)(), lead) for name, lead in POOLS}
    d["valid_count"] = mgr.valid_count().cpu().numpy().astype(np.int64).reshape(-1)
    H = states_bytes.shape[-1] // 600
    d["states"] = row_digests(states_bytes.reshape(-1, H, 600), 2)
    for name, t in committed.items():
        d[name] = (t.cpu().numpy().astype(np.int64).reshape(-1) if t.dtype == torch.int64
                   and t.dim() == 3 else row_digests(t, 3))
    return d
