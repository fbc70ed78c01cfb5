"""Head-parallel MegaCache over n ranks (one process per GPU).

Every stage of the cache path -- state machine, frame routing, merge
accumulation, plan, pack and attention -- works on each head independently,
so n ranks can split the 12 heads of a layer.  The model side is
sequence-parallel (rank r holds tokens ``[r L/n, (r+1) L/n)`` of the block for
all heads); a Ulysses-style exchange turns that into head-parallel data for
the cache path and back:

* before ``update`` / ``attend``: ``tokens_to_heads`` -- one
  ``all_to_all_single`` that sends each rank the block's tokens for its heads
  (``[1, L/n, H, D]`` -> ``[1, L, H/n, D]``);
* after ``attend``: ``heads_to_tokens`` -- the inverse for the output.

The per-rank cache is an ordinary MegaCache built for the rank's heads (its
label columns, its state bytes), so its results are exactly the single-GPU
results for those heads.  The exchange is NCCL over NVLink on GPUs and gloo on
CPU (the tests).  No counterpart in the reference, which runs the cache on one
GPU; the layer split follows its head-independent design
(pyramidkv/_mega_cache.py:136-569 loops or vectorises over heads only).
"""
from __future__ import annotations

from typing import Sequence

import torch
import torch.distributed as dist


def head_range(rank: int, world: int, num_heads: int) -> tuple[int, int]:
    """Heads ``[h0, h1)`` owned by ``rank``; ``num_heads`` must divide evenly."""
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split over {world} ranks")
    per = num_heads // world
    return rank * per, (rank + 1) * per


def token_range(rank: int, world: int, num_tokens: int) -> tuple[int, int]:
    """Tokens ``[t0, t1)`` of a block held by ``rank`` on the model side."""
    if num_tokens % world:
        raise ValueError(f"{num_tokens} tokens do not split over {world} ranks")
    per = num_tokens // world
    return rank * per, (rank + 1) * per


def _world(group) -> int:
    return dist.get_world_size(group)


def _all_to_all_bytes(recv: torch.Tensor, send: torch.Tensor, group) -> None:
    """all_to_all_single over the raw bytes (dim 0 split evenly), so any element
    type travels, including ones a backend does not take (gloo has no int16)."""
    dist.all_to_all_single(recv.view(torch.uint8), send.view(torch.uint8), group=group)


def tokens_to_heads(x: torch.Tensor, group=None) -> torch.Tensor:
    """``[1, L/n, H, D]`` (this rank's tokens, all heads) -> ``[1, L, H/n, D]``
    (all tokens in order, this rank's heads)."""
    n = _world(group)
    if x.dim() != 4 or x.shape[0] != 1:
        raise ValueError(f"expected [1, L/n, H, D], got {tuple(x.shape)}")
    _, lt, h, d = x.shape
    if h % n:
        raise ValueError(f"{h} heads do not split over {n} ranks")
    hl = h // n
    send = x[0].reshape(lt, n, hl, d).permute(1, 0, 2, 3).contiguous()  # by destination rank
    recv = torch.empty_like(send)                                         # [n, L/n, H/n, D]
    _all_to_all_bytes(recv, send, group)
    return recv.reshape(n * lt, hl, d).unsqueeze(0)


def heads_to_tokens(x: torch.Tensor, group=None) -> torch.Tensor:
    """Inverse of :func:`tokens_to_heads`: ``[1, L, H/n, D]`` -> ``[1, L/n, H, D]``."""
    n = _world(group)
    if x.dim() != 4 or x.shape[0] != 1:
        raise ValueError(f"expected [1, L, H/n, D], got {tuple(x.shape)}")
    _, l, hl, d = x.shape
    if l % n:
        raise ValueError(f"{l} tokens do not split over {n} ranks")
    lt = l // n
    send = x[0].reshape(n, lt, hl, d).contiguous()  # token chunk i goes to rank i
    recv = torch.empty_like(send)                    # [n (source = head group), L/n, H/n, D]
    _all_to_all_bytes(recv, send, group)
    return recv.permute(1, 0, 2, 3).reshape(lt, n * hl, d).unsqueeze(0)


class HeadParallelMegaCache:
    """One layer's cache on this rank's heads, fed and read in the model's
    token-sharded layout.  ``local`` is any object with the MegaCache
    ``update(new_k, new_v, current_start, cache_update_mode=...)`` and
    ``attend(q, current_start, ...)`` methods over ``[1, L, H/n, D]``
    tensors (normally a :class:`~pyramidkv._mega_cache.MegaCache`)."""

    def __init__(self, local, group=None):
        self.local = local
        self.group = group

    def update(self, new_k: torch.Tensor, new_v: torch.Tensor, current_start: int,
               **kwargs) -> None:
        self.local.update(tokens_to_heads(new_k, self.group),
                          tokens_to_heads(new_v, self.group), current_start, **kwargs)

    def attend(self, q: torch.Tensor, current_start: int, **kwargs) -> torch.Tensor:
        out = self.local.attend(tokens_to_heads(q, self.group), current_start, **kwargs)
        return heads_to_tokens(out, self.group)


def build_head_parallel_caches(num_layers: int, num_heads: int, head_dim: int,
                               frame_seqlen: int, max_sink_frames: int,
                               max_middle_frames: int, max_recent_frames: int,
                               compositions: Sequence[Sequence], *, group=None,
                               **kwargs) -> list[HeadParallelMegaCache]:
    """``build_mega_caches`` for this rank's heads of the full ``[L][H]``
    composition matrix, wrapped for the token-sharded model side."""
    from ._mega_cache import build_mega_caches
    rank, world = dist.get_rank(group), _world(group)
    h0, h1 = head_range(rank, world, num_heads)
    local = build_mega_caches(num_layers, h1 - h0, head_dim, frame_seqlen, max_sink_frames,
                              max_middle_frames, max_recent_frames,
                              [list(row)[h0:h1] for row in compositions], **kwargs)
    return [HeadParallelMegaCache(c, group) for c in local]
