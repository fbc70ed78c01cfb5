"""Head-parallel MegaCache over n ranks (one process per GPU).

Every stage of the cache path -- state machine, frame routing, merge
accumulation, plan, pack and attention -- works on each head independently,
so n ranks can split the 12 heads of a layer.  The model side is
sequence-parallel (rank r holds tokens ``[r L/n, (r+1) L/n)`` of the block for
all heads); a Ulysses-style exchange turns that into head-parallel data for
the cache path and back:

* before ``update`` / ``attend``: one ``all_to_all_single`` sends each rank
  the block's tokens for its heads (``[1, L/n, H, D]`` -> ``[1, L, H/n, D]``).
  :meth:`HeadParallelMegaCache.step` moves Q, K and V in that one exchange;
  ``update`` moves K and V together and ``attend`` moves Q, for callers that
  keep the reference's two calls;
* after ``attend``: one ``all_to_all_single`` returns the output to the
  token owners.

On CUDA the send side is one gather kernel (``adahead.pkv_chunk_copy``) into
a by-destination buffer whose per-token chunks interleave Q, K and V, so the
received buffer already is ``[L, 3, H/n, D]`` and the cache reads Q, K and V
from it as strided views without a copy; the output is scattered back into
``[1, L/n, H, D]`` by the same kernel.  Send and receive buffers live on the
:class:`HeadParallelExchange` and are reused by every layer.  (In the model
the exchanges of consecutive layers cannot overlap each other's cache work:
layer l+1's Q/K/V come from layer l's output.)

The per-rank cache is an ordinary MegaCache built for the rank's heads (its
label columns, its state bytes), so its results are the single-GPU results for
those heads (bit for bit where the attention schedule is the same; at the
model's full sizes the SM-balanced attention may cut units differently on a
rank with fewer heads, which changes the fp32 summation order only).  The
exchange is NCCL over NVLink on GPUs and gloo on CPU (the tests).  No
counterpart in the reference, which runs the cache on one GPU; the layer split
follows its head-independent design (pyramidkv/_mega_cache.py:136-569 loops or
vectorises over heads only).
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
    dist.all_to_all_single(recv.reshape(-1).view(torch.uint8),
                           send.reshape(-1).view(torch.uint8), group=group)


def _native(t: torch.Tensor) -> bool:
    return t.is_cuda and t.dtype == torch.bfloat16


def _chunk_copy(srcs, src_ts, src_gs, dst, dst_ts, dst_gs, dst_is, tokens, groups, elems):
    from . import _ops
    _ops.ops().pkv_chunk_copy(list(srcs), list(src_ts), list(src_gs), dst, dst_ts, dst_gs,
                              dst_is, tokens, groups, elems)


class HeadParallelExchange:
    """The all-to-alls of one head-parallel group, with send / receive buffers
    kept across calls (every layer of a model shares one exchange)."""

    def __init__(self, group=None):
        self.group = group
        self.n = _world(group)
        self._bufs: dict = {}

    def _buf(self, key, shape, like: torch.Tensor) -> torch.Tensor:
        b = self._bufs.get(key)
        if b is None or tuple(b.shape) != tuple(shape) or b.device != like.device \
                or b.dtype != like.dtype:
            b = torch.empty(shape, dtype=like.dtype, device=like.device)
            self._bufs[key] = b
        return b

    def to_heads(self, *xs: torch.Tensor) -> tuple:
        """1-4 tensors ``[1, L/n, H, D]`` (this rank's tokens, all heads), in one
        exchange -> the same number of ``[1, L, H/n, D]`` views (all tokens,
        this rank's heads) into the receive buffer, valid until the next
        exchange of this object."""
        n, m = self.n, len(xs)
        x0 = xs[0]
        if x0.dim() != 4 or x0.shape[0] != 1:
            raise ValueError(f"expected [1, L/n, H, D], got {tuple(x0.shape)}")
        if any(tuple(x.shape) != tuple(x0.shape) or x.dtype != x0.dtype for x in xs):
            raise ValueError("exchanged tensors must share shape and dtype")
        _, lt, h, d = x0.shape
        if h % n:
            raise ValueError(f"{h} heads do not split over {n} ranks")
        hl = h // n
        send = self._buf(("send", m), (n, lt, m, hl, d), x0)
        recv = self._buf(("recv", m), (n, lt, m, hl, d), x0)
        if _native(x0) and all(x.stride(3) == 1 for x in xs):
            # send[r, t, i] = xs[i][0, t, r*hl:(r+1)*hl]
            _chunk_copy(xs, [x.stride(1) for x in xs], [hl * x.stride(2) for x in xs],
                        send, m * hl * d, lt * m * hl * d, hl * d, lt, n, hl * d)
        else:
            for i, x in enumerate(xs):
                send[:, :, i].copy_(x[0].reshape(lt, n, hl, d).permute(1, 0, 2, 3))
        _all_to_all_bytes(recv, send, self.group)
        flat = recv.view(n * lt, m, hl, d)   # source rank r's tokens are [r*lt, (r+1)*lt)
        return tuple(flat[:, i].unsqueeze(0) for i in range(m))

    def to_tokens(self, x: torch.Tensor) -> torch.Tensor:
        """``[1, L, H/n, D]`` (this rank's heads) -> a new ``[1, L/n, H, D]``
        (this rank's tokens, all heads)."""
        n = self.n
        if x.dim() != 4 or x.shape[0] != 1:
            raise ValueError(f"expected [1, L, H/n, D], got {tuple(x.shape)}")
        _, l, hl, d = x.shape
        if l % n:
            raise ValueError(f"{l} tokens do not split over {n} ranks")
        lt = l // n
        send = x[0].contiguous().view(n, lt, hl, d)  # token chunk r goes to rank r
        recv = self._buf(("recv_o",), (n, lt, hl, d), send)  # [source = head group, ...]
        _all_to_all_bytes(recv, send, self.group)
        out = torch.empty((1, lt, n * hl, d), dtype=x.dtype, device=x.device)
        if _native(x):
            # out[0, t, g*hl:(g+1)*hl] = recv[g, t]
            _chunk_copy([recv], [hl * d], [lt * hl * d], out, n * hl * d, hl * d, 0, lt, n,
                        hl * d)
        else:
            out[0].view(lt, n, hl, d).copy_(recv.permute(1, 0, 2, 3))
        return out


def tokens_to_heads(x: torch.Tensor, group=None) -> torch.Tensor:
    """``[1, L/n, H, D]`` (this rank's tokens, all heads) -> ``[1, L, H/n, D]``
    (all tokens in order, this rank's heads); a fresh contiguous tensor."""
    return HeadParallelExchange(group).to_heads(x)[0].contiguous()


def heads_to_tokens(x: torch.Tensor, group=None) -> torch.Tensor:
    """Inverse of :func:`tokens_to_heads`: ``[1, L, H/n, D]`` -> ``[1, L/n, H, D]``."""
    return HeadParallelExchange(group).to_tokens(x)


class HeadParallelMegaCache:
    """One layer's cache on this rank's heads, fed and read in the model's
    token-sharded layout.  ``local`` is any object with the MegaCache
    ``update(new_k, new_v, current_start, cache_update_mode=...)`` and
    ``attend(q, current_start, ...)`` methods over ``[1, L, H/n, D]``
    tensors (normally a :class:`~pyramidkv._mega_cache.MegaCache`).
    ``exchange`` is shared by the layers of one model (one per group)."""

    def __init__(self, local, group=None, exchange: HeadParallelExchange | None = None):
        self.local = local
        self.group = group
        self.exchange = exchange if exchange is not None else HeadParallelExchange(group)
        # optional callable(name) at the exchange boundaries ("exchanged_in",
        # "cache_done"), for timing the collectives apart from the cache work
        self.on_stage = None

    def _stage(self, name: str) -> None:
        if self.on_stage is not None:
            self.on_stage(name)

    def update(self, new_k: torch.Tensor, new_v: torch.Tensor, current_start: int,
               **kwargs) -> None:
        k, v = self.exchange.to_heads(new_k, new_v)
        self.local.update(k, v, current_start, **kwargs)

    def attend(self, q: torch.Tensor, current_start: int, **kwargs) -> torch.Tensor:
        (qh,) = self.exchange.to_heads(q)
        out = self.local.attend(qh, current_start, **kwargs)
        return self.exchange.to_tokens(out)

    def step(self, q: torch.Tensor, new_k: torch.Tensor, new_v: torch.Tensor,
             current_start: int, cache_update_mode: str = "clean", **kwargs) -> torch.Tensor:
        """``update(new_k, new_v)`` then ``attend(q)`` with Q, K and V in one
        exchange; returns the output in the token-sharded layout."""
        qh, kh, vh = self.exchange.to_heads(q, new_k, new_v)
        self._stage("exchanged_in")
        self.local.update(kh, vh, current_start, cache_update_mode=cache_update_mode)
        out = self.local.attend(qh, current_start, **kwargs)
        self._stage("cache_done")
        return self.exchange.to_tokens(out)


def build_head_parallel_caches(num_layers: int, num_heads: int, head_dim: int,
                               frame_seqlen: int, max_sink_frames: int,
                               max_middle_frames: int, max_recent_frames: int,
                               compositions: Sequence[Sequence], *, group=None,
                               **kwargs) -> list[HeadParallelMegaCache]:
    """``build_mega_caches`` for this rank's heads of the full ``[L][H]``
    composition matrix, wrapped for the token-sharded model side; the layers
    share one :class:`HeadParallelExchange`."""
    from ._mega_cache import build_mega_caches
    rank, world = dist.get_rank(group), _world(group)
    h0, h1 = head_range(rank, world, num_heads)
    local = build_mega_caches(num_layers, h1 - h0, head_dim, frame_seqlen, max_sink_frames,
                              max_middle_frames, max_recent_frames,
                              [list(row)[h0:h1] for row in compositions], **kwargs)
    ex = HeadParallelExchange(group)
    return [HeadParallelMegaCache(c, group, ex) for c in local]
