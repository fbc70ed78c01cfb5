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


class PeerHeadExchange:
    """The same exchanges over NVLink peer memory, without NCCL on the data
    path: every rank's receive and output buffers are symmetric memory
    (``torch.distributed._symmetric_memory``), so the one pass that packs Q,
    K and V (``adahead.pkv_chunk_copy_peers``) stores each destination rank's
    share straight into that rank's receive buffer, and the one pass over the
    attention output stores each token owner's rows straight into its
    ``[L/n, H, D]`` output, at the rank's own heads.  After each pass the ranks
    barrier on the stream (bounded wait).  Receive buffers alternate between
    two, so a rank writing step i+1's data cannot overwrite what a slower peer
    still reads from step i (it passes step i+1's first barrier only after
    every peer has finished step i), and outputs rotate over three, so an
    output stays valid for the next two steps (time for an asynchronous copy
    out).  CUDA, bf16, fixed shapes per object; results equal
    :class:`HeadParallelExchange`'s bit for bit (both are plain copies).  No
    counterpart in the reference."""

    def __init__(self, group, shard_shape, device, timeout_ms: int = 10000):
        import torch.distributed._symmetric_memory as symm
        self.group = group
        self.n = _world(group)
        self.rank = dist.get_rank(group)
        _, lt, h, d = shard_shape
        if h % self.n:
            raise ValueError(f"{h} heads do not split over {self.n} ranks")
        self.lt, self.h, self.d, self.hl = lt, h, d, h // self.n
        self.timeout_ms = timeout_ms
        gname = group.group_name if group is not None else dist.group.WORLD.group_name
        self._recv, self._out = [], []
        for _ in range(2):
            recv = symm.empty(self.n, lt, 3, self.hl, d, dtype=torch.bfloat16, device=device)
            self._recv.append((recv, symm.rendezvous(recv, gname)))
        for _ in range(3):
            out = symm.empty(lt, h, d, dtype=torch.bfloat16, device=device)
            self._out.append((out, symm.rendezvous(out, gname)))
        self._ir = self._io = 0

    def to_heads(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> tuple:
        """Q, K, V ``[1, L/n, H, D]`` -> three ``[1, L, H/n, D]`` views."""
        from . import _ops
        recv, hr = self._recv[self._ir]
        self._ir ^= 1
        n, lt, hl, d = self.n, self.lt, self.hl, self.d
        blk = lt * 3 * hl * d                      # one source rank's block in a receive buffer
        dst = [int(p) + 2 * self.rank * blk for p in hr.buffer_ptrs]
        xs = (q, k, v)
        _ops.ops().pkv_chunk_copy_peers(list(xs), [x.stride(1) for x in xs],
                                        [hl * x.stride(2) for x in xs], dst, 3 * hl * d, hl * d,
                                        lt, hl * d)
        hr.barrier(channel=0, timeout_ms=self.timeout_ms)
        flat = recv.view(n * lt, 3, hl, d)
        return tuple(flat[:, i].unsqueeze(0) for i in range(3))

    def to_tokens(self, x: torch.Tensor) -> torch.Tensor:
        """``[1, L, H/n, D]`` (this rank's heads) -> ``[1, L/n, H, D]`` view of
        one of this rank's three output buffers (valid for the next two
        exchanges)."""
        from . import _ops
        out, ho = self._out[self._io]
        self._io = (self._io + 1) % 3
        lt, hl, d = self.lt, self.hl, self.d
        xs = x[0] if x.is_contiguous() else x[0].contiguous()
        # token chunk g (its lt rows) goes to rank g's output at this rank's heads
        dst = [int(p) + 2 * self.rank * hl * d for p in ho.buffer_ptrs]
        _ops.ops().pkv_chunk_copy_peers([xs], [hl * d], [lt * hl * d], dst, self.h * d, 0, lt,
                                        hl * d)
        ho.barrier(channel=0, timeout_ms=self.timeout_ms)
        return out.unsqueeze(0)


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
        if isinstance(self.exchange, PeerHeadExchange):
            raise NotImplementedError("the peer-memory exchange moves Q, K and V together: "
                                      "use step()")
        k, v = self.exchange.to_heads(new_k, new_v)
        self.local.update(k, v, current_start, **kwargs)

    def attend(self, q: torch.Tensor, current_start: int, **kwargs) -> torch.Tensor:
        if isinstance(self.exchange, PeerHeadExchange):
            raise NotImplementedError("the peer-memory exchange moves Q, K and V together: "
                                      "use step()")
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
                               exchange: str = "nccl", block_tokens: int | None = None,
                               **kwargs) -> list[HeadParallelMegaCache]:
    """``build_mega_caches`` for this rank's heads of the full ``[L][H]``
    composition matrix, wrapped for the token-sharded model side; the layers
    share one exchange: ``"nccl"`` (:class:`HeadParallelExchange`) or
    ``"peer"`` (:class:`PeerHeadExchange`, CUDA; needs ``block_tokens``, the
    tokens of a block, to size its symmetric buffers; ``step`` only)."""
    from ._mega_cache import build_mega_caches
    rank, world = dist.get_rank(group), _world(group)
    h0, h1 = head_range(rank, world, num_heads)
    local = build_mega_caches(num_layers, h1 - h0, head_dim, frame_seqlen, max_sink_frames,
                              max_middle_frames, max_recent_frames,
                              [list(row)[h0:h1] for row in compositions], **kwargs)
    if exchange == "peer":
        if block_tokens is None or block_tokens % world:
            raise ValueError("the peer exchange needs block_tokens divisible by the ranks")
        ex = PeerHeadExchange(group, (1, block_tokens // world, num_heads, head_dim),
                              kwargs.get("device", "cuda"))
    elif exchange == "nccl":
        ex = HeadParallelExchange(group)
    else:
        raise ValueError(f"unknown exchange {exchange!r}")
    return [HeadParallelMegaCache(c, group, ex) for c in local]
