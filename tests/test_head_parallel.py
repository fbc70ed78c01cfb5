"""Head-parallel cache path on 2 CPU ranks (gloo).

The exchange layer of ``pyramidkv.head_parallel`` (token-sharded model side,
head-sharded cache side) is tested with the CPU oracle standing in for each
rank's GPU cache: every rank runs the oracle MegaCache on its own heads behind
``HeadParallelMegaCache``, and its attention outputs must equal, bit for bit,
the token shard of a single-process oracle run over all heads on the same
inputs.  Ranks are spawned (not forked) processes.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import pkv_oracle as O

WORLD = 2
L, H, D, W, HG, F = 2, 4, 64, 6, 4, 3
FSEQ = W * HG
BLOCKS = 5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, port: int, world: int = WORLD) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _oracle(labels):
    from pyramidkv import policy
    states, caps = policy.states_from_labels(labels, "baseline")
    tables, _ = O.rope_freq_tables(D)
    return O.OracleMegaCache(L, labels.shape[1], D, FSEQ, 3, 24, 4, states, caps,
                             spatial_width=W, sink_time_mapping_mode="window_clamp",
                             sink_time_clamp_min=18, sink_time_clamp_max=21,
                             freq_tables=tables)


class _OracleLayer:
    """One layer of the oracle behind the MegaCache update / attend interface
    (bf16 bits travel as int16 tensors)."""

    def __init__(self, orc, layer):
        self.orc, self.layer = orc, layer

    def update(self, k, v, start, cache_update_mode="clean"):
        as_u16 = lambda t: t.numpy().view(np.uint16)  # noqa: E731
        self.orc.update(self.layer, as_u16(k), as_u16(v), start, cache_update_mode)

    def attend(self, q, start):
        out, _ = self.orc.attend(self.layer, q.numpy().view(np.uint16), start)
        return torch.from_numpy(np.ascontiguousarray(out, dtype=np.float32))


def _inputs(seed=3):
    rng = np.random.default_rng(seed)
    mk = lambda: O.f32_to_bf16(rng.standard_normal((1, F * FSEQ, H, D), np.float32))  # noqa
    return [[(mk(), mk(), mk()) for _ in range(L)] for _ in range(BLOCKS)]


def _labels():
    return np.array([[-1, 1, 2, 2], [2, 1, -1, 1]])


def _expected():
    orc = _oracle(_labels())
    outs = []
    for blk, layers in enumerate(_inputs()):
        start = blk * F * FSEQ
        for mode in ("noisy", "clean"):
            for layer, (k, v, q) in enumerate(layers):
                orc.update(layer, k, v, start, mode)
                out, _ = orc.attend(layer, q, start)
                outs.append(out.astype(np.float32))
    return outs


def _worker_exchange(rank: int, port: int) -> None:
    from pyramidkv import head_parallel as hp
    _init(rank, port)
    try:
        g = torch.Generator().manual_seed(11)
        full = torch.randn(1, F * FSEQ, H, D, generator=g)      # same on every rank
        t0, t1 = hp.token_range(rank, WORLD, F * FSEQ)
        h0, h1 = hp.head_range(rank, WORLD, H)
        got = hp.tokens_to_heads(full[:, t0:t1].contiguous())
        assert torch.equal(got, full[:, :, h0:h1])
        back = hp.heads_to_tokens(got)
        assert torch.equal(back, full[:, t0:t1])
    finally:
        dist.destroy_process_group()


def _worker_cache(rank: int, port: int, expected, world: int = WORLD,
                  batched: bool = False) -> None:
    from pyramidkv import head_parallel as hp
    _init(rank, port, world)
    try:
        h0, h1 = hp.head_range(rank, world, H)
        t0, t1 = hp.token_range(rank, world, F * FSEQ)
        orc = _oracle(_labels()[:, h0:h1])
        ex = hp.HeadParallelExchange()
        layers = [hp.HeadParallelMegaCache(_OracleLayer(orc, l), exchange=ex) for l in range(L)]
        shard = lambda a: torch.from_numpy(np.ascontiguousarray(a[:, t0:t1]).view(np.int16))  # noqa
        i = 0
        for blk, inputs in enumerate(_inputs()):
            start = blk * F * FSEQ
            for mode in ("noisy", "clean"):
                for layer, (k, v, q) in enumerate(inputs):
                    if batched:   # Q, K and V in one exchange
                        out = layers[layer].step(shard(q), shard(k), shard(v), start,
                                                 cache_update_mode=mode).numpy()
                    else:
                        layers[layer].update(shard(k), shard(v), start, cache_update_mode=mode)
                        out = layers[layer].attend(shard(q), start).numpy()
                    want = expected[i][:, t0:t1]
                    assert out.shape == want.shape, (out.shape, want.shape)
                    assert np.array_equal(out, want), (rank, blk, mode, layer,
                                                       float(np.abs(out - want).max()))
                    i += 1
    finally:
        dist.destroy_process_group()


def test_head_and_token_ranges():
    from pyramidkv import head_parallel as hp
    assert [hp.head_range(r, 4, 12) for r in range(4)] == [(0, 3), (3, 6), (6, 9), (9, 12)]
    assert hp.token_range(1, 2, 4680) == (2340, 4680)
    with pytest.raises(ValueError):
        hp.head_range(0, 8, 12)


def test_exchange_round_trip_two_ranks():
    mp.spawn(_worker_exchange, args=(_free_port(),), nprocs=WORLD, join=True)


def test_head_parallel_cache_matches_single_rank():
    mp.spawn(_worker_cache, args=(_free_port(), _expected()), nprocs=WORLD, join=True)


@pytest.mark.parametrize("world", [2, 4])
def test_head_parallel_step_one_exchange(world):
    """``step``: Q, K and V travel in one all-to-all (2 and 4 ranks; at 4 ranks
    each rank owns one head); outputs equal the single-rank run bit for bit."""
    mp.spawn(_worker_cache, args=(_free_port(), _expected(), world, True), nprocs=world,
             join=True)
