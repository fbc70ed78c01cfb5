"""A layer step of the cache path captured in a CUDA graph.

``MegaCache.update`` and ``MegaCache.attend`` enqueue device work only (no
host synchronisation, no device allocation outside torch's allocator), so a
layer step can be captured with ``torch.cuda.graph``.  Two cache sets start
identical; one runs a block's noisy pass, clean pass and attend eagerly, the
other captures the same calls and replays the graph once.  Outputs, pools,
valid counts and state bytes must agree bit for bit.  With the block's time
in device memory (``MegaCacheCtx.device_block_time``) one captured graph of a
layer step replays block after block: the second test captures it once and
replays it for three consecutive blocks against an eager run.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import pkv_oracle as O

pytestmark = pytest.mark.gpu

L, H, D, W, HG, F = 2, 4, 128, 13, 8, 3
FSEQ = W * HG


def _caches():
    from pyramidkv import _mega_cache, policy
    _, full = O.rope_freq_tables(D)
    labels = np.array([[-1, 1, 2, 2], [2, 1, -1, 1]])
    return _mega_cache.build_mega_caches(
        L, H, D, FSEQ, 3, 24, 4, policy.compositions_from_labels(labels), device="cuda:0",
        sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18, sink_time_clamp_max=21,
        spatial_width=W, spatial_height=HG, freqs=full)


def _state(caches):
    m = caches[0].ctx.mgr
    parts = [m.sink_k_pool(), m.middle_k_pool(), m.recent_k_pool(), m.recent_v_pool(),
             m.valid_count(), m.merge_k_pool(), m.merge_token_count(), caches[0].ctx.states_bytes]
    return [p.detach().clone().view(torch.uint8) if p.dtype != torch.uint8 else p.clone()
            for p in parts]


def test_layer_step_replays_like_eager(cuda):
    g = torch.Generator(device="cpu").manual_seed(9)
    rnd = lambda: torch.randn(1, F * FSEQ, H, D, generator=g).to(cuda, torch.bfloat16)  # noqa
    a, b, warm = _caches(), _caches(), _caches()
    blocks = [[(rnd(), rnd(), rnd()) for _ in range(L)] for _ in range(6)]
    for blk, layers in enumerate(blocks[:-1]):          # identical history on a and b
        start = blk * F * FSEQ
        for caches in (a, b, warm):
            for mode in ("noisy", "clean"):
                for layer, (k, v, q) in enumerate(layers):
                    caches[layer].update(k, v, start, cache_update_mode=mode)
                    caches[layer].attend(q, start)
    torch.cuda.synchronize()
    start = 5 * F * FSEQ
    last = blocks[-1]
    for layer, (k, v, q) in enumerate(last):             # warm-up of lazy host state
        warm[layer].update(k, v, start, cache_update_mode="clean")
        warm[layer].attend(q, start)
    torch.cuda.synchronize()

    eager = []
    for layer, (k, v, q) in enumerate(last):
        a[layer].update(k, v, start, cache_update_mode="noisy")
        a[layer].update(k, v, start, cache_update_mode="clean")
        eager.append(a[layer].attend(q, start))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = []
        for layer, (k, v, q) in enumerate(last):
            b[layer].update(k, v, start, cache_update_mode="noisy")
            b[layer].update(k, v, start, cache_update_mode="clean")
            captured.append(b[layer].attend(q, start))
    graph.replay()
    torch.cuda.synchronize()
    for x, y in zip(eager, captured):
        assert torch.equal(x.view(torch.int16), y.view(torch.int16))
    for x, y in zip(_state(a), _state(b)):
        assert torch.equal(x, y)
    assert a[0].ctx.check_status() == 0 and b[0].ctx.check_status() == 0


def test_one_graph_replays_across_blocks(cuda):
    g = torch.Generator(device="cpu").manual_seed(19)
    rnd = lambda: torch.randn(1, F * FSEQ, H, D, generator=g).to(cuda, torch.bfloat16)  # noqa
    a, b = _caches(), _caches()
    blocks = [[(rnd(), rnd(), rnd()) for _ in range(L)] for _ in range(7)]
    warm = 4
    for blk, layers in enumerate(blocks[:warm]):          # identical history, eager
        start = blk * F * FSEQ
        for caches in (a, b):
            for mode in ("noisy", "clean"):
                for layer, (k, v, q) in enumerate(layers):
                    caches[layer].update(k, v, start, cache_update_mode=mode)
                    caches[layer].attend(q, start)
    torch.cuda.synchronize()
    # b's kernels now read the block time from device memory; its inputs live
    # in static buffers the graph reads
    bt = b[0].ctx.device_block_time()
    static = [tuple(torch.empty_like(x) for x in blocks[0][0]) for _ in range(L)]
    bt.fill_(warm * F)
    for layer in range(L):
        for dst, src in zip(static[layer], blocks[warm][layer]):
            dst.copy_(src)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = []
        for layer, (k, v, q) in enumerate(static):
            b[layer].update(k, v, 0, cache_update_mode="noisy")   # time from bt
            b[layer].update(k, v, 0, cache_update_mode="clean")
            outs.append(b[layer].attend(q, 0))
    # capture enqueues nothing: replay block `warm` and the next ones
    for blk in range(warm, len(blocks)):
        start = blk * F * FSEQ
        eager = []
        for layer, (k, v, q) in enumerate(blocks[blk]):
            a[layer].update(k, v, start, cache_update_mode="noisy")
            a[layer].update(k, v, start, cache_update_mode="clean")
            eager.append(a[layer].attend(q, start))
        bt.fill_(blk * F)
        for layer in range(L):
            for dst, src in zip(static[layer], blocks[blk][layer]):
                dst.copy_(src)
        graph.replay()
        torch.cuda.synchronize()
        for x, y in zip(eager, outs):
            assert torch.equal(x.view(torch.int16), y.view(torch.int16)), blk
        for x, y in zip(_state(a), _state(b)):
            assert torch.equal(x, y), blk
    assert a[0].ctx.check_status() == 0 and b[0].ctx.check_status() == 0
