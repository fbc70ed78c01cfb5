"""Head-parallel cache path on 2 and 4 GPUs (NCCL), against one GPU.

Spawned ranks (one per GPU) each own 4/n of the 4 heads of a small model and
feed ``HeadParallelMegaCache`` their token shard of every block, through the
reference's two calls (``update`` then ``attend``: K and V in one exchange, Q
in another) or through ``step`` (Q, K and V in one exchange), with the NCCL
all-to-all exchange or the peer-memory one (symmetric memory: the pack kernel
stores each rank's share into the other ranks' buffers over NVLink).  The single-GPU
MegaCache over all heads runs on the same inputs; the gathered outputs of the
ranks must equal it bit for bit (these shapes give every rank the same
one-CTA-per-unit attention schedule as the single GPU).  Skipped with fewer
GPUs than ranks.  NVLS is off (NCCL_NVLS_ENABLE=0) and the process group has a
short timeout, so a failing rank ends the test with an error instead of a wait.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import pkv_oracle as O

pytestmark = pytest.mark.gpu
L, H, D, W, HG, F = 2, 4, 128, 13, 8, 3
FSEQ = W * HG
BLOCKS = 4


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _labels():
    return np.array([[-1, 1, 2, 2], [2, 1, -1, 1]])


def _build(num_heads, labels, device, builder=None):
    from pyramidkv import _mega_cache, policy
    _, full = O.rope_freq_tables(D)
    kw = dict(device=device, sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18,
              sink_time_clamp_max=21, spatial_width=W, spatial_height=HG, freqs=full)
    comps = policy.compositions_from_labels(labels)
    if builder is None:
        return _mega_cache.build_mega_caches(L, num_heads, D, FSEQ, 3, 24, 4, comps, **kw)
    return builder(L, H, D, FSEQ, 3, 24, 4, comps, **kw)


def _inputs():
    g = torch.Generator().manual_seed(21)
    mk = lambda: torch.randn(1, F * FSEQ, H, D, generator=g).to(torch.bfloat16)  # noqa: E731
    return [[(mk(), mk(), mk()) for _ in range(L)] for _ in range(BLOCKS)]


def _worker(rank: int, world: int, port: int, out_dir: str, batched: bool,
            exchange: str = "nccl") -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from pyramidkv import head_parallel as hp
        builder = lambda *a, **k: hp.build_head_parallel_caches(  # noqa: E731
            *a, exchange=exchange, block_tokens=F * FSEQ, **k)
        caches = _build(H, _labels(), dev, builder=builder)
        t0, t1 = hp.token_range(rank, world, F * FSEQ)
        got = []
        for blk, layers in enumerate(_inputs()):
            start = blk * F * FSEQ
            for mode in ("noisy", "clean"):
                for layer, (k, v, q) in enumerate(layers):
                    sh = lambda x: x[:, t0:t1].contiguous().to(dev)  # noqa: E731
                    if batched:
                        got.append(caches[layer].step(sh(q), sh(k), sh(v), start,
                                                      cache_update_mode=mode).cpu())
                    else:
                        caches[layer].update(sh(k), sh(v), start, cache_update_mode=mode)
                        got.append(caches[layer].attend(sh(q), start).cpu())
        torch.cuda.synchronize()
        torch.save(got, os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,batched,exchange", [(2, False, "nccl"), (2, True, "nccl"),
                                                    (4, True, "nccl"), (2, True, "peer"),
                                                    (4, True, "peer")])
def test_head_parallel_matches_one_gpu(tmp_path, world, batched, exchange):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_worker, args=(world, _port(), str(tmp_path), batched, exchange), nprocs=world,
             join=True)
    ref = _build(H, _labels(), "cuda:0")
    want = []
    for blk, layers in enumerate(_inputs()):
        start = blk * F * FSEQ
        for mode in ("noisy", "clean"):
            for layer, (k, v, q) in enumerate(layers):
                ref[layer].update(k.cuda(), v.cuda(), start, cache_update_mode=mode)
                want.append(ref[layer].attend(q.cuda(), start).cpu())
    parts = [torch.load(os.path.join(tmp_path, f"rank{r}.pt")) for r in range(world)]
    for i, w in enumerate(want):
        got = torch.cat([parts[r][i] for r in range(world)], dim=1)
        assert torch.equal(got.view(torch.int16), w.view(torch.int16)), i
