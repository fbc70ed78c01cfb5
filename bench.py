#!/usr/bin/env python
"""Benchmark: the per-layer-step KV-cache path of causal Wan2.1-T2V-1.3B.

Metric: cache-update + ragged-attention microseconds per DiT
layer-step, reported as latent frames/s.  One "step" is one 120-latent-frame
video's cache path (configs[1], C2): 40 blocks of 3 latent frames, each block
4 noisy + 1 clean forwards, each forward 30 layers of
``MegaCache.update(k, v)`` + ``MegaCache.attend(q)`` -- 6000 layer-steps.
12 heads x 128, 1560 tokens per latent frame (30 x 52), sink/middle/recent
pools 3/24/4 frames, window_clamp(18, 21) sink time, a seeded random [30, 12]
label matrix over {-1, 1, 2} under the BASELINE routing (stride for 1,
periodic for 2, merge for -1).  The DiT's GEMMs, text encoder and VAE are
outside the path and not run; Q/K/V are seeded N(0, 1) bf16 tensors from a
rotating set of 8 (inputs + cache pools are larger than L2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs N independent videos, one per rank (weak scaling, no collective on
the data path); at N = 2, 3, 4, 6 and 8 the line also carries a
``head_parallel`` object: videos split by heads over groups of n = N ranks
(n = 4 at N = 8), each layer-step's Q/K/V and output crossing NVLink in two
NCCL all-to-alls inside the timed region.  ``--head-parallel n`` makes that
the line's own measurement.  ``--impl reference`` times the CPU oracle port of
the reference path on the host cores (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "pyramid-forcing_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "cache-update+ragged-attn µs per DiT layer-step; latent frames/sec"
# DRAM bytes per FLOP of the attention (ncu, balanced schedule, C2 kernel case:
# 478.9 MB read + 26.1 MB written for 0.492 TFLOP)
ATTN_DRAM_BYTES_PER_FLOP = 505.0e6 / 492.171264e9
L_, H_, D_, W_, HG_ = 30, 12, 128, 52, 30
FSEQ = W_ * HG_
FRAMES_PER_BLOCK = 3
PASSES = ("noisy", "noisy", "noisy", "noisy", "clean")
N_SETS = 8


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--frames", type=int, default=120)
    ap.add_argument("--merge-fraction", type=float, default=None,
                    help="exact share of merge heads (configs[2] uses 0.5)")
    ap.add_argument("--e2e-steps", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--kernel-case",
                    choices=["attn", "attn-plain", "attn-c4", "attn-d64", "pack", "update",
                             "rope-q", "chunk-copy"],
                    default=None,
                    help="run one kernel on a standalone steady-state-sized input "
                         "(small device footprint, for profiler captures) and exit")
    ap.add_argument("--kernel-iters", type=int, default=4)
    ap.add_argument("--kernel-heads", type=int, default=H_,
                    help="heads of the attn kernel cases (6 / 3: a head-parallel rank's share)")
    ap.add_argument("--batch", type=int, default=1,
                    help="videos per attention launch of --kernel-case attn-c4 (configs[3])")
    ap.add_argument("--head-parallel", type=int, default=0, metavar="n",
                    help="split each video's heads over groups of n ranks (n divides 12 and "
                         "the rank count); the line then measures world/n head-parallel videos")
    ap.add_argument("--no-dit", action="store_true",
                    help="skip the random-init DiT leg (latent frames/s over DiT wall time)")
    ap.add_argument("--hp-exchange", choices=["peer", "nccl"], default="peer",
                    help="head-parallel exchange: NVLink peer stores into symmetric memory, "
                         "or NCCL all_to_all_single")
    ap.add_argument("--hp-steps", type=int, default=3,
                    help="videos timed by the head-parallel leg added to N > 1 lines")
    return ap.parse_args()


def workload_config(args):
    cfg = {"workload": ("C2 cache path of causal Wan2.1-T2V-1.3B: %d latent frames, 30 layers x "
                        "12 heads x 128, 1560 tokens/frame, 3-frame blocks x (4 noisy + 1 clean)"
                        % args.frames),
           "layers": L_, "heads": H_, "head_dim": D_, "frame_tokens": FSEQ,
           "frames_per_block": FRAMES_PER_BLOCK, "passes_per_block": len(PASSES),
           "latent_frames": args.frames, "pools_frames": {"sink": 3, "middle": 24, "recent": 4},
           "routing": "baseline (1: stride, 2: periodic, -1: merge)",
           "labels": "seeded uniform [30,12]" if args.merge_fraction is None
           else f"seeded, merge share {args.merge_fraction}",
           "l2": "inputs larger than L2 (multi-GB cache pools, 8 rotating Q/K/V sets)"}
    return cfg


class Workload:
    """30 MegaCache layers + rotating device inputs for one video."""

    @staticmethod
    def build(device, seed: int, merge_fraction=None):
        import torch
        from pyramidkv import _mega_cache, policy

        w = Workload.__new__(Workload)
        w.device = device
        w.labels = policy.random_labels(L_, H_, seed=seed, merge_fraction=merge_fraction)
        comps = policy.compositions_from_labels(w.labels, "baseline")
        w.caches = _mega_cache.build_mega_caches(
            L_, H_, D_, FSEQ, 3, 24, 4, comps, max_attend_chunks=8, device=str(device),
            sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18,
            sink_time_clamp_max=21, spatial_width=W_, spatial_height=HG_,
            freqs=rope_table(D_))
        w.ctx = w.caches[0].ctx
        w.init_states = w.ctx.states_bytes.clone()
        w.ctx.token_counter = torch.zeros(1, dtype=torch.int64, device=device)
        g = torch.Generator(device=device).manual_seed(1000 + seed)
        shape = (1, FRAMES_PER_BLOCK * FSEQ, H_, D_)
        w.sets = [tuple(torch.randn(shape, generator=g, device=device, dtype=torch.bfloat16)
                        for _ in range(3)) for _ in range(N_SETS)]
        return w

    def reset(self):
        """Empty cache, initial strategy states (start of a new video)."""
        ctx = self.ctx
        ctx.mgr.reset()
        ctx.states_bytes.copy_(self.init_states)
        if ctx.committed_vc is not None:
            ctx.committed_vc.zero_()


def rope_table(d: int):
    """The model's RoPE table (wan/modules/causal_model.py:586-591 layout):
    complex128 [1024, d/2] = polar(1, t * 10000^(-2i/dim)) for the t / y / x
    parts of sizes d - 4(d//6), 2(d//6), 2(d//6)."""
    import torch

    def part(dim):
        inv = 1.0 / torch.pow(10000, torch.arange(0, dim, 2).to(torch.float64).div(dim))
        ang = torch.outer(torch.arange(1024), inv)
        return torch.polar(torch.ones_like(ang), ang)

    return torch.cat([part(d - 4 * (d // 6)), part(2 * (d // 6)), part(2 * (d // 6))], dim=1)


def run_video(w, frames: int, inputs=None, hooks=None):
    """One video's cache path.  inputs(i) -> (q, k, v) for layer-step i (default:
    the rotating device sets); hooks: (before_update, after_update, after_attend)
    callables receiving the layer-step index."""
    caches = w.caches
    i = 0
    n_blocks = frames // FRAMES_PER_BLOCK
    for blk in range(n_blocks):
        start = blk * FRAMES_PER_BLOCK * FSEQ
        for mode in PASSES:
            for layer in range(L_):
                q, k, v = inputs(i) if inputs is not None else w.sets[i % N_SETS]
                if hooks:
                    hooks[0](i)
                caches[layer].update(k, v, start, cache_update_mode=mode)
                if hooks:
                    hooks[1](i)
                out = caches[layer].attend(q, start)
                if hooks:
                    hooks[2](i, out)
                i += 1
    return i


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
_CLOCK_FIELDS = ["clocks.sm", "clocks.max.sm", "power.draw",
                 "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
                 "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]


def clocks_start(gpu: int):
    path = os.path.join("/tmp", f"pkv_clocks_{os.getpid()}_{gpu}.csv")
    try:
        f = open(path, "w")
        p = subprocess.Popen(["nvidia-smi", "-i", str(gpu), "--query-gpu=" + ",".join(_CLOCK_FIELDS),
                              "--format=csv,noheader,nounits", "-lms", "200"],
                             stdout=f, stderr=subprocess.DEVNULL)
        return p, f, path
    except OSError:
        return None


def clocks_stop(h):
    if h is None:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
    p, f, path = h
    p.terminate()
    try:
        p.wait(timeout=5)
    except subprocess.TimeoutExpired:
        p.kill()
    f.close()
    sm, mx, pw, reasons = [], [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in open(path).read().strip().splitlines():
        cols = [c.strip() for c in line.split(",")]
        if len(cols) < 7:
            continue
        try:
            sm.append(float(cols[0]))
            mx.append(float(cols[1]))
            pw.append(float(cols[2]))
        except ValueError:
            continue
        for n, v in zip(names, cols[3:7]):
            if v.lower() == "active":
                reasons.add(n)
    os.unlink(path)
    loaded = [s for s, p_ in zip(sm, pw) if p_ > 300] or sm
    return {"sm_mhz": statistics.median(loaded) if loaded else None,
            "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
            "samples": len(sm), "power_w_max": max(pw) if pw else None}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
# Algorithmic bytes of the update stage (the per-unit figures of the path's
# measurement contract): every pass writes each head's 3 new frames to sink or
# recent, K and V read and written (2 * F * D * 2 * 2 B) plus the generated
# positions (F * 3 * 8 B); a clean pass adds the middle frames (periodic heads:
# all 3; stride heads: t % 6 == 0) at the same cost, and per merge head reads
# the 3 frames' K/V (F * D * 2 * 2 B), read-modify-writes the fp32
# accumulators of the 390 patch groups (390 * D * 4 * 2 * 2 B per frame) and
# writes each completed 4-frame block's anchors (390 * D * 2 * 2 B).
FRAME_KV_RW = 2 * FSEQ * D_ * 2 * 2
FRAME_POS_W = FSEQ * 3 * 8
MERGE_GROUPS = (HG_ // 2) * (W_ // 2)


def update_algorithmic_bytes(labels, frames: int) -> float:
    """B_upd per layer-step, averaged over one video of the label matrix."""
    import numpy as np
    labels = np.asarray(labels)
    n_stride = int((labels == 1).sum())
    n_cyclic = int((labels == 2).sum())
    n_merge = int((labels == -1).sum())
    heads_layers = labels.size
    total = 0
    for blk in range(frames // FRAMES_PER_BLOCK):
        ts = range(blk * FRAMES_PER_BLOCK, (blk + 1) * FRAMES_PER_BLOCK)
        # sink / recent writes of all passes, all heads of all layers
        total += len(PASSES) * heads_layers * FRAMES_PER_BLOCK * (FRAME_KV_RW + FRAME_POS_W)
        middle = n_cyclic * FRAMES_PER_BLOCK + n_stride * sum(1 for t in ts if t % 6 == 0)
        total += middle * (FRAME_KV_RW + FRAME_POS_W)
        finals = sum(1 for t in ts if t % 4 == 3)
        total += n_merge * (FRAMES_PER_BLOCK * (FSEQ * D_ * 2 * 2 + MERGE_GROUPS * D_ * 4 * 2 * 2)
                            + finals * MERGE_GROUPS * D_ * 2 * 2)
    return total / layer_steps(frames)


def layer_steps(frames: int) -> int:
    return (frames // FRAMES_PER_BLOCK) * len(PASSES) * L_


def timed_videos(w, args, events: bool):
    """K videos back to back inside one timed region; returns (ms, per-stage
    event lists or None)."""
    import torch
    n_ls = layer_steps(args.frames)
    stage = None
    if events:
        stage = [[torch.cuda.Event(enable_timing=True) for _ in range(4)]
                 for _ in range(n_ls * args.steps)]
        cur = [0]
        w.ctx.on_stage = lambda _name: stage[cur[0]][2].record()
        hooks = (lambda i: stage[cur[0]][0].record(),
                 lambda i: stage[cur[0]][1].record(),
                 lambda i, out: (stage[cur[0]][3].record(), cur.__setitem__(0, cur[0] + 1)))
    else:
        hooks = None
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    t0.record()
    for _ in range(args.steps):
        w.reset()
        run_video(w, args.frames, hooks=hooks)
    t1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    w.ctx.on_stage = None
    return t0.elapsed_time(t1), stage


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def e2e_videos(w, args, world: int):
    """Same workload through the public API with host inputs: every layer-step
    copies its Q/K/V from pinned host memory to the device and its attention
    output back to pinned host memory, inside the timed region.  The copies go
    through pyramidkv.host_staging.HostStaging (two device slots, copy-in and
    copy-out streams), so layer-step i+1's inputs cross PCIe while layer-step
    i's kernels run."""
    import torch
    from pyramidkv.host_staging import HostStaging
    host = [tuple(x.cpu().pin_memory() for x in s) for s in w.sets]
    host_out = [torch.empty(tuple(w.sets[0][0].shape), dtype=torch.bfloat16).pin_memory()
                for _ in range(2)]
    stage = HostStaging(w.sets[0], w.device, depth=2)
    n_ls = layer_steps(args.frames)
    steps = max(1, args.e2e_steps)
    total = n_ls * steps
    cur = [0]

    def inputs(i):
        if cur[0] == 0:
            stage.put(host[0])
        if cur[0] + 1 < total:
            stage.put(host[(cur[0] + 1) % N_SETS])
        return stage.get()

    def after_attend(i, out):
        stage.done(out, host_out[cur[0] % 2])
        cur[0] += 1

    hooks = (lambda i: None, lambda i: None, after_attend)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        w.reset()
        run_video(w, args.frames, inputs=inputs, hooks=hooks)
    # the last outputs are read back: the copy-out stream joins before t1
    torch.cuda.current_stream().wait_stream(stage.copy_out)
    t1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(t0.elapsed_time(t1), world)
    per = w.sets[0][0].numel() * 2
    return {"value": world * steps * args.frames / (ms / 1e3), "unit": "latent frames/s",
            "h2d_bytes_per_step": 3 * per * n_ls, "d2h_bytes_per_step": per * n_ls,
            "steps": steps, "ms_per_step": ms / steps,
            "path": ("MegaCache.update/attend with pinned host Q/K/V in and O out per "
                     "layer-step, staged by pyramidkv.host_staging.HostStaging (copies "
                     "overlap the neighbouring layer-steps' kernels)")}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port of the reference path on the host cores
# ---------------------------------------------------------------------------
def cpu_sample(args, budget_s: float = 12.0, warm_blocks: int = 12):
    """Time one layer-step of the cache path on the CPU oracle at the cache
    size reached after `warm_blocks` blocks (36 latent frames), layer 0 of the
    same label matrix: a noisy and a clean update, the plan + pack with RoPE,
    and the fp32 attention of as many (chunk, head) segments as fit the time
    budget (scaled to all 36).  Returns (latent frames/s, detail dict)."""
    import numpy as np
    from oracle import pkv_oracle as O
    from pyramidkv import policy

    O.set_threads(os.cpu_count() or 1)    # the pack over all host cores
    labels = policy.random_labels(L_, H_, seed=args.seed, merge_fraction=args.merge_fraction)
    states, caps = policy.states_from_labels(labels[:1], "baseline")
    tables, _ = O.rope_freq_tables(D_)
    orc = O.OracleMegaCache(1, H_, D_, FSEQ, 3, 24, 4, states, caps, spatial_width=W_,
                            sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18,
                            sink_time_clamp_max=21, freq_tables=tables)
    rng = np.random.default_rng(args.seed)
    shape = (1, FRAMES_PER_BLOCK * FSEQ, H_, D_)
    k, v, q = (O.f32_to_bf16(rng.standard_normal(shape).astype(np.float32)) for _ in range(3))
    for blk in range(warm_blocks):
        orc.update(0, k, v, blk * FRAMES_PER_BLOCK * FSEQ, "clean")
    start = warm_blocks * FRAMES_PER_BLOCK * FSEQ
    t = time.perf_counter()
    orc.update(0, k, v, start, "noisy")
    orc.update(0, k, v, start, "clean")
    t_update = (time.perf_counter() - t) / 2
    t = time.perf_counter()
    pk = orc.plan_and_pack(0, start, FRAMES_PER_BLOCK)
    t_pack = time.perf_counter() - t
    kf, vf, cu = O.bf16_to_f32(pk["k"]), O.bf16_to_f32(pk["v"]), pk["cu"]
    qf = O.bf16_to_f32(q[0])
    n_seg = FRAMES_PER_BLOCK * H_
    done, t_attn = 0, 0.0
    for i in range(n_seg):
        c, h = divmod(i, H_)
        t = time.perf_counter()
        O.attention_fp32(qf[c * FSEQ:(c + 1) * FSEQ, h:h + 1], kf[cu[i]:cu[i + 1]],
                         vf[cu[i]:cu[i + 1]], np.array([0, cu[i + 1] - cu[i]], np.int32), 1, 1,
                         FSEQ)
        t_attn += time.perf_counter() - t
        done += 1
        if t_update + t_pack + t_attn > budget_s:
            break
    t_attn_all = t_attn * n_seg / done
    t_ls = t_update + t_pack + t_attn_all
    fps = args.frames / (layer_steps(args.frames) * t_ls)
    return fps, {"us_per_layer_step": t_ls * 1e6, "update_s": t_update, "plan_pack_s": t_pack,
                 "attention_s": t_attn_all, "segments_timed": done, "segments": n_seg,
                 "kv_tokens": int(pk["total"])}


def cpu_baseline_json(fps, detail, cores):
    return {"value": fps, "unit": "latent frames/s", "cores": cores, "kind": "port",
            "sample": ("one layer-step of layer 0 at the cache size after 36 latent frames "
                       f"({detail['kv_tokens']} packed K/V tokens): noisy+clean update, plan+pack "
                       f"with RoPE, fp32 attention of {detail['segments_timed']}/"
                       f"{detail['segments']} (chunk, head) segments scaled to all; "
                       "C restatement (pack OpenMP over segments) and numpy BLAS attention "
                       "on all cores; "
                       "scaled to 6000 layer-steps per 120-frame video"),
            "us_per_layer_step": detail["us_per_layer_step"]}


def host_threads():
    """All host cores for the CPU legs: torchrun sets OMP_NUM_THREADS=1 when it
    starts more than one process, which would leave numpy's BLAS on one
    thread; the limit is lifted for the BLAS pools here and for the C pack by
    the oracle's own thread count.  Returns (threads asked, BLAS pools' threads)."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info, threadpool_limits
        threadpool_limits(limits=n)
        used = sorted({int(p.get("num_threads", 0)) for p in threadpool_info()})
    except ImportError:  # pragma: no cover
        used = []
    return n, used


def run_reference(args, rank: int):
    if rank != 0:
        return
    cores, blas_threads = host_threads()
    fps_all = []
    detail = None
    for i in range(args.warmup + args.steps):
        fps, detail = cpu_sample(args, budget_s=4.0)
        if i >= args.warmup:
            fps_all.append(fps)
    fps = statistics.mean(fps_all)
    line = {"impl": "reference", "metric": METRIC, "value": fps, "unit": "latent frames/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": args.frames / fps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args),
            "cpu_baseline": cpu_baseline_json(fps, detail, cores),
            "e2e": {"value": fps, "unit": "latent frames/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "sampled": True, "layer_steps_timed_per_step": 1,
            "threads": {"asked": cores, "blas_pools": blas_threads,
                        "c_pack": cores},
            "parts": {"update (routing, state machine, frame copies, merge)":
                      "port: oracle/pkv_oracle.c + oracle/pkv_oracle.py restating "
                      "_mega_cache.py:136-414 and its kernels",
                      "plan + pack with RoPE": "port: oracle/pkv_oracle.c restating "
                      "mega_plan.cc and pyramidkv_pack.cu",
                      "attention": "numpy fp32 BLAS standing in for flash_attn_varlen_func"},
            "note": ("each step times one layer-step of the cache path at the 36-frame cache "
                     "size (update, plan + pack, attention of the 36 (chunk, head) segments, "
                     "scaled from the segments that fit a 4 s budget) and scales it to the "
                     "6000 layer-steps of a 120-frame video; the value is the host's, the same "
                     "at every GPU count.  The reference's own code for this path is CUDA "
                     "kernels plus a host planner that needs a CUDA device; its Python parts "
                     "cannot travel to the GPU box, so timed is the oracle port of that path")}
    print(json.dumps(line), flush=True)


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, \
            "fallback"


# ---------------------------------------------------------------------------
# head-parallel: one video over a group of n ranks (heads split, NCCL exchange)
# ---------------------------------------------------------------------------
class HPWorkload:
    """One group's video: this rank's heads of the 30 layers behind
    HeadParallelMegaCache, and this rank's token shard of the rotating
    Q/K/V sets (the same seeded video on every rank of the group)."""

    @staticmethod
    def build(device, seed: int, group, merge_fraction=None, exchange="peer"):
        import torch
        import torch.distributed as dist
        from pyramidkv import head_parallel as hp, policy

        w = HPWorkload.__new__(HPWorkload)
        w.device = device
        w.n = dist.get_world_size(group)
        r = dist.get_rank(group)
        labels = policy.random_labels(L_, H_, seed=seed, merge_fraction=merge_fraction)
        comps = policy.compositions_from_labels(labels, "baseline")
        w.caches = hp.build_head_parallel_caches(
            L_, H_, D_, FSEQ, 3, 24, 4, comps, group=group, exchange=exchange,
            block_tokens=FRAMES_PER_BLOCK * FSEQ, max_attend_chunks=8,
            device=str(device), sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18,
            sink_time_clamp_max=21, spatial_width=W_, spatial_height=HG_, freqs=rope_table(D_))
        w.ctx = w.caches[0].local.ctx
        w.init_states = w.ctx.states_bytes.clone()
        w.ctx.token_counter = torch.zeros(1, dtype=torch.int64, device=device)
        t0, t1 = hp.token_range(r, w.n, FRAMES_PER_BLOCK * FSEQ)
        g = torch.Generator(device=device).manual_seed(1000 + seed)
        shape = (1, FRAMES_PER_BLOCK * FSEQ, H_, D_)
        w.sets = []
        for _ in range(N_SETS):
            full = [torch.randn(shape, generator=g, device=device, dtype=torch.bfloat16)
                    for _ in range(3)]
            w.sets.append(tuple(x[:, t0:t1].contiguous() for x in full))
        return w

    def reset(self):
        Workload.reset(self)


def run_video_hp(w, frames: int, inputs=None, hooks=None):
    """One head-parallel video: per layer-step ``step(q, k, v)`` (Q/K/V in one
    exchange, update + attend on this rank's heads, output exchanged back)."""
    i = 0
    for blk in range(frames // FRAMES_PER_BLOCK):
        start = blk * FRAMES_PER_BLOCK * FSEQ
        for mode in PASSES:
            for layer in range(L_):
                q, k, v = inputs(i) if inputs is not None else w.sets[i % N_SETS]
                if hooks:
                    hooks[0](i)
                out = w.caches[layer].step(q, k, v, start, cache_update_mode=mode)
                if hooks:
                    hooks[2](i, out)
                i += 1
    return i


def head_parallel_measure(args, rank: int, world: int, local: int, n: int, steps: int,
                          warmup: int, with_e2e: bool):
    """world/n videos, each split by heads over n ranks; returns the measured
    dict on every rank (rank 0 prints it)."""
    import torch
    import torch.distributed as dist
    if H_ % n or world % n:
        raise ValueError(f"head-parallel over {n} ranks needs n | {H_} and n | {world}")
    groups = [dist.new_group(list(range(g * n, (g + 1) * n))) for g in range(world // n)]
    gi = rank // n
    dev = torch.device("cuda", local)
    w = HPWorkload.build(dev, seed=args.seed + gi, group=groups[gi],
                         merge_fraction=args.merge_fraction, exchange=args.hp_exchange)
    for _ in range(warmup):
        w.reset()
        run_video_hp(w, args.frames)
    torch.cuda.synchronize()
    w.ctx.check_status()
    w.ctx.token_counter.zero_()
    n_ls = layer_steps(args.frames)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n_ls * steps)]
    cur = [0]

    def stage(name):
        ev[cur[0]][1 if name == "exchanged_in" else 2].record()
    for c in w.caches:
        c.on_stage = stage
    hooks = (lambda i: ev[cur[0]][0].record(), None,
             lambda i, out: (ev[cur[0]][3].record(), cur.__setitem__(0, cur[0] + 1)))
    dist.barrier()
    torch.cuda.synchronize()
    clk = clocks_start(local)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        w.reset()
        run_video_hp(w, args.frames, hooks=hooks)
    t1.record()
    torch.cuda.synchronize()
    clocks = clocks_stop(clk)
    for c in w.caches:
        c.on_stage = None
    ms = max_over_ranks(t0.elapsed_time(t1), world)
    tot = n_ls * steps
    ex_in = sum(e[0].elapsed_time(e[1]) for e in ev) * 1e3 / tot
    cache = sum(e[1].elapsed_time(e[2]) for e in ev) * 1e3 / tot
    ex_out = sum(e[2].elapsed_time(e[3]) for e in ev) * 1e3 / tot
    shard = w.sets[0][0]
    lt = shard.shape[1]
    bytes_in = 3 * shard.numel() * 2 * (n - 1) // n   # Q/K/V leaving this rank
    bytes_out = shard.numel() * 2 * (n - 1) // n
    res = {"n": n, "groups": world // n, "videos": world // n, "steps": steps,
           "warmup": warmup, "ms_per_video": ms / steps,
           "value": (world // n) * steps * args.frames / (ms / 1e3), "unit": "latent frames/s",
           "scaling": "strong within a group (one video's heads over n GPUs)",
           "us_per_layer_step": ms * 1e3 / tot,
           "breakdown_us_per_layer_step_rank": {
               "exchange_in (pack + transfer of Q/K/V)": ex_in,
               "cache (update + plan/pack + attention)": cache,
               "exchange_out (transfer + scatter of O)": ex_out},
           "heads_per_rank": H_ // n, "tokens_per_rank": lt,
           "nvlink_bytes_per_layer_step_rank": {"qkv": bytes_in, "out": bytes_out},
           "collective": ("NVLink peer stores into symmetric-memory buffers (pack kernel writes "
                          "each rank's Q/K/V share into its receive buffer; the output pass "
                          "writes each token owner's rows at this rank's heads), one barrier per "
                          "exchange" if args.hp_exchange == "peer" else
                          "torch.distributed all_to_all_single (NCCL), Q/K/V together, O back"),
           "clocks": clocks}
    if with_e2e:
        from pyramidkv.host_staging import HostStaging
        host = [tuple(x.cpu().pin_memory() for x in s_) for s_ in w.sets]
        host_out = [torch.empty(tuple(shard.shape), dtype=torch.bfloat16).pin_memory()
                    for _ in range(2)]
        st = HostStaging(w.sets[0], dev, depth=2)
        pos = [0]

        def inputs(i):
            if pos[0] == 0:
                st.put(host[0])
            if pos[0] + 1 < n_ls:
                st.put(host[(pos[0] + 1) % N_SETS])
            return st.get()

        def after(i, out):
            st.done(out, host_out[pos[0] % 2])
            pos[0] += 1
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        w.reset()
        run_video_hp(w, args.frames, inputs=inputs, hooks=(lambda i: None, None, after))
        torch.cuda.current_stream().wait_stream(st.copy_out)
        e1.record()
        torch.cuda.synchronize()
        ems = max_over_ranks(e0.elapsed_time(e1), world)
        res["e2e"] = {"value": (world // n) * args.frames / (ems / 1e3), "unit": "latent frames/s",
                      "h2d_bytes_per_step": 3 * shard.numel() * 2 * n_ls * world,
                      "d2h_bytes_per_step": shard.numel() * 2 * n_ls * world,
                      "ms_per_step": ems,
                      "path": "HeadParallelMegaCache.step with each rank's pinned host token "
                              "shard of Q/K/V in and O out per layer-step (HostStaging)"}
    res["device_status"] = w.ctx.check_status()
    del w
    torch.cuda.empty_cache()
    return res


def run_head_parallel_line(args, rank: int, world: int, local: int):
    """``--head-parallel n``: the line measures world/n head-parallel videos."""
    n = args.head_parallel
    res = head_parallel_measure(args, rank, world, local, n, args.steps, args.warmup,
                                with_e2e=not args.no_e2e)
    if rank != 0:
        return
    line = {"metric": METRIC, "value": res["value"], "unit": "latent frames/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["ms_per_video"], "higher_is_better": True,
            "scaling": "strong" if world == n else "weak", "vs_baseline": None,
            "dtype": "bf16",
            "data": ("synthetic: seeded N(0,1) bf16 Q/K/V per layer-step, seeded random [30,12] "
                     "label matrix, model RoPE table; no checkpoint (cache path only)"),
            "config": dict(workload_config(args), parallelism=f"head-parallel x{n}, "
                           f"{world // n} video(s)"),
            "us_per_layer_step": res["us_per_layer_step"], "head_parallel": res,
            "e2e": res.get("e2e"), "clocks": res["clocks"],
            # per layer-step: exchange in, route + copy, attend, exchange out
            "gpu_launches": layer_steps(args.frames) * args.steps * (4 + attend_launches()),
            "device_status": res["device_status"]}
    print(json.dumps(line), flush=True)


def dit_measure(args, local: int, cache_us_per_layer_step: float):
    """configs[1] as defined: latent frames/s = frames / DiT wall time.  The
    random-init causal Wan2.1-T2V-1.3B DiT (pyramid-forcing_b200/causal_dit)
    generates one video of `--frames` latent frames (4 denoising steps + the
    clean pass per 3-frame block) from seeded N(0,1) noise [1, 16, F, 60, 104]
    and a seeded N(0,1) text context [1, 512, 4096] (text encoder and VAE
    excluded), its self-attention on this library's MegaCache, cross-attention
    on its ragged attention kernel, GEMMs on cuBLAS.  One 6-frame video warms
    up; one full video is timed with CUDA events."""
    import torch
    from causal_dit import CausalWanDiT, WanConfig, generate_video
    from pyramidkv import _mega_cache, policy
    dev = torch.device("cuda", local)
    cfg = WanConfig()
    model = CausalWanDiT(cfg, dev, seed=args.seed)
    labels = policy.random_labels(L_, H_, seed=args.seed, merge_fraction=args.merge_fraction)
    caches = _mega_cache.build_mega_caches(
        L_, H_, D_, FSEQ, 3, 24, 4, policy.compositions_from_labels(labels, "baseline"),
        max_attend_chunks=8, device=str(dev), sink_time_mapping_mode="window_clamp",
        sink_time_clamp_min=18, sink_time_clamp_max=21, spatial_width=W_, spatial_height=HG_,
        freqs=model.freqs)
    ctx = caches[0].ctx
    init_states = ctx.states_bytes.clone()
    g = torch.Generator(device=dev).manual_seed(2000 + args.seed)
    text = torch.randn(1, cfg.text_len, cfg.text_dim, generator=g, device=dev)
    noise = torch.randn(1, cfg.in_dim, args.frames, 2 * HG_, 2 * W_, generator=g, device=dev,
                        dtype=torch.bfloat16)

    def reset():
        ctx.mgr.reset()
        ctx.states_bytes.copy_(init_states)
        if ctx.committed_vc is not None:
            ctx.committed_vc.zero_()
    reset()
    generate_video(model, caches, noise[:, :, :6], text, generator=g)
    torch.cuda.synchronize()
    reset()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    out = generate_video(model, caches, noise, text, generator=g)
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    status = ctx.check_status()
    n_ls = layer_steps(args.frames)
    res = {"value": args.frames / (ms / 1e3), "unit": "latent frames/s",
           "ms_per_video": ms, "us_per_layer_step": ms * 1e3 / n_ls,
           "cache_path_us_per_layer_step": cache_us_per_layer_step,
           "cache_path_share": cache_us_per_layer_step / (ms * 1e3 / n_ls),
           "finite": bool(torch.isfinite(out.float()).all().item()),
           "device_status": status,
           "workload": ("configs[1]: random-init causal Wan2.1-T2V-1.3B DiT (30 layers, dim 1536, "
                        "12x128 heads, FFN 8960, patch 1x2x2), %d latent frames of 16x60x104 in "
                        "3-frame blocks, timesteps 1000/750/500/250 + clean pass, seeded N(0,1) "
                        "noise and [1,512,4096] text context; T5 and VAE excluded" % args.frames),
           "videos_timed": 1, "warmup": "one 6-frame video"}
    del model, caches
    torch.cuda.empty_cache()
    return res


def run_ours(args, rank: int, world: int, local: int):
    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    w = Workload.build(dev, seed=args.seed + rank, merge_fraction=args.merge_fraction)
    for _ in range(args.warmup):
        w.reset()
        run_video(w, args.frames)
    torch.cuda.synchronize()
    if w.ctx.check_status() != 0:
        raise RuntimeError("device status set during warm-up")
    w.ctx.token_counter.zero_()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    clk = clocks_start(local)
    ms, stage = timed_videos(w, args, events=True)
    clocks = clocks_stop(clk)
    ms_max = max_over_ranks(ms, world)
    tokens = int(w.ctx.token_counter.item())
    n_ls = layer_steps(args.frames)
    n_total = n_ls * args.steps
    upd = sum(e[0].elapsed_time(e[1]) for e in stage)
    pack = sum(e[1].elapsed_time(e[2]) for e in stage)
    attn = sum(e[2].elapsed_time(e[3]) for e in stage)
    status = w.ctx.check_status()
    peaks, peak_kind = measured_peaks()
    attn_flops = 4.0 * FSEQ * D_ * tokens
    achieved = attn_flops / (attn / 1e3) / 1e12
    peak = float(peaks["bf16_tflops_sustained"])
    pack_bytes = tokens * (2 * D_ * 2 * 2 + 3 * 8 * 2)
    has_merge = bool(w.ctx.has_merge_head)
    clean_steps = n_ls // len(PASSES)
    launches_per_video = n_ls * (2 + attend_launches()) + (clean_steps if has_merge else 0)
    e2e = None if args.no_e2e else e2e_videos(w, args, world)
    fps = world * args.steps * args.frames / (ms_max / 1e3)
    line = {
        "metric": METRIC, "value": fps, "unit": "latent frames/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": ("synthetic: seeded N(0,1) bf16 Q/K/V per layer-step, seeded random [30,12] "
                 "label matrix, model RoPE table; no checkpoint (cache path only)"),
        "config": workload_config(args),
        "us_per_layer_step": ms_max * 1e3 / n_total,
        "breakdown_us_per_layer_step": {"update": upd * 1e3 / n_total,
                                        "plan_pack": pack * 1e3 / n_total,
                                        "attention": attn * 1e3 / n_total},
        "roofline": {"kernel": "attn_tc2_kernel (ragged attention, tcgen05/TMEM, "
                               "SM-balanced persistent schedule)",
                     "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak,
                     "peak_source": f"{peak_kind} bf16_tflops_sustained (kernel timed inside a "
                                    "long step)",
                     "frac_of_burst": achieved / float(peaks["bf16_tflops"]),
                     "flops_per_launch": attn_flops / n_total,
                     # DRAM bytes per launch: one ncu capture of the kernel case
                     # of the kernel case (bench.py --kernel-case attn), scaled by work
                     "traffic": ATTN_DRAM_BYTES_PER_FLOP * attn_flops / n_total,
                     "traffic_source": "ncu dram__bytes_read+write of the kernel case, balanced "
                                       "schedule (505.0 MB / 0.492 TFLOP), scaled to this "
                                       "launch"},
        "pack_roofline": {"bound": "hbm", "unit": "GB/s",
                          "achieved": pack_bytes / (pack / 1e3) / 1e9,
                          "peak": float(peaks["hbm_gbs"]),
                          "frac": pack_bytes / (pack / 1e3) / 1e9 / float(peaks["hbm_gbs"]),
                          "bytes_per_launch": pack_bytes / n_total},
        "update_roofline": {"bound": "hbm", "unit": "GB/s",
                            "achieved": update_algorithmic_bytes(w.labels, args.frames) /
                            (upd / n_total / 1e3) / 1e9,
                            "peak": float(peaks["hbm_gbs"]),
                            "frac": update_algorithmic_bytes(w.labels, args.frames) /
                            (upd / n_total / 1e3) / 1e9 / float(peaks["hbm_gbs"]),
                            "bytes_per_layer_step": update_algorithmic_bytes(w.labels,
                                                                             args.frames),
                            "kernels": "route_kernel + copy_kernel (+ merge_grid_kernel on "
                                       "clean passes with merge heads)"},
        "kv_tokens_per_layer_step": tokens / n_total,
        "e2e": e2e,
        "gpu_launches": launches_per_video * args.steps,
        "clocks": clocks,
        "device_status": status,
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        host_threads()
        fps_cpu, detail = cpu_sample(args)
        line["cpu_baseline"] = cpu_baseline_json(fps_cpu, detail, os.cpu_count())
    if world == 1 and not args.no_dit:
        del w
        torch.cuda.empty_cache()
        line["dit"] = dit_measure(args, local, line["us_per_layer_step"])
    if world > 1 and args.hp_steps > 0:
        n = world if H_ % world == 0 else (4 if world % 4 == 0 else 0)
        if n:
            del w
            torch.cuda.empty_cache()
            line["head_parallel"] = head_parallel_measure(
                args, rank, world, local, n, args.hp_steps, 1, with_e2e=False)
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_attn_c4(args):
    """the ragged-attention microbench.  Per video and layer, each
    of the 12 heads attends 4680 queries (3 chunks of 1560) to a K/V length
    drawn uniformly from 3..21 frames of 1560 tokens (seed 0, a fresh draw per
    layer); a launch covers one layer of `--batch` videos (batch x 12
    segments of 4680 query rows), K/V ~ N(0, 1) bf16 standing for RoPE'd
    keys.  30 layers are timed back to back (CUDA events per launch, after
    warm-up), through the SM-balanced path MegaCache.attend uses."""
    import torch
    from pyramidkv import _ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ops = _ops.ops()
    B, rows = args.batch, FRAMES_PER_BLOCK * FSEQ
    g = torch.Generator(device="cpu").manual_seed(args.seed)
    frames = torch.randint(3, 22, (L_, B * H_), generator=g)      # per layer, per (video, head)
    lens = frames * FSEQ
    cus = []
    for l in range(L_):
        cu = torch.zeros(B * H_ + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(lens[l], 0).int()
        cus.append(cu.to(dev))
    T = int(lens.sum(1).max())
    q = torch.randn(B * rows, H_, D_, generator=g).to(dev, torch.bfloat16)
    k = torch.randn(T, D_, generator=g).to(dev, torch.bfloat16)
    v = torch.randn(T, D_, generator=g).to(dev, torch.bfloat16)
    ws = torch.zeros(int(ops.pkv_attention_ws_bytes(B, H_, rows)), dtype=torch.uint8, device=dev)
    # video b's queries are rows [b*rows, (b+1)*rows) of every head: one
    # "chunk" per video with rows_per_chunk = 4680, segment (b, h) = its K/V
    run = lambda l: ops.pkv_attention_ws(q, k, v, cus[l], B, rows, D_ ** -0.5, ws)  # noqa
    for _ in range(3):
        for l in range(L_):
            run(l)
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(L_)]
    for l in range(L_):
        ev[l][0].record()
        run(l)
        ev[l][1].record()
    torch.cuda.synchronize()
    ms = [e[0].elapsed_time(e[1]) for e in ev]
    flops = [4.0 * rows * D_ * float(lens[l].sum()) for l in range(L_)]
    peaks, kind = measured_peaks()
    rate = sum(flops) / (sum(ms) / 1e3) / 1e12
    print(json.dumps({
        "kernel_case": "attn-c4", "batch": B, "layers": L_,
        "us_per_layer": sum(ms) * 1e3 / L_, "tflops": rate,
        "frac_of_sustained": rate / float(peaks["bf16_tflops_sustained"]),
        "frac_of_burst": rate / float(peaks["bf16_tflops"]), "peak_source": kind,
        "kv_frames_mean": float(frames.float().mean()),
        "flop_per_layer": sum(flops) / L_,
        "workload": "configs[3]: Q 4680/head, 12 heads, Lk ~ U{3..21} frames x 1560, "
                    "30 layers, bf16, N(0,1) K/V"}), flush=True)


def attend_launches() -> int:
    """Launches of one MegaCache.attend at the C2 shape: the pack that plans
    for itself and the attention, or planner + pack + attention when
    PKV_FUSED_PLAN_PACK=0 keeps the planner a launch of its own."""
    return 3 if os.environ.get("PKV_FUSED_PLAN_PACK", "1").startswith("0") else 2


def run_kernel_case(args):
    """One kernel on inputs shaped like the C2 steady state: 3 chunks x 12 heads
    of 1560 queries over per-head KV of 8-14 frames (the plan's mix of sink,
    recent, middle frames and 390-token merge anchors), ~0.3-0.5 GB on the
    device.  Prints per-launch time (CUDA events) and the work per launch."""
    import torch
    from pyramidkv import _ops, policy
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device="cpu").manual_seed(args.seed)
    C = FRAMES_PER_BLOCK
    Hk = args.kernel_heads if args.kernel_case in ("attn", "attn-plain") else H_
    frames = torch.randint(8, 15, (C * Hk,), generator=g)
    lens = frames * FSEQ + (torch.rand(C * Hk, generator=g) < 0.3).long() * 390
    cu = torch.zeros(C * Hk + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0).int()
    T = int(cu[-1])
    ops = _ops.ops()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    if args.kernel_case in ("attn", "attn-plain"):
        # attn: the SM-balanced path MegaCache.attend runs (workspace given);
        # attn-plain: one CTA per (segment, query-tile pair), no workspace
        q = torch.randn(1, C * FSEQ, Hk, D_, generator=g).to(dev, torch.bfloat16)
        k = torch.randn(T, D_, generator=g).to(dev, torch.bfloat16)
        v = torch.randn(T, D_, generator=g).to(dev, torch.bfloat16)
        cud = cu.to(dev)
        if args.kernel_case == "attn":
            ws = torch.zeros(int(ops.pkv_attention_ws_bytes(C, Hk, FSEQ)), dtype=torch.uint8,
                             device=dev)
            run = lambda: ops.pkv_attention_ws(q[0], k, v, cud, C, FSEQ, D_ ** -0.5, ws)  # noqa
        else:
            run = lambda: ops.pkv_attention(q[0], k, v, cud, C, FSEQ, D_ ** -0.5)  # noqa: E731
        work, unit = 4.0 * FSEQ * D_ * T, "FLOP"
    elif args.kernel_case == "attn-d64":
        # the CUDA-core kernel (head_dim other than 128): 3 chunks x 4 heads of
        # 1560 queries over 2-4 frames each, head_dim 64
        Hs, Ds = 4, 64
        lens_s = (torch.randint(2, 5, (C * Hs,), generator=g) * FSEQ)
        cu_s = torch.zeros(C * Hs + 1, dtype=torch.int32)
        cu_s[1:] = torch.cumsum(lens_s, 0).int()
        Ts = int(cu_s[-1])
        q = torch.randn(C * FSEQ, Hs, Ds, generator=g).to(dev, torch.bfloat16)
        k = torch.randn(Ts, Ds, generator=g).to(dev, torch.bfloat16)
        v = torch.randn(Ts, Ds, generator=g).to(dev, torch.bfloat16)
        cud = cu_s.to(dev)
        run = lambda: ops.pkv_attention(q, k, v, cud, C, FSEQ, Ds ** -0.5)  # noqa: E731
        work, unit = 4.0 * FSEQ * Ds * Ts, "FLOP"
    elif args.kernel_case == "rope-q":
        # the model's query RoPE of one block: [4680, 12, 128] bf16 at frame 30
        from pyramidkv.rope import causal_rope_apply
        x = torch.randn(1, C * FSEQ, H_, D_, generator=g).to(dev, torch.bfloat16)
        freqs = rope_table(D_).to(dev)
        run = lambda: causal_rope_apply(x, None, freqs, start_frame=30,  # noqa: E731
                                        grid_int=((C, HG_, W_),))
        work, unit = 2 * x.numel() * 2, "B"
    elif args.kernel_case == "chunk-copy":
        # the head-parallel pack of one rank's token shard (x2): Q, K, V
        # [2340, 12, 128] into the by-destination send layout, in this GPU's memory
        n = 2
        xs = [torch.randn(1, C * FSEQ // n, H_, D_, generator=g).to(dev, torch.bfloat16)
              for _ in range(3)]
        lt, hl = C * FSEQ // n, H_ // n
        send = torch.empty(n, lt, 3, hl, D_, device=dev, dtype=torch.bfloat16)
        run = lambda: ops.pkv_chunk_copy(xs, [x.stride(1) for x in xs],  # noqa: E731
                                         [hl * x.stride(2) for x in xs], send, 3 * hl * D_,
                                         lt * 3 * hl * D_, hl * D_, lt, n, hl * D_)
        work, unit = 2 * 3 * xs[0].numel() * 2, "B"
    elif args.kernel_case == "update":
        # one layer with a third of its heads merge heads, after 30 blocks; a
        # run is the noisy and the clean update of the next block (route, copy
        # and, on the clean pass, merge kernels)
        from pyramidkv import _mega_cache
        labels = policy.random_labels(1, H_, seed=args.seed, merge_fraction=1.0 / 3.0)
        caches = _mega_cache.build_mega_caches(
            1, H_, D_, FSEQ, 3, 24, 4, policy.compositions_from_labels(labels),
            device="cuda:0", sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18,
            sink_time_clamp_max=21, spatial_width=W_, spatial_height=HG_, freqs=rope_table(D_))
        c = caches[0]
        shape = (1, C * FSEQ, H_, D_)
        kk = torch.randn(shape, generator=g).to(dev, torch.bfloat16)
        vv = torch.randn(shape, generator=g).to(dev, torch.bfloat16)
        for blk in range(30):
            c.update(kk, vv, blk * C * FSEQ, cache_update_mode="clean")
        nxt = [30]

        def run():
            start = nxt[0] * C * FSEQ
            nxt[0] += 1
            c.update(kk, vv, start, cache_update_mode="noisy")
            c.update(kk, vv, start, cache_update_mode="clean")
        work, unit = 2 * 2 * 2 * kk.numel() * 2, "B"   # K and V of 2 passes, read + written
    else:
        from pyramidkv import _mega_cache
        labels = policy.random_labels(1, H_, seed=args.seed)
        caches = _mega_cache.build_mega_caches(
            1, H_, D_, FSEQ, 3, 24, 4, policy.compositions_from_labels(labels),
            device="cuda:0", sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18,
            sink_time_clamp_max=21, spatial_width=W_, spatial_height=HG_, freqs=rope_table(D_))
        c = caches[0]
        shape = (1, C * FSEQ, H_, D_)
        kk = torch.randn(shape, generator=g).to(dev, torch.bfloat16)
        for blk in range(30):           # reach a steady-state cache
            c.update(kk, kk, blk * C * FSEQ, cache_update_mode="clean")
        ctx = c.ctx
        start = 30 * C * FSEQ
        counter = torch.zeros(1, dtype=torch.int64, device=dev)
        ft, fy, fx = ctx.freq_parts_flat
        run = lambda: ops.pkv_attend_pack(ctx.mgr, c.states_bytes_for_layer, 0, C * FSEQ,  # noqa
                                          start // FSEQ, 1, 18, 21, 0, ft, fy, fx, counter)
        run()
        torch.cuda.synchronize()
        tokens = int(counter.item())
        work, unit = tokens * (2 * D_ * 2 * 2 + 3 * 8 * 2), "B"
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.kernel_iters):
        # the GPU sleeps while the host enqueues the call, so the events time
        # the device work and not the host's launch overhead
        torch.cuda._sleep(1_000_000)
        ev[0].record()
        run()
        ev[1].record()
        torch.cuda.synchronize()
        times.append(ev[0].elapsed_time(ev[1]))
    ms = statistics.median(times)
    rate = work / (ms / 1e3) / 1e12
    print(json.dumps({"kernel_case": args.kernel_case, "ms": ms, "work": work, "unit": unit,
                      "rate": rate, "rate_unit": "T" + unit + "/s"}), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.kernel_case == "attn-c4":
        run_attn_c4(args)
        return
    if args.kernel_case:
        run_kernel_case(args)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    try:
        if args.head_parallel:
            run_head_parallel_line(args, rank, world, local)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
