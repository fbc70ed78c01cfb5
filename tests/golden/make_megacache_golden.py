"""Golden digests of the reference's own ``MegaCache.update`` at the benchmark's
full layer size, for ``tests/test_gpu_megacache_reference.py``.

Run in a container where the reference checkout is present:

    python tests/golden/make_megacache_golden.py --reference /path/to/Pyramid-Forcing

It drives the reference's ``pyramidkv/_mega_cache.py`` -- its ``MegaCache``
class and ``MegaCacheCtx`` as they are, with its ``update`` (:136-414: the
committed-snapshot restore, the per-head sink / recent routing with FIFO
shift, the descriptor split between pool writes and merge accumulation, the
global middle-slot arithmetic and the commit) and its
``_mega_state_ops.mega_merge_accum_cuda`` wrapper -- on CPU tensors.  Only
the three CUDA kernels it launches (``mega_state_update``,
``pyramidkv_update``, ``mega_merge_accum``) are stood in for by the C oracle
(oracle/pkv_oracle.c), which the GPU tests pin bit for bit to those kernels
built from the reference's sources (tests/test_gpu_reference.py); the manager
is a stand-in object exposing the reference's pool shapes
(pyramidkv_manager.cc:80-137) over the oracle's numpy arrays.  The label ->
state mapping is the reference's factory (``factory.build_compositions`` +
``_composition_to_perhead_state`` + ``pack_states``, BASELINE routing, the
settings of tests/golden/compositions.npz).

Workload (BASELINE configs[0] layer shape): one layer, 12 heads x 128,
1560-token frames (30 x 52 grid), pools 3 / 24 / 4 frames, 20 blocks of 3
frames, each block a noisy then a clean update with fresh seeded N(0, 1) bf16
K/V (numpy, reproducible on any machine).  Two label rows: ``c1`` (uniform
over {-1, 1, 2}, seed 0) and ``merge`` (half the heads merge, seed 1: 15 merge
blocks per head, so the merge FIFO evicts, quirks Q2/Q3).  After every call
the generator stores row digests (tests/golden/megacache_digest.py) of every
pool, the valid counts, the per-head state bytes and the committed snapshot;
after the last block, the oracle's plan + RoPE pack (pinned to the
reference's planner and pack kernels) of that state: cu_seqlens_k and per
segment digests of the packed K, V and positions.

Output: ``megacache_c1.npz`` next to this script.
"""
from __future__ import annotations

import argparse
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

L, H, D, W, HG = 1, 12, 128, 52, 30
FSEQ = W * HG
F = 3
BLOCKS = 20
SINK, MIDDLE, RECENT = 3, 24, 4
CONFIGS = {"c1": dict(seed=0, merge_fraction=None), "merge": dict(seed=1, merge_fraction=0.5)}
PASSES = ("noisy", "clean")


def inputs(seed: int):
    """Seeded bf16 K/V per (block, pass) and the final block's Q (uint16 bits)."""
    from oracle import pkv_oracle as O
    rng = np.random.default_rng(7000 + seed)
    shape = (1, F * FSEQ, H, D)
    kv = [[tuple(O.f32_to_bf16(rng.standard_normal(shape, np.float32)) for _ in range(2))
           for _ in PASSES] for _ in range(BLOCKS)]
    q = O.f32_to_bf16(rng.standard_normal(shape, np.float32))
    return kv, q


def labels_for(cfg) -> np.ndarray:
    rng = np.random.default_rng(cfg["seed"])
    if cfg["merge_fraction"] is None:
        return rng.choice(np.asarray([-1, 1, 2]), size=(L, H))
    n_merge = int(round(H * cfg["merge_fraction"]))
    rest = H - n_merge
    flat = np.array([-1] * n_merge + [1] * (rest // 2) + [2] * (rest - rest // 2))
    rng.shuffle(flat)
    return flat.reshape(L, H)


def reference_states(factory, mega_cache, ops, labels):
    """State bytes and sink caps from the reference's factory (BASELINE routing)."""
    common = dict(
        cyclic_enabled=True, cyclic_period=6, cyclic_bucket_cap=4,
        stride_enabled=True, stride_interval=6, stride_capacity=4,
        merge_enabled=True, merge_patch_size=2, merge_capacity=4,
        label_sink_frames_map={"-1": 1, "1": 3, "2": 3},
        label_recent_frames_map={"-1": 4, "1": 4, "2": 4},
        label_stride_interval_map={"1": 6},
        label_merge_patch_size_map={"-1": 2, "2": 2},
        label_merge_capacity_map={"-1": 4, "2": 4},
        cyclic_osc_only=False,
        label_phase_bucket_map={"2": 4, "-1": 0, "1": 0},
        label_stride_enabled_map={"1": True, "2": False},
        label_merge_enabled_map={"-1": True, "1": False, "2": False},
    )
    with tempfile.TemporaryDirectory() as td:
        csv = os.path.join(td, "labels.csv")
        with open(csv, "w") as f:
            for row in labels:
                f.write(",".join(str(int(x)) for x in row) + "\n")
        comps = factory.build_compositions(L, H, [[32760] * H] * L, csv, **common)
    per = [mega_cache._composition_to_perhead_state(c) for c in comps[0]]
    states = ops.pack_states(per).view(np.uint8).reshape(1, -1).copy()
    caps = np.array([[s.sink_capacity for s in per]], np.int64)
    any_merge = any(s.kind == 4 for s in per)
    return states, caps, any_merge


class StandInManager:
    """The accessors of the reference's PyramidKVCacheManager that
    MegaCache.update and mega_merge_accum_cuda call, as CPU torch views of an
    OracleMegaCache's numpy pools (shapes of pyramidkv_manager.cc:80-137)."""

    def __init__(self, orc):
        import torch
        self.orc = orc

        def bf(a):
            return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
        t = torch.from_numpy
        self._t = {
            "sink_k_pool": bf(orc.sink_k), "sink_v_pool": bf(orc.sink_v),
            "sink_pos_pool": t(orc.sink_pos), "middle_k_pool": bf(orc.mid_k),
            "middle_v_pool": bf(orc.mid_v), "middle_pos_pool": t(orc.mid_pos),
            "recent_k_pool": bf(orc.rec_k), "recent_v_pool": bf(orc.rec_v),
            "recent_pos_pool": t(orc.rec_pos), "valid_count": t(orc.vc),
            "merge_k_pool": bf(orc.mg_k), "merge_v_pool": bf(orc.mg_v),
            "merge_pos_pool": t(orc.mg_pos), "merge_token_count": t(orc.mtc),
            "merge_accum_sum_k": t(orc.acc_k), "merge_accum_sum_v": t(orc.acc_v),
            "merge_accum_pos": t(orc.acc_pos), "merge_accum_group_ids": t(orc.acc_gid),
            "merge_accum_tokens_per_group": t(orc.acc_tpg),
            "merge_accum_num_groups": t(orc.acc_ng),
        }
        for name, ten in self._t.items():
            setattr(self, name, (lambda x: (lambda: x))(ten))

    def max_sink(self):
        return self.orc.max_sink

    def max_middle(self):
        return self.orc.max_middle

    def max_recent(self):
        return self.orc.max_recent


class OracleKernels:
    """``torch.ops.adahead`` as the reference's update calls it, with the C
    oracle in place of the three CUDA kernels (CPU tensors in and out)."""

    def __init__(self, orc):
        self.orc = orc

    @staticmethod
    def _u16(t):
        import torch
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    def mega_state_update(self, states, t_vals, d0, d1, d2, d3, d4, d5, d6, d7, H_, F_, pk):
        from oracle import pkv_oracle as O
        st = states.numpy()            # the layer's uint8 row, mutated in place
        descs = O.state_update(st, t_vals.numpy(), int(pk), int(H_))
        for dst, src in zip((d0, d1, d2, d3, d4, d5, d6, d7), descs):
            dst.copy_(__import__("torch").from_numpy(src))

    def pyramidkv_update(self, mgr, nk, nv, npos, kind, slot, frame, head):
        from oracle import pkv_oracle as O
        o = self.orc
        flat = lambda a: a.reshape(-1)  # noqa: E731
        O.lib().orc_update_frames(
            O._p(self._u16(nk)), O._p(self._u16(nv)), O._p(npos.contiguous().numpy()),
            O._p(flat(o.sink_k)), O._p(flat(o.sink_v)), O._p(flat(o.mid_k)),
            O._p(flat(o.mid_v)), O._p(flat(o.rec_k)), O._p(flat(o.rec_v)),
            O._p(flat(o.sink_pos)), O._p(flat(o.mid_pos)), O._p(flat(o.rec_pos)),
            O._p(kind.contiguous().numpy()), O._p(slot.contiguous().numpy()),
            O._p(frame.contiguous().numpy()), O._p(head.contiguous().numpy()),
            int(kind.numel()), o.H, o.FSEQ, o.D)

    def mega_merge_accum(self, states, nk, nv, npos, dk, dslot, dfin, dnew, acc_k, acc_v,
                         acc_pos, acc_gid, acc_tpg, acc_ng, mk, mv, mpos, mtc):
        from oracle import pkv_oracle as O
        o = self.orc
        Fn = nk.shape[0]
        O.lib().orc_merge_accum(
            O._p(states.contiguous().numpy()), O._p(self._u16(nk)), O._p(self._u16(nv)),
            O._p(npos.contiguous().numpy()), O._p(dk.contiguous().numpy()),
            O._p(dslot.contiguous().numpy()), O._p(dfin.contiguous().numpy()),
            O._p(dnew.contiguous().numpy()),
            O._p(acc_k.numpy()), O._p(acc_v.numpy()), O._p(acc_pos.numpy()),
            O._p(acc_gid.numpy()), O._p(acc_tpg.numpy()), O._p(acc_ng.numpy()),
            O._p(mk.view(__import__("torch").int16).numpy()),
            O._p(mv.view(__import__("torch").int16).numpy()), O._p(mpos.numpy()),
            O._p(mtc.numpy()), o.H, int(Fn), o.FSEQ, o.D, o.mma, o.mmb, o.mtpa)


def run_config(name, cfg, ref_modules):
    import torch
    from oracle import pkv_oracle as O
    import megacache_digest as MD
    mega_cache, factory, ops, rops = ref_modules
    labels = labels_for(cfg)
    states, caps, any_merge = reference_states(factory, mega_cache, ops, labels)
    tables, _ = O.rope_freq_tables(D)
    orc = O.OracleMegaCache(L, H, D, FSEQ, SINK, MIDDLE, RECENT, states, caps,
                            spatial_width=W, sink_time_mapping_mode="window_clamp",
                            sink_time_clamp_min=18, sink_time_clamp_max=21, freq_tables=tables)
    mgr = StandInManager(orc)
    kern = OracleKernels(orc)
    rops.ops = lambda: kern            # the reference's own _ops.ops(), pointed at the oracle
    ctx = mega_cache.MegaCacheCtx(
        mgr=mgr, states_bytes=torch.from_numpy(states.copy()), num_layers=L, num_heads=H,
        head_dim=D, frame_seqlen=FSEQ, sink_time_mapping_mode="window_clamp",
        sink_time_clamp_min=18, sink_time_clamp_max=21, spatial_width=W, spatial_height=HG,
        has_merge_head=any_merge, sink_caps_per_head=torch.from_numpy(caps))
    cache = mega_cache.MegaCache(ctx, 0)
    kv, q = inputs(cfg["seed"])
    bf = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)  # noqa: E731
    calls = []
    for blk in range(BLOCKS):
        for p, mode in enumerate(PASSES):
            k, v = kv[blk][p]
            cache.update(bf(k), bf(v), blk * F * FSEQ, cache_update_mode=mode)
            committed = {"committed_vc": ctx.committed_vc,
                         "committed_recent_k": ctx.committed_recent_k,
                         "committed_recent_v": ctx.committed_recent_v,
                         "committed_recent_pos": ctx.committed_recent_pos}
            calls.append(MD.state_digests(mgr, ctx.states_bytes, committed))
        print(f"{name}: block {blk} done", flush=True)
    out = {f"{name}_labels": labels.astype(np.int32), f"{name}_sink_caps": caps,
           f"{name}_states0": states}
    for key in calls[0]:
        out[f"{name}_{key}"] = np.stack([c[key] for c in calls])
    # plan + RoPE pack of the final state for the next block's three chunks
    orc.states[0] = ctx.states_bytes[0].numpy()
    start = BLOCKS * F * FSEQ
    pk = orc.plan_and_pack(0, start, F)
    cu = pk["cu"].astype(np.int32)
    segs = []
    for a_, b_ in zip(cu[:-1], cu[1:]):
        segs.append([MD.blob_digest(bf(pk["k"][a_:b_].copy())),
                     MD.blob_digest(bf(pk["v"][a_:b_].copy())),
                     MD.blob_digest(torch.from_numpy(pk["pos"][a_:b_].copy()))])
    out[f"{name}_plan_cu"] = cu
    out[f"{name}_plan_seg_digests"] = np.array(segs, np.int64)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    sys.path.insert(0, HERE)
    sys.path.insert(0, ROOT)
    sys.path.insert(0, args.reference)
    from pyramidkv import _mega_cache as mega_cache, factory, _mega_state_ops as ops
    from pyramidkv import _ops as rops
    out = {}
    for name, cfg in CONFIGS.items():
        out.update(run_config(name, cfg, (mega_cache, factory, ops, rops)))
    out["blocks"] = np.int32(BLOCKS)
    np.savez_compressed(os.path.join(HERE, "megacache_c1.npz"), **out)
    print("wrote", os.path.join(HERE, "megacache_c1.npz"))


if __name__ == "__main__":
    main()
