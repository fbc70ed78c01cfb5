"""Bit-exact parity against the reference's own kernels on the GPU.

oracle/_ref/adahead_ref.so is the reference's pyramidkv/csrc compiled from its
sources (oracle/Makefile.ref, the flags of its JIT loader).  A child process
(oracle/ref_runner.py) runs it on the inputs recorded here; this process runs
the product library and the CPU oracle on the same inputs.  Compared:
state machine (all 600 bytes, including the merge bookkeeping the reference's
Python mirror omits), multi-chunk plan, pack with fused RoPE (which also pins
the FMA evaluation order the reference's build uses), merge accumulation.
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT, golden
from oracle import pkv_oracle as O

pytestmark = pytest.mark.gpu

REF_SO = os.path.join(ROOT, "oracle", "_ref", "adahead_ref.so")
MIX = [
    {"kind": O.SK_CYCLIC, "period": 6, "bucket_cap": 4, "sink_capacity": 1},
    {"kind": O.SK_STRIDE, "interval": 6, "capacity": 4, "sink_capacity": 3},
    {"kind": O.SK_MERGE, "patch_size": 2, "capacity": 4, "sink_capacity": 3},
    {"kind": O.SK_LAG, "capacity": 7, "sink_capacity": 0},
    {"kind": O.SK_STRIDE, "interval": 1, "capacity": 24, "sink_capacity": 2},
    {"kind": O.SK_RECENT, "sink_capacity": 1},
]


def _rand_bf16(rng, shape):
    return O.f32_to_bf16(rng.standard_normal(shape).astype(np.float32))


@pytest.fixture(scope="module")
def ref_results(tmp_path_factory):
    if not os.path.exists(REF_SO):
        pytest.skip("reference extension not built (oracle/Makefile.ref)")
    rng = np.random.default_rng(2024)
    cases = []
    # 1. state machine over the golden sequences
    g = golden("state_sequences.npz")
    for i in range(0, int(g["n_cases"]), 3):
        cases.append(dict(op="state", states=g[f"c{i}_init"], H=g[f"c{i}_H"], F=g[f"c{i}_F"],
                          t=g[f"c{i}_t"], pk=g[f"c{i}_pk"]))
    # 2. plan on realistic states
    L, H, D, F, ms, mm, mr = 2, len(MIX), 128, 52, 3, 24, 4
    for trial in range(4):
        st = O.make_states(MIX)
        t = 0
        for _ in range(int(rng.integers(2, 20))):
            O.state_update(st, range(t, t + 3), 1, H)
            t += 3
        vc = np.zeros((L, H, 3), np.int64)
        vc[..., 0] = rng.integers(0, ms + 1, (L, H))
        vc[..., 2] = rng.integers(0, mr + 1, (L, H))
        mtc = rng.integers(1, 420, (L, H, 6)).astype(np.int32)
        cases.append(dict(op="plan", dims=np.array([L, H, D, F, ms, mm, mr, 4]), vc=vc, mtc=mtc,
                          states=st, layer=trial % L, ct=np.arange(t, t + 3, dtype=np.int64),
                          modes=np.array([trial % 2, 18, 21, 1])))
    # 3. pack with RoPE on random pools, plan from the oracle
    W = 13
    pools = {}
    for name, slots in (("sink", ms), ("middle", mm), ("recent", mr)):
        pools[name + "_k"] = _rand_bf16(rng, (L, H, slots, F, D))
        pools[name + "_v"] = _rand_bf16(rng, (L, H, slots, F, D))
        pos = np.zeros((L, H, slots, F, 3), np.int64)
        pos[..., 0] = rng.integers(-2, 40, (L, H, slots))[..., None]
        pos[..., 1] = np.arange(F) // W
        pos[..., 2] = np.arange(F) % W
        pools[name + "_pos"] = pos
    pools["merge_k"] = _rand_bf16(rng, (L, H, 6, 420, D))
    pools["merge_v"] = _rand_bf16(rng, (L, H, 6, 420, D))
    pools["merge_pos"] = rng.integers(0, 30, (L, H, 6, 420, 3)).astype(np.int64)
    st = cases[-1]["states"]
    vc, mtc = cases[-1]["vc"], cases[-1]["mtc"]
    cu, sk, sg, sl, dst, traw, tremap, total = O.plan_multi(
        vc, mtc, st, L=L, H=H, F=F, max_sink=ms, max_middle=mm, max_recent=mr, layer=1,
        current_t_list=[30, 31, 32], sink_mode="window_clamp", cmin=18, cmax=21)
    sga = O.layer_offset(sk, sg, 1, H, ms, mm, mr)
    (ft, fy, fx), _ = O.rope_freq_tables(D)
    for rope in (1, 0):
        cases.append(dict(op="pack", dims=np.array([L, H, D, F, ms, mm, mr, 4]), sk=sk, sg=sga,
                          sl=sl, dst=dst, tremap=tremap, ft=ft, fy=fy, fx=fx, total=total,
                          rope=rope, **pools))
    # 4. merge accumulation over several blocks
    Hm, FSEQ, Fb = 2, W * 8, 3
    mst = O.make_states([{"kind": O.SK_MERGE, "patch_size": 2, "capacity": 4},
                         {"kind": O.SK_MERGE, "patch_size": 1, "capacity": 2}])
    ts = np.array([[b * Fb + i for i in range(Fb)] for b in range(8)], np.int64)
    pos = np.zeros((8, Fb, Hm, FSEQ, 3), np.int64)
    pos[..., 0] = ts[:, :, None, None]
    pos[..., 1] = np.arange(FSEQ) // W
    pos[..., 2] = np.arange(FSEQ) % W
    cases.append(dict(op="merge", dims=np.array([1, Hm, D, FSEQ, 3, 8, 4, 2]), states=mst, H=Hm,
                      Fb=Fb, t=ts, nk=_rand_bf16(rng, (8, Fb, Hm, FSEQ, D)),
                      nv=_rand_bf16(rng, (8, Fb, Hm, FSEQ, D)), pos=pos))
    flat = {"n_cases": np.array(len(cases))}
    for i, c in enumerate(cases):
        for k, v in c.items():
            flat[f"c{i}_{k}"] = np.asarray(v)
    d = tmp_path_factory.mktemp("ref")
    inp, outp = str(d / "cases.npz"), str(d / "out.npz")
    np.savez(inp, **flat)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "oracle", "ref_runner.py"), inp, outp],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return cases, np.load(outp)


def test_state_machine_equals_reference_kernel(cuda, ref_results):
    cases, out = ref_results
    for i, c in enumerate(cases):
        if c["op"] != "state":
            continue
        H, F = int(c["H"]), int(c["F"])
        mine = torch.from_numpy(c["states"].copy()).to(cuda)
        orc = c["states"].copy()
        for j, tv in enumerate(c["t"]):
            d = [torch.full((H * F,), 7, dtype=torch.int32, device=cuda) for _ in range(8)]
            torch.ops.adahead.mega_state_update(mine, torch.from_numpy(tv).to(cuda), *d, H, F,
                                                int(c["pk"][j]))
            np.testing.assert_array_equal(np.stack([x.cpu().numpy() for x in d]),
                                          out[f"c{i}_desc"][j])
            O.state_update(orc, tv, int(c["pk"][j]), H)
        np.testing.assert_array_equal(mine.cpu().numpy(), out[f"c{i}_states"])
        np.testing.assert_array_equal(orc, out[f"c{i}_states"])


def test_plan_equals_reference_planner(cuda, ref_results):
    from pyramidkv import _mega_state_ops as so
    cases, out = ref_results
    for i, c in enumerate(cases):
        if c["op"] != "plan":
            continue
        L, H, D, F, ms, mm, mr, mac = (int(x) for x in c["dims"])
        mgr = torch.classes.adahead.PyramidKVCacheManager(L, H, D, F, ms, mm, mr, "cuda:0",
                                                          "bfloat16", mac)
        mgr.valid_count().copy_(torch.from_numpy(c["vc"]))
        mgr.merge_token_count().copy_(torch.from_numpy(c["mtc"]))
        mode, cmin, cmax, lag = (int(x) for x in c["modes"])
        got = so.mega_plan_multi_cuda(mgr, torch.from_numpy(c["states"]).to(cuda),
                                      int(c["layer"]), c["ct"].tolist(),
                                      sink_time_mapping_mode=["lag", "window_clamp"][mode],
                                      sink_time_clamp_min=cmin, sink_time_clamp_max=cmax,
                                      decoupled_sink_time_lag=lag)
        orc = O.plan_multi(c["vc"], c["mtc"], c["states"], L=L, H=H, F=F, max_sink=ms,
                           max_middle=mm, max_recent=mr, layer=int(c["layer"]),
                           current_t_list=c["ct"].tolist(), sink_mode=mode, cmin=cmin,
                           cmax=cmax, lag=lag)
        for j, name in enumerate(("cu", "sk", "sg", "sl", "dst", "traw", "tremap")):
            np.testing.assert_array_equal(got[j].cpu().numpy(), out[f"c{i}_{name}"], err_msg=name)
            np.testing.assert_array_equal(orc[j], out[f"c{i}_{name}"], err_msg="oracle " + name)


def test_pack_equals_reference_kernel_and_pins_rope_order(cuda, ref_results):
    from pyramidkv import _ops
    cases, out = ref_results
    checked = 0
    for i, c in enumerate(cases):
        if c["op"] != "pack":
            continue
        L, H, D, F, ms, mm, mr, mac = (int(x) for x in c["dims"])
        mgr = torch.classes.adahead.PyramidKVCacheManager(L, H, D, F, ms, mm, mr, "cuda:0",
                                                          "bfloat16", mac)
        for name in ("sink", "middle", "recent"):
            for part in ("k", "v"):
                t = getattr(mgr, f"{name}_{part}_pool")()
                t.copy_(torch.from_numpy(c[f"{name}_{part}"].view(np.int16)).view(torch.bfloat16)
                        .view(t.shape))
            getattr(mgr, f"{name}_pos_pool")().copy_(torch.from_numpy(c[f"{name}_pos"]))
        for part in ("k", "v"):
            t = getattr(mgr, f"merge_{part}_pool")()
            t.copy_(torch.from_numpy(c[f"merge_{part}"].view(np.int16)).view(torch.bfloat16)
                    .view(t.shape))
        mgr.merge_pos_pool().copy_(torch.from_numpy(c["merge_pos"]))
        T = int(c["total"])
        dv = lambda k: torch.from_numpy(c[k]).to(cuda)  # noqa: E731
        kw = {}
        if int(c["rope"]):
            kw = dict(anchor_t_remap=dv("tremap"), freqs_ft_flat=dv("ft"),
                      freqs_fy_flat=dv("fy"), freqs_fx_flat=dv("fx"))
        _ops.pyramidkv_pack(mgr, dv("sk"), dv("sg"), dv("sl"), dv("dst"), **kw)
        torch.cuda.synchronize()
        got_k = mgr.k_flat_out()[:T].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        np.testing.assert_array_equal(got_k.reshape(T, D), out[f"c{i}_k"],
                                      err_msg=f"packed K (rope={int(c['rope'])})")
        got_v = mgr.v_flat_out()[:T].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        np.testing.assert_array_equal(got_v.reshape(T, D), out[f"c{i}_v"])
        np.testing.assert_array_equal(mgr.pos_flat_out()[:T].cpu().numpy(), out[f"c{i}_pos"])
        checked += 1
    assert checked == 2


def test_merge_equals_reference_kernel(cuda, ref_results):
    from pyramidkv import _mega_state_ops as so
    cases, out = ref_results
    for i, c in enumerate(cases):
        if c["op"] != "merge":
            continue
        L, H, D, FSEQ, ms, mm, mr, mac = (int(x) for x in c["dims"])
        Fb = int(c["Fb"])
        mgr = torch.classes.adahead.PyramidKVCacheManager(L, H, D, FSEQ, ms, mm, mr, "cuda:0",
                                                          "bfloat16", mac)
        st = torch.from_numpy(c["states"].copy()).to(cuda)
        for j in range(c["t"].shape[0]):
            d = [torch.full((H * Fb,), -1, dtype=torch.int32, device=cuda) for _ in range(8)]
            torch.ops.adahead.mega_state_update(st, torch.from_numpy(c["t"][j]).to(cuda), *d, H,
                                                Fb, 1)
            dk = torch.where(d[0] == 5, d[0], torch.full_like(d[0], -1))
            bf = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(cuda)  # noqa
            so.mega_merge_accum_cuda(mgr, 0, st, bf(c["nk"][j]), bf(c["nv"][j]),
                                     torch.from_numpy(c["pos"][j]).to(cuda),
                                     (dk, d[4], d[6], d[7]))
        torch.cuda.synchronize()
        u16 = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa
        np.testing.assert_array_equal(st.cpu().numpy(), out[f"c{i}_states"])
        np.testing.assert_array_equal(mgr.merge_accum_sum_k()[0].cpu().numpy(), out[f"c{i}_acc_k"])
        np.testing.assert_array_equal(mgr.merge_accum_sum_v()[0].cpu().numpy(), out[f"c{i}_acc_v"])
        np.testing.assert_array_equal(u16(mgr.merge_k_pool()[0]), out[f"c{i}_mk"])
        np.testing.assert_array_equal(u16(mgr.merge_v_pool()[0]), out[f"c{i}_mv"])
        np.testing.assert_array_equal(mgr.merge_pos_pool()[0].cpu().numpy(), out[f"c{i}_mpos"])
        np.testing.assert_array_equal(mgr.merge_token_count()[0].cpu().numpy(), out[f"c{i}_mtc"])
        np.testing.assert_array_equal(mgr.merge_accum_tokens_per_group()[0].cpu().numpy(),
                                      out[f"c{i}_tpg"])
        assert out[f"c{i}_mtc"].max() > 0
