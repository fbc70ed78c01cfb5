"""GPU parity of the cache kernels against the CPU oracle (bit-exact).

Each test drives one reference op through ``torch.ops.adahead`` (the C ABI
underneath) and the oracle's restatement of the reference kernel on the same
seeded inputs:

* mega_state_update   pyramidkv/csrc/anchor_store_update.cu:233-313
* mega_plan(_multi)   pyramidkv/csrc/mega_plan.cc:133-264, :510-654
* pyramidkv_update    pyramidkv/csrc/pyramidkv_update.cu:21-110
* pyramidkv_pack      pyramidkv/csrc/pyramidkv_pack.cu:28-185
* mega_merge_accum    pyramidkv/csrc/mega_merge_accum.cu:52-252
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import pkv_oracle as O

pytestmark = pytest.mark.gpu


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _bf16(a: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(dev)


def _rand_bf16(rng, shape):
    return O.f32_to_bf16(rng.standard_normal(shape).astype(np.float32))


def _states_after(rng, kinds, steps, F=3, t0=0):
    """Advance oracle states over `steps` clean blocks to get realistic state."""
    H = len(kinds)
    st = O.make_states(kinds)
    t = t0
    for _ in range(steps):
        O.state_update(st, range(t, t + F), 1, H)
        t += F
    return st, t


MIX = [
    {"kind": O.SK_CYCLIC, "period": 6, "bucket_cap": 4, "sink_capacity": 1},
    {"kind": O.SK_STRIDE, "interval": 6, "capacity": 4, "sink_capacity": 3},
    {"kind": O.SK_MERGE, "patch_size": 2, "capacity": 4, "sink_capacity": 3},
    {"kind": O.SK_LAG, "capacity": 7, "sink_capacity": 0},
    {"kind": O.SK_STRIDE, "interval": 1, "capacity": 24, "sink_capacity": 2},
    {"kind": O.SK_RECENT, "sink_capacity": 1},
    {"kind": O.SK_CYCLIC, "period": 5, "bucket_cap": 3, "sink_capacity": 0},
    {"kind": O.SK_MERGE, "patch_size": 1, "capacity": 2, "sink_capacity": 1},
]


def test_state_update_matches_reference_sequences(cuda):
    from pyramidkv import _ops
    g = golden("state_sequences.npz")
    ops = _ops.ops()
    for i in range(int(g["n_cases"])):
        H = int(g[f"c{i}_H"])
        ref_states = g[f"c{i}_init"].copy()
        dev_states = torch.from_numpy(ref_states.copy()).to(cuda)
        for j in range(g[f"c{i}_t"].shape[0]):
            tv = g[f"c{i}_t"][j]
            pk = int(g[f"c{i}_pk"][j])
            want = O.state_update(ref_states, tv, pk, H)
            F = len(tv)
            d = [torch.full((H * F,), 7, dtype=torch.int32, device=cuda) for _ in range(8)]
            ops.mega_state_update(dev_states, torch.tensor(tv, device=cuda), *d, H, F, pk)
            got = np.stack([x.cpu().numpy() for x in d])
            np.testing.assert_array_equal(got, np.stack(want), err_msg=f"case {i} call {j}")
            np.testing.assert_array_equal(dev_states.cpu().numpy(), ref_states,
                                          err_msg=f"case {i} call {j}")


def _mgr(L, H, D, F, ms, mm, mr, mac=4):
    return torch.classes.adahead.PyramidKVCacheManager(L, H, D, F, ms, mm, mr, "cuda:0",
                                                       "bfloat16", mac)


@pytest.mark.parametrize("sink_mode", ["lag", "window_clamp"])
@pytest.mark.parametrize("ms,mm,mr", [(3, 24, 4), (5, 24, 6)])
def test_plan_multi_bit_exact(cuda, sink_mode, ms, mm, mr):
    """(3, 24, 4): the warp-per-(chunk, head) planner; (5, 24, 6): more sink
    and recent slots than its candidate list holds, the thread-per-(chunk,
    head) planner (plan_kernel)."""
    from pyramidkv import _mega_state_ops as so
    rng = np.random.default_rng(3)
    L, H, D, F = 3, len(MIX), 16, 8
    mgr = _mgr(L, H, D, F, ms, mm, mr)
    for trial in range(6):
        st, t_end = _states_after(rng, MIX, steps=int(rng.integers(1, 25)))
        layer = int(rng.integers(0, L))
        vc = np.zeros((L, H, 3), np.int64)
        vc[:, :, 0] = rng.integers(0, ms + 2, (L, H))
        vc[:, :, 1] = rng.integers(0, mm, (L, H))
        vc[:, :, 2] = rng.integers(0, mr + 2, (L, H))
        mtc = rng.integers(0, 420, (L, H, 6)).astype(np.int32)
        mgr.valid_count().copy_(torch.from_numpy(vc))
        mgr.merge_token_count().copy_(torch.from_numpy(mtc))
        C = int(rng.integers(1, 4))
        cts = [t_end + c for c in range(C)]
        want = O.plan_multi(vc, mtc, st, L=L, H=H, F=F, max_sink=ms, max_middle=mm,
                            max_recent=mr, layer=layer, current_t_list=cts,
                            sink_mode=sink_mode, cmin=18, cmax=21, lag=2)
        got = so.mega_plan_multi_cuda(mgr, torch.from_numpy(st).to(cuda), layer, cts,
                                      sink_time_mapping_mode=sink_mode, sink_time_clamp_min=18,
                                      sink_time_clamp_max=21, decoupled_sink_time_lag=2)
        for w, gt, name in zip(want[:7], got, ["cu", "sk", "sg", "sl", "dst", "traw", "tremap"]):
            np.testing.assert_array_equal(gt.cpu().numpy(), w, err_msg=f"trial {trial} {name}")
        single = so.mega_plan_cuda(mgr, torch.from_numpy(st).to(cuda), layer, cts[0],
                                   sink_time_mapping_mode=sink_mode, sink_time_clamp_min=18,
                                   sink_time_clamp_max=21, decoupled_sink_time_lag=2)
        w1 = O.plan_multi(vc, mtc, st, L=L, H=H, F=F, max_sink=ms, max_middle=mm,
                          max_recent=mr, layer=layer, current_t_list=cts[:1],
                          sink_mode=sink_mode, cmin=18, cmax=21, lag=2)
        for w, gt in zip(w1[:7], single):
            np.testing.assert_array_equal(gt.cpu().numpy(), w)


def test_plan_overflow_raises(cuda):
    from pyramidkv import _mega_state_ops as so
    H, D, F, ms, mm, mr = 2, 16, 4, 2, 4, 2
    mgr = _mgr(1, H, D, F, ms, mm, mr, mac=1)
    # 24 lag slots per head (more than max_middle) make each chunk emit
    # 2 + 2 + 24 frames -> 3 chunks exceed the one-chunk workspace
    st, _ = _states_after(np.random.default_rng(0), [{"kind": O.SK_LAG, "capacity": 24}] * H,
                          steps=8)
    mgr.valid_count()[0, :, 0] = ms
    mgr.valid_count()[0, :, 2] = mr
    with pytest.raises(RuntimeError, match="exceed pack-workspace capacity"):
        so.mega_plan_multi_cuda(mgr, torch.from_numpy(st).to(cuda), 0, [30, 31, 32])
    assert int(torch.ops.adahead.pkv_status(mgr)) == 0  # cleared by the raise path


def _fill_pools(mgr, rng, W):
    pools = {}
    for name in ("sink", "middle", "recent"):
        k = getattr(mgr, f"{name}_k_pool")()
        v = getattr(mgr, f"{name}_v_pool")()
        p = getattr(mgr, f"{name}_pos_pool")()
        kk = _rand_bf16(rng, tuple(k.shape))
        vv = _rand_bf16(rng, tuple(v.shape))
        pp = np.zeros(tuple(p.shape), np.int64)
        F = p.shape[3]
        pp[..., 0] = rng.integers(-2, 40, p.shape[:3])[..., None]
        pp[..., 1] = (np.arange(F) // W)[None, None, None]
        pp[..., 2] = (np.arange(F) % W)[None, None, None]
        k.copy_(_bf16(kk, k.device).view(k.shape))
        v.copy_(_bf16(vv, v.device).view(v.shape))
        p.copy_(torch.from_numpy(pp))
        pools[name] = (kk, vv, pp)
    mk, mv, mp = mgr.merge_k_pool(), mgr.merge_v_pool(), mgr.merge_pos_pool()
    kk = _rand_bf16(rng, tuple(mk.shape))
    vv = _rand_bf16(rng, tuple(mv.shape))
    pp = rng.integers(0, 30, tuple(mp.shape)).astype(np.int64)
    mk.copy_(_bf16(kk, mk.device).view(mk.shape))
    mv.copy_(_bf16(vv, mv.device).view(mv.shape))
    mp.copy_(torch.from_numpy(pp))
    pools["merge"] = (kk, vv, pp)
    return pools


@pytest.mark.parametrize("rope_mode", [O.ROPE_FMA_FIRST, O.ROPE_FMA_SECOND, O.ROPE_NO_FMA])
def test_pack_bit_exact(cuda, rope_mode):
    from pyramidkv import _mega_attention as ma, _mega_state_ops as so, _ops
    rng = np.random.default_rng(11)
    L, H, D, F, ms, mm, mr, W = 2, len(MIX), 128, 52, 3, 24, 4, 13
    mgr = _mgr(L, H, D, F, ms, mm, mr)
    pools = _fill_pools(mgr, rng, W)
    st, t_end = _states_after(rng, MIX, steps=12)
    layer = 1
    vc = np.zeros((L, H, 3), np.int64)
    vc[:, :, 0] = ms
    vc[:, :, 2] = rng.integers(0, mr + 1, (L, H))
    mtc = rng.integers(1, 420, (L, H, 6)).astype(np.int32)
    mgr.valid_count().copy_(torch.from_numpy(vc))
    mgr.merge_token_count().copy_(torch.from_numpy(mtc))
    cts = [t_end, t_end + 1, t_end + 2]
    cu, sk, sg, sl, dst, traw, tremap, total = O.plan_multi(
        vc, mtc, st, L=L, H=H, F=F, max_sink=ms, max_middle=mm, max_recent=mr, layer=layer,
        current_t_list=cts, sink_mode="window_clamp", cmin=18, cmax=21)
    sga = O.layer_offset(sk, sg, layer, H, ms, mm, mr)
    (ft, fy, fx), _ = O.rope_freq_tables(D)
    k_out = np.zeros((total, D), np.uint16)
    v_out = np.zeros((total, D), np.uint16)
    pos_out = np.zeros((total, 3), np.int64)
    P = O._p
    flat = lambda a: np.ascontiguousarray(a).reshape(-1)  # noqa: E731
    O.lib().orc_pack(P(flat(pools["sink"][0])), P(flat(pools["sink"][1])),
                     P(flat(pools["middle"][0])), P(flat(pools["middle"][1])),
                     P(flat(pools["recent"][0])), P(flat(pools["recent"][1])),
                     P(flat(pools["merge"][0])), P(flat(pools["merge"][1])),
                     P(flat(pools["sink"][2])), P(flat(pools["middle"][2])),
                     P(flat(pools["recent"][2])), P(flat(pools["merge"][2])),
                     P(k_out), P(v_out), P(pos_out), P(sk), P(sga), P(sl), P(dst), sk.size,
                     P(tremap), P(ft), ft.shape[0], 22, P(fy), fy.shape[0], 21, P(fx),
                     fx.shape[0], 21, F, 420, D, rope_mode)
    tens = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    prev = _ops.ops().pkv_rope_rounding(rope_mode)
    try:
        _ops.pyramidkv_pack(mgr, tens(sk), tens(sga), tens(sl), tens(dst),
                            anchor_t_remap=tens(tremap), freqs_ft_flat=tens(ft),
                            freqs_fy_flat=tens(fy), freqs_fx_flat=tens(fx))
        torch.cuda.synchronize()
    finally:
        _ops.ops().pkv_rope_rounding(prev)
    np.testing.assert_array_equal(_u16(mgr.k_flat_out()[:total]).reshape(total, D), k_out)
    np.testing.assert_array_equal(_u16(mgr.v_flat_out()[:total]).reshape(total, D), v_out)
    np.testing.assert_array_equal(mgr.pos_flat_out()[:total].cpu().numpy(), pos_out)
    # plain copy path (no RoPE): packed K == pool K
    _ops.pyramidkv_pack(mgr, tens(sk), tens(sga), tens(sl), tens(dst))
    O.lib().orc_pack(P(flat(pools["sink"][0])), P(flat(pools["sink"][1])),
                     P(flat(pools["middle"][0])), P(flat(pools["middle"][1])),
                     P(flat(pools["recent"][0])), P(flat(pools["recent"][1])),
                     P(flat(pools["merge"][0])), P(flat(pools["merge"][1])),
                     P(flat(pools["sink"][2])), P(flat(pools["middle"][2])),
                     P(flat(pools["recent"][2])), P(flat(pools["merge"][2])),
                     P(k_out), P(v_out), P(pos_out), P(sk), P(sga), P(sl), P(dst), sk.size,
                     None, None, 0, 0, None, 0, 0, None, 0, 0, F, 420, D, 0)
    np.testing.assert_array_equal(_u16(mgr.k_flat_out()[:total]).reshape(total, D), k_out)
    assert int(torch.ops.adahead.pkv_status(mgr)) == 0
    del so, ma


def test_pack_rejects_out_of_range_segments_without_fault(cuda):
    from pyramidkv import _ops
    L, H, D, F = 1, 2, 128, 16
    mgr = _mgr(L, H, D, F, 1, 2, 1, mac=1)
    sk = torch.tensor([1, 0, 3], dtype=torch.int32, device=cuda)
    sg = torch.tensor([99, 0, 0], dtype=torch.int32, device=cuda)      # slot 99 out of pool
    sl = torch.tensor([F, F, 5], dtype=torch.int32, device=cuda)
    cap = mgr.max_pack_tokens()
    dst = torch.tensor([0, cap - 3, 0], dtype=torch.int32, device=cuda)  # runs past the end
    _ops.pyramidkv_pack(mgr, sk, sg, sl, dst)
    torch.cuda.synchronize()
    st = int(torch.ops.adahead.pkv_status(mgr))
    assert st & 0x2 and st & 0x1


def test_update_frames_bit_exact(cuda):
    from pyramidkv import _ops
    rng = np.random.default_rng(5)
    L, H, D, F, ms, mm, mr = 2, 3, 128, 40, 3, 6, 4
    mgr = _mgr(L, H, D, F, ms, mm, mr)
    Fb = 3
    nk = _rand_bf16(rng, (Fb, H, F, D))
    nv = _rand_bf16(rng, (Fb, H, F, D))
    npos = rng.integers(0, 50, (Fb, H, F, 3)).astype(np.int64)
    n = 10
    kind = rng.integers(-1, 3, n).astype(np.int32)
    slots = {0: ms, 1: mm, 2: mr}
    sg = np.array([rng.integers(0, L * H * slots[max(int(k), 0)]) for k in kind], np.int32)
    fr = rng.integers(0, Fb, n).astype(np.int32)
    hd = rng.integers(0, H, n).astype(np.int32)
    pools = {k: (np.zeros((L * H * s, F, D), np.uint16), np.zeros((L * H * s, F, D), np.uint16),
                 np.zeros((L * H * s, F, 3), np.int64)) for k, s in slots.items()}
    P = O._p
    O.lib().orc_update_frames(P(nk), P(nv), P(npos), P(pools[0][0]), P(pools[0][1]),
                              P(pools[1][0]), P(pools[1][1]), P(pools[2][0]), P(pools[2][1]),
                              P(pools[0][2]), P(pools[1][2]), P(pools[2][2]), P(kind), P(sg),
                              P(fr), P(hd), n, H, F, D)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    _ops.ops().pyramidkv_update(mgr, _bf16(nk, cuda).view(Fb, H, F, D),
                                _bf16(nv, cuda).view(Fb, H, F, D), t(npos), t(kind), t(sg), t(fr),
                                t(hd))
    for k, name in ((0, "sink"), (1, "middle"), (2, "recent")):
        np.testing.assert_array_equal(_u16(getattr(mgr, f"{name}_k_pool")()).reshape(-1, F, D),
                                      pools[k][0])
        np.testing.assert_array_equal(_u16(getattr(mgr, f"{name}_v_pool")()).reshape(-1, F, D),
                                      pools[k][1])
        np.testing.assert_array_equal(getattr(mgr, f"{name}_pos_pool")().cpu().numpy()
                                      .reshape(-1, F, 3), pools[k][2])


@pytest.mark.parametrize("W,Hgrid,D", [(52, 30, 128), (13, 7, 128), (13, 7, 64)])
def test_merge_accum_bit_exact(cuda, W, Hgrid, D):
    """Several blocks of merge frames through the op vs the oracle; accumulators,
    group ids / divisors / positions and finalized anchors all bit-identical.
    head_dim 128 takes the batched 4-dims-per-lane path, 64 the element loop."""
    from pyramidkv import _mega_state_ops as so
    rng = np.random.default_rng(W)
    H, FSEQ, Fb = 3, W * Hgrid, 3
    kinds = [{"kind": O.SK_MERGE, "patch_size": 2, "capacity": 4},
             {"kind": O.SK_MERGE, "patch_size": 1, "capacity": 2},
             {"kind": O.SK_STRIDE, "interval": 2, "capacity": 4}]
    st = O.make_states(kinds)
    dst = torch.from_numpy(st.copy()).to(cuda)
    mgr = _mgr(1, H, D, FSEQ, 3, 8, 4)
    MMA, MMB, MTPA = 2, 6, 420
    acc = dict(k=np.zeros((H, MMA, MTPA, D), np.float32), v=np.zeros((H, MMA, MTPA, D), np.float32),
               pos=np.zeros((H, MMA, MTPA, 3), np.int64), gid=np.zeros((H, MMA, FSEQ), np.int32),
               tpg=np.zeros((H, MMA, MTPA), np.float32), ng=np.zeros((H, MMA), np.int32),
               mk=np.zeros((H, MMB, MTPA, D), np.uint16), mv=np.zeros((H, MMB, MTPA, D), np.uint16),
               mpos=np.zeros((H, MMB, MTPA, 3), np.int64), mtc=np.zeros((H, MMB), np.int32))
    P = O._p
    for blk in range(7):
        tv = list(range(blk * Fb, blk * Fb + Fb))
        d = O.state_update(st, tv, 1, H)
        dk = np.where(d[0] == 5, d[0], -1).astype(np.int32)
        nk = _rand_bf16(rng, (Fb, H, FSEQ, D))
        nv = _rand_bf16(rng, (Fb, H, FSEQ, D))
        pos = np.zeros((Fb, H, FSEQ, 3), np.int64)
        pos[..., 0] = np.asarray(tv)[:, None, None]
        pos[..., 1] = np.arange(FSEQ) // W
        pos[..., 2] = np.arange(FSEQ) % W
        O.lib().orc_merge_accum(P(st), P(nk), P(nv), P(pos), P(dk), P(d[4]), P(d[6]), P(d[7]),
                                P(acc["k"]), P(acc["v"]), P(acc["pos"]), P(acc["gid"]),
                                P(acc["tpg"]), P(acc["ng"]), P(acc["mk"]), P(acc["mv"]),
                                P(acc["mpos"]), P(acc["mtc"]), H, Fb, FSEQ, D, MMA, MMB, MTPA)
        # device: same state machine on the device copy, then the merge op
        dd = [torch.full((H * Fb,), -1, dtype=torch.int32, device=cuda) for _ in range(8)]
        torch.ops.adahead.mega_state_update(dst, torch.tensor(tv, device=cuda), *dd, H, Fb, 1)
        dk_dev = torch.where(dd[0] == 5, dd[0], torch.full_like(dd[0], -1))
        so.mega_merge_accum_cuda(mgr, 0, dst, _bf16(nk, cuda).view(Fb, H, FSEQ, D),
                                 _bf16(nv, cuda).view(Fb, H, FSEQ, D),
                                 torch.from_numpy(pos).to(cuda), (dk_dev, dd[4], dd[6], dd[7]))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(dst.cpu().numpy(), st)
        np.testing.assert_array_equal(mgr.merge_accum_sum_k()[0].cpu().numpy(), acc["k"])
        np.testing.assert_array_equal(mgr.merge_accum_sum_v()[0].cpu().numpy(), acc["v"])
        np.testing.assert_array_equal(mgr.merge_accum_group_ids()[0].cpu().numpy(), acc["gid"])
        np.testing.assert_array_equal(mgr.merge_accum_tokens_per_group()[0].cpu().numpy(),
                                      acc["tpg"])
        np.testing.assert_array_equal(mgr.merge_accum_num_groups()[0].cpu().numpy(), acc["ng"])
        np.testing.assert_array_equal(mgr.merge_accum_pos()[0].cpu().numpy(), acc["pos"])
        np.testing.assert_array_equal(_u16(mgr.merge_k_pool()[0]).reshape(acc["mk"].shape), acc["mk"])
        np.testing.assert_array_equal(_u16(mgr.merge_v_pool()[0]).reshape(acc["mv"].shape), acc["mv"])
        np.testing.assert_array_equal(mgr.merge_pos_pool()[0].cpu().numpy(), acc["mpos"])
        np.testing.assert_array_equal(mgr.merge_token_count()[0].cpu().numpy(), acc["mtc"])
    assert acc["mtc"].max() > 0  # anchors were finalized
