"""MegaCache end to end (update + attend over many blocks) vs the oracle.

The oracle restates the reference's orchestration (pyramidkv/_mega_cache.py
:136-569) on numpy pools; the product runs the fused device ops.  After every
call the cache state must be bit-identical: valid_count, every pool (K, V,
pos), the committed snapshot, the state bytes, the merge anchors, and the
packed K/V the attention read (RoPE-rotated K included).  The attention output
is checked against the oracle's fp32 attention within the bf16 tolerance.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import pkv_oracle as O

pytestmark = pytest.mark.gpu


def _u16(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _bf16(a, dev):
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(dev)


def _build(cuda, labels, routing, W, Hgrid, D=128, sink_mode="window_clamp"):
    from pyramidkv import _mega_cache, policy
    labels = np.asarray(labels)
    L, H = labels.shape
    FSEQ = W * Hgrid
    states, caps = policy.states_from_labels(labels, routing)
    (ft, fy, fx), full = O.rope_freq_tables(D)
    comps = policy.compositions_from_labels(labels, routing)
    caches = _mega_cache.build_mega_caches(
        L, H, D, FSEQ, 3, 24, 4, comps, max_attend_chunks=8, device="cuda:0",
        sink_time_mapping_mode=sink_mode, sink_time_clamp_min=18, sink_time_clamp_max=21,
        spatial_width=W, spatial_height=Hgrid, freqs=full)
    orc = O.OracleMegaCache(L, H, D, FSEQ, 3, 24, 4, states, caps, spatial_width=W,
                            sink_time_mapping_mode=sink_mode, sink_time_clamp_min=18,
                            sink_time_clamp_max=21, freq_tables=(ft, fy, fx),
                            rope_mode=O.ROPE_FMA_FIRST)
    np.testing.assert_array_equal(caches[0].ctx.states_bytes.cpu().numpy(), orc.states)
    return caches, orc


def _compare_state(cache, orc, layer, where):
    mgr, ctx = cache.ctx.mgr, cache.ctx
    chk = np.testing.assert_array_equal
    chk(mgr.valid_count().cpu().numpy(), orc.vc, err_msg=f"{where}: valid_count")
    chk(ctx.committed_vc.cpu().numpy(), orc.committed_vc, err_msg=f"{where}: committed_vc")
    chk(ctx.states_bytes.cpu().numpy(), orc.states, err_msg=f"{where}: states")
    for name, ok, ov, op in (("sink", orc.sink_k, orc.sink_v, orc.sink_pos),
                             ("middle", orc.mid_k, orc.mid_v, orc.mid_pos),
                             ("recent", orc.rec_k, orc.rec_v, orc.rec_pos)):
        chk(_u16(getattr(mgr, f"{name}_k_pool")()).reshape(ok.shape), ok, err_msg=f"{where}: {name}_k")
        chk(_u16(getattr(mgr, f"{name}_v_pool")()).reshape(ov.shape), ov, err_msg=f"{where}: {name}_v")
        chk(getattr(mgr, f"{name}_pos_pool")().cpu().numpy(), op, err_msg=f"{where}: {name}_pos")
    chk(_u16(ctx.committed_recent_k).reshape(orc.committed_rec_k.shape), orc.committed_rec_k,
        err_msg=f"{where}: committed recent k")
    chk(ctx.committed_recent_pos.cpu().numpy(), orc.committed_rec_pos,
        err_msg=f"{where}: committed recent pos")
    chk(_u16(mgr.merge_k_pool()).reshape(orc.mg_k.shape), orc.mg_k, err_msg=f"{where}: merge_k")
    chk(mgr.merge_pos_pool().cpu().numpy(), orc.mg_pos, err_msg=f"{where}: merge_pos")
    chk(mgr.merge_token_count().cpu().numpy(), orc.mtc, err_msg=f"{where}: merge_token_count")
    # the merge accumulators (the grid-position merge kernel on this path)
    chk(mgr.merge_accum_sum_k().cpu().numpy().reshape(orc.acc_k.shape), orc.acc_k,
        err_msg=f"{where}: accum_sum_k")
    chk(mgr.merge_accum_sum_v().cpu().numpy().reshape(orc.acc_v.shape), orc.acc_v,
        err_msg=f"{where}: accum_sum_v")
    chk(mgr.merge_accum_pos().cpu().numpy().reshape(orc.acc_pos.shape), orc.acc_pos,
        err_msg=f"{where}: accum_pos")
    chk(mgr.merge_accum_group_ids().cpu().numpy().reshape(orc.acc_gid.shape), orc.acc_gid,
        err_msg=f"{where}: accum_group_ids")
    chk(mgr.merge_accum_tokens_per_group().cpu().numpy().reshape(orc.acc_tpg.shape), orc.acc_tpg,
        err_msg=f"{where}: accum_tokens_per_group")
    chk(mgr.merge_accum_num_groups().cpu().numpy().reshape(orc.acc_ng.shape), orc.acc_ng,
        err_msg=f"{where}: accum_num_groups")


@pytest.mark.parametrize("routing,W,Hgrid", [("baseline", 13, 8), ("yaml", 52, 30),
                                             ("baseline", 52, 32)])
def test_megacache_blocks_match_oracle(cuda, routing, W, Hgrid):
    """52 x 32 has 416 patch groups, more than a merge anchor holds (390): the
    reference folds the excess tokens into group 0."""
    rng = np.random.default_rng(17)
    labels = np.array([[-1, 1, 2, -1], [2, 2, 1, -1]])
    caches, orc = _build(cuda, labels, routing, W, Hgrid)
    L, H = labels.shape
    D, FSEQ, F = 128, W * Hgrid, 3
    n_blocks = 14 if W == 13 else 9 if Hgrid == 30 else 5
    for blk in range(n_blocks):
        start = blk * F * FSEQ
        for mode in ("noisy", "noisy", "clean"):
            for layer in range(L):
                k = O.f32_to_bf16(rng.standard_normal((1, F * FSEQ, H, D)).astype(np.float32))
                v = O.f32_to_bf16(rng.standard_normal((1, F * FSEQ, H, D)).astype(np.float32))
                q = O.f32_to_bf16(rng.standard_normal((1, F * FSEQ, H, D)).astype(np.float32))
                orc.update(layer, k, v, start, mode)
                caches[layer].update(_bf16(k, cuda).view(1, -1, H, D),
                                     _bf16(v, cuda).view(1, -1, H, D), start,
                                     cache_update_mode=mode)
                want, pk = orc.attend(layer, q, start)
                got = caches[layer].attend(_bf16(q, cuda).view(1, -1, H, D), start)
                torch.cuda.synchronize()
                where = f"block {blk} {mode} layer {layer}"
                _compare_state(caches[layer], orc, layer, where)
                mgr = caches[layer].ctx.mgr
                total = pk["total"]
                np.testing.assert_array_equal(mgr.cu_seqlens_k()[:3 * H + 1].cpu().numpy(),
                                              pk["cu"], err_msg=where)
                np.testing.assert_array_equal(_u16(mgr.k_flat_out()[:total]).reshape(total, D),
                                              pk["k"], err_msg=f"{where}: packed K")
                np.testing.assert_array_equal(_u16(mgr.v_flat_out()[:total]).reshape(total, D),
                                              pk["v"], err_msg=f"{where}: packed V")
                err = (got.float().cpu().numpy() - want).__abs__()
                assert err.max() <= 2e-2 and err.mean() <= 2e-3, (where, err.max(), err.mean())
    assert caches[0].ctx.check_status() == 0
    assert orc.mtc.max() > 0 or routing == "yaml"


@pytest.mark.parametrize("F", [1, 4])
def test_megacache_frames_per_call(cuda, F):
    """Updates of 1 and 4 frames per call (the model's blocks have 3): the
    merge kernel takes a call's frames in batches of 3, the pack plans F
    chunks.  State, pools, accumulators and packed K/V bit-exact."""
    rng = np.random.default_rng(23 + F)
    labels = np.array([[-1, 1, 2, -1]])
    W, Hgrid = 13, 8
    caches, orc = _build(cuda, labels, "baseline", W, Hgrid)
    L, H = labels.shape
    D, FSEQ = 128, W * Hgrid
    for blk in range(12 if F == 1 else 6):
        start = blk * F * FSEQ
        for mode in ("noisy", "clean"):
            k = O.f32_to_bf16(rng.standard_normal((1, F * FSEQ, H, D)).astype(np.float32))
            v = O.f32_to_bf16(rng.standard_normal((1, F * FSEQ, H, D)).astype(np.float32))
            q = O.f32_to_bf16(rng.standard_normal((1, F * FSEQ, H, D)).astype(np.float32))
            orc.update(0, k, v, start, mode)
            caches[0].update(_bf16(k, cuda).view(1, -1, H, D), _bf16(v, cuda).view(1, -1, H, D),
                             start, cache_update_mode=mode)
            want, pk = orc.attend(0, q, start)
            got = caches[0].attend(_bf16(q, cuda).view(1, -1, H, D), start)
            torch.cuda.synchronize()
            where = f"F={F} block {blk} {mode}"
            _compare_state(caches[0], orc, 0, where)
            mgr = caches[0].ctx.mgr
            total = pk["total"]
            np.testing.assert_array_equal(mgr.cu_seqlens_k()[:F * H + 1].cpu().numpy(), pk["cu"],
                                          err_msg=where)
            np.testing.assert_array_equal(_u16(mgr.k_flat_out()[:total]).reshape(total, D),
                                          pk["k"], err_msg=f"{where}: packed K")
            err = (got.float().cpu().numpy() - want).__abs__()
            assert err.max() <= 2e-2 and err.mean() <= 2e-3, (where, err.max(), err.mean())
    assert caches[0].ctx.check_status() == 0
    assert orc.mtc.max() > 0


def test_self_planning_pack_bounds_checks_corrupt_counts(cuda):
    """Merge token counts far past an anchor's capacity (a corrupted manager):
    the pack that plans for itself must flag the segments (pack overflow, slot
    range) and skip them, not read or write out of bounds, and attend raises
    the reference's capacity error; the cache keeps working once the counts
    are sane again."""
    labels = np.array([[-1, -1, 1, 2]])
    caches, orc = _build(cuda, labels, "baseline", 13, 8)
    H, D, FSEQ, F = 4, 128, 13 * 8, 3
    rng = np.random.default_rng(5)
    mk = lambda: _bf16(O.f32_to_bf16(rng.standard_normal((1, F * FSEQ, H, D))  # noqa: E731
                                     .astype(np.float32)), cuda).view(1, -1, H, D)
    for blk in range(6):
        caches[0].update(mk(), mk(), blk * F * FSEQ, cache_update_mode="clean")
    caches[0].attend(mk(), 6 * F * FSEQ)
    assert caches[0].ctx.check_status() == 0
    mtc = caches[0].ctx.mgr.merge_token_count()
    assert int(mtc.max()) > 0, "no merge anchor was finalized"
    saved = mtc.clone()
    mtc.masked_fill_(mtc > 0, 60000)
    # the reference's planner raises on a plan past the workspace; the op
    # reads the device's overflow bit (and clears the status word) to do so
    with pytest.raises(RuntimeError, match="exceed pack-workspace capacity"):
        caches[0].attend(mk(), 6 * F * FSEQ)
    mtc.copy_(saved)
    out = caches[0].attend(mk(), 6 * F * FSEQ)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert caches[0].ctx.check_status() == 0


def test_update_rejects_bad_shapes(cuda):
    caches, _ = _build(cuda, np.array([[1, 2]]), "baseline", 13, 8)
    with pytest.raises((AssertionError, RuntimeError)):
        caches[0].update(torch.zeros(1, 100, 2, 128, device=cuda, dtype=torch.bfloat16),
                         torch.zeros(1, 100, 2, 128, device=cuda, dtype=torch.bfloat16), 0)
    # unknown mode is a no-op, as in the reference
    caches[0].update(torch.zeros(1, 104, 2, 128, device=cuda, dtype=torch.bfloat16),
                     torch.zeros(1, 104, 2, 128, device=cuda, dtype=torch.bfloat16), 0,
                     cache_update_mode="other")
    assert int(caches[0].ctx.mgr.valid_count().abs().sum()) == 0


def test_megacache_two_launch_plan_pack(cuda):
    """The same blocks with the planner and the pack as two launches
    (PKV_FUSED_PLAN_PACK=0; the default pack plans for itself)."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, PKV_FUSED_PLAN_PACK="0")
    here = os.path.dirname(os.path.abspath(__file__))
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p",
                        "no:cacheprovider", os.path.join(here, "test_gpu_megacache.py"),
                        "-k", "blocks_match_oracle and baseline-13"],
                       env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert " passed" in r.stdout
