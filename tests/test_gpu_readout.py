"""The per-layer readout wrappers of pyramidkv._mega_attention on the GPU.

Restates the reference's known-answer tests for these wrappers
(tests/test_mega_readout.py:43-148 and tests/test_mega_attention_step.py:
46-162): pools planted with seeded K/V and a stride state with known tkey
slots, then

* ``mega_readout_kv_only`` must gather sink -> recent -> middle frames in the
  planner's order, bit for bit, with cu_seqlens_k = per-head token counts;
* ``mega_readout`` must match a torch fp32 softmax over that gather;
* ``mega_attention_step`` over two blocks of a stride head must advance the
  state (tkey_count 2 then 4, tkey_t [0, 1, 2, 3]), write the new frames'
  raw K into middle slots 0-3, and its second readout must match fp32
  attention over sink + recent + middle;
* ``_flash_attn_varlen()`` (the flash_attn_varlen_func-shaped callable) must
  match fp32 attention per equal-length query sequence.

head_dim 16 as in the reference tests (the CUDA-core kernel) and 128 (the
tcgen05 kernel).  Tolerance: max abs 2e-2, mean abs 2e-3 against fp32 (the
reference's own tests allow 5e-2).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _check(got, want):
    err = (got.float() - want).abs()
    assert err.max().item() <= MAX_ABS, err.max().item()
    assert err.mean().item() <= MEAN_ABS, err.mean().item()


def _ref_attn(q, k, v, scale=None):
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    return torch.softmax((q.float() @ k.float().T) * scale, dim=-1) @ v.float()


def _mgr(H, D, FSEQ, ms, mm, mr, L=1, chunks=4):
    from pyramidkv import _ops
    assert _ops._ensure_loaded()
    return torch.classes.adahead.PyramidKVCacheManager(L, H, D, FSEQ, ms, mm, mr, "cuda:0",
                                                       "bfloat16", chunks)


def _states(states, device):
    from pyramidkv import _mega_state_ops as ops
    return torch.from_numpy(np.frombuffer(ops.pack_states(states).tobytes(),
                                          dtype=np.uint8).copy()).to(device)


def _unpack(states_bytes, n):
    from pyramidkv import _mega_state_ops as ops
    arr = states_bytes.cpu().numpy().view(ops.PER_HEAD_STATE_DTYPE).reshape(n).copy()
    return ops.unpack_states(arr)


def _planted(cuda, H, D, FSEQ, ms, mm, mr):
    """Manager with seeded sink / middle / recent pools, full sink and recent,
    and H stride heads whose tkey ring holds slots 0-2."""
    from pyramidkv import _mega_state_ref as ref
    mgr = _mgr(H, D, FSEQ, ms, mm, mr)
    mgr.reset()
    g = torch.Generator(device="cpu").manual_seed(42)
    rnd = lambda *s: torch.randn(*s, generator=g).to(cuda, torch.bfloat16)  # noqa: E731
    pools = {"sink_k": rnd(H, ms, FSEQ, D), "sink_v": rnd(H, ms, FSEQ, D),
             "mid_k": rnd(H, mm, FSEQ, D), "mid_v": rnd(H, mm, FSEQ, D),
             "rec_k": rnd(H, mr, FSEQ, D), "rec_v": rnd(H, mr, FSEQ, D)}
    mgr.sink_k_pool()[0].copy_(pools["sink_k"])
    mgr.sink_v_pool()[0].copy_(pools["sink_v"])
    mgr.middle_k_pool()[0].copy_(pools["mid_k"])
    mgr.middle_v_pool()[0].copy_(pools["mid_v"])
    mgr.recent_k_pool()[0].copy_(pools["rec_k"])
    mgr.recent_v_pool()[0].copy_(pools["rec_v"])
    vc = mgr.valid_count()
    vc[0, :, 0] = ms
    vc[0, :, 1] = 3
    vc[0, :, 2] = mr
    states = [ref.make_stride(interval=1, capacity=mm) for _ in range(H)]
    for s in states:
        s.tkey_count = 3
        s.tkey_t = [10, 11, 12] + [0] * 21
        s.tkey_slot = [0, 1, 2] + [-1] * 21
    g2 = torch.Generator(device="cpu").manual_seed(43)
    q = torch.randn(1, FSEQ, H, D, generator=g2).to(cuda, torch.bfloat16)
    return mgr, _states(states, cuda), pools, q


def _gathered(pools, h, D):
    """Head h's K/V in the planner's order: sink, recent, middle slots 0-2."""
    k = torch.cat([pools["sink_k"][h].reshape(-1, D), pools["rec_k"][h].reshape(-1, D),
                   pools["mid_k"][h, :3].reshape(-1, D)])
    v = torch.cat([pools["sink_v"][h].reshape(-1, D), pools["rec_v"][h].reshape(-1, D),
                   pools["mid_v"][h, :3].reshape(-1, D)])
    return k, v


@pytest.mark.parametrize("D", [16, 128])
def test_mega_readout_kv_only_gathers_in_plan_order(cuda, D):
    from pyramidkv import _mega_attention
    H, FSEQ, ms, mm, mr = 2, 4, 2, 4, 2
    mgr, sb, pools, _ = _planted(cuda, H, D, FSEQ, ms, mm, mr)
    k, v, cu = _mega_attention.mega_readout_kv_only(mgr, sb, 0, 100, H, D)
    per = (ms + mr + 3) * FSEQ
    assert cu.tolist() == [0, per, 2 * per]
    for h in range(H):
        kw, vw = _gathered(pools, h, D)
        assert torch.equal(k[h * per:(h + 1) * per].reshape(-1, D), kw)
        assert torch.equal(v[h * per:(h + 1) * per].reshape(-1, D), vw)


@pytest.mark.parametrize("D", [16, 128])
def test_mega_readout_matches_direct_attention(cuda, D):
    from pyramidkv import _mega_attention
    H, FSEQ, ms, mm, mr = 2, 4, 2, 4, 2
    mgr, sb, pools, q = _planted(cuda, H, D, FSEQ, ms, mm, mr)
    out = _mega_attention.mega_readout(mgr=mgr, per_head_states_bytes=sb, q=q, layer_idx=0,
                                       current_t=100, max_seqlen_k=(ms + mm + mr) * FSEQ)
    assert out.shape == (1, FSEQ, H, D) and out.dtype == torch.bfloat16
    for h in range(H):
        kw, vw = _gathered(pools, h, D)
        _check(out[0, :, h], _ref_attn(q[0, :, h], kw, vw))


@pytest.mark.parametrize("D", [16, 128])
def test_mega_attention_step_two_blocks_stride(cuda, D):
    from pyramidkv import _mega_attention
    from pyramidkv import _mega_state_ref as ref
    H, FSEQ, ms, mm, mr, F = 1, 4, 2, 4, 2, 2
    mgr = _mgr(H, D, FSEQ, ms, mm, mr)
    mgr.reset()
    g = torch.Generator(device="cpu").manual_seed(7)
    rnd = lambda *s: torch.randn(*s, generator=g).to(cuda, torch.bfloat16)  # noqa: E731
    sink_k, sink_v = rnd(H, ms, FSEQ, D), rnd(H, ms, FSEQ, D)
    rec_k, rec_v = rnd(H, mr, FSEQ, D), rnd(H, mr, FSEQ, D)
    mgr.sink_k_pool()[0].copy_(sink_k)
    mgr.sink_v_pool()[0].copy_(sink_v)
    mgr.recent_k_pool()[0].copy_(rec_k)
    mgr.recent_v_pool()[0].copy_(rec_v)
    vc = mgr.valid_count()
    vc[0, 0, 0] = ms
    vc[0, 0, 2] = mr
    sb = _states([ref.make_stride(interval=1, capacity=mm)], cuda)
    frames = lambda x: x.view(1, F, FSEQ, H, D).permute(0, 1, 3, 2, 4).reshape(F, H, FSEQ, D)  # noqa
    ks, vs = [], []
    for blk in range(2):
        q, k, v = rnd(1, F * FSEQ, H, D), rnd(1, F * FSEQ, H, D), rnd(1, F * FSEQ, H, D)
        t = torch.arange(blk * F, (blk + 1) * F, dtype=torch.int64, device=cuda)
        out = _mega_attention.mega_attention_step(
            mgr=mgr, per_head_states_bytes=sb, q=q, k_new=k, v_new=v, new_t_vals=t,
            layer_idx=0, current_t=blk * F, pass_kind=1, max_seqlen_k=(ms + mm + mr) * FSEQ)
        assert out.shape == (1, F * FSEQ, H, D)
        st = _unpack(sb, H)[0]
        assert st.tkey_count == 2 * (blk + 1)
        assert list(st.tkey_t[:2 * (blk + 1)]) == list(range(2 * (blk + 1)))
        ks.append(frames(k)[:, 0])
        vs.append(frames(v)[:, 0])
        assert torch.equal(mgr.middle_k_pool()[0, 0, blk * F:(blk + 1) * F], ks[-1])
    K = torch.cat([sink_k[0].reshape(-1, D), rec_k[0].reshape(-1, D),
                   torch.cat(ks).reshape(-1, D)])
    V = torch.cat([sink_v[0].reshape(-1, D), rec_v[0].reshape(-1, D),
                   torch.cat(vs).reshape(-1, D)])
    _check(out[0, :, 0], _ref_attn(q[0, :, 0], K, V))


@pytest.mark.parametrize("D", [16, 128])
def test_flash_attn_varlen_shim(cuda, D):
    from pyramidkv import _mega_attention
    varlen = _mega_attention._flash_attn_varlen()
    n_seg, rows = 5, 200
    lens = [300, 1, 128, 0, 1000]
    g = torch.Generator(device="cpu").manual_seed(11)
    q = torch.randn(n_seg * rows, 1, D, generator=g).to(cuda, torch.bfloat16)
    T = sum(lens)
    k = torch.randn(T, 1, D, generator=g).to(cuda, torch.bfloat16)
    v = torch.randn(T, 1, D, generator=g).to(cuda, torch.bfloat16)
    cu_q = torch.arange(0, (n_seg + 1) * rows, rows, dtype=torch.int32, device=cuda)
    cu_k = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32,
                        device=cuda)
    out = varlen(q, k, v, cu_q, cu_k, rows, max(lens), softmax_scale=0.1, causal=False)
    assert out.shape == q.shape
    for s in range(n_seg):
        a, b = int(cu_k[s]), int(cu_k[s + 1])
        got = out[s * rows:(s + 1) * rows, 0]
        if b == a:
            assert got.abs().max().item() == 0.0
            continue
        _check(got, _ref_attn(q[s * rows:(s + 1) * rows, 0], k[a:b, 0], v[a:b, 0], 0.1))
    with pytest.raises(NotImplementedError):
        varlen(q, k, v, cu_q, cu_k, rows, max(lens), causal=True)
