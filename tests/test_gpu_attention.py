"""Ragged attention kernel vs a plain PyTorch fp32 reference.

The reference's attention is flash_attn_varlen_func over the packed K/V
(pyramidkv/_mega_cache.py:529-569), pinned by its own tests only against an
fp32 softmax (tests/test_mega_readout.py:43-56).  Tolerance (bf16 output vs
fp32 reference): max abs 2e-2, mean abs 2e-3.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _reference(q, k, v, cu, C, H, Lq, scale):
    out = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    for c in range(C):
        for h in range(H):
            i = c * H + h
            a, b = int(cu[i]), int(cu[i + 1])
            if b <= a:
                continue
            qh = q[c * Lq:(c + 1) * Lq, h].float()
            s = (qh @ k[a:b].float().T) * scale
            out[c * Lq:(c + 1) * Lq, h] = torch.softmax(s, dim=-1) @ v[a:b].float()
    return out


def _case(cuda, C, H, Lq, D, lens, seed=0, kv_scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(C * Lq, H, D, generator=g).to(cuda, torch.bfloat16)
    T = int(sum(lens))
    k = (torch.randn(T + 7, D, generator=g) * kv_scale).to(cuda, torch.bfloat16)
    v = torch.randn(T + 7, D, generator=g).to(cuda, torch.bfloat16)
    cu = torch.zeros(C * H + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int32), 0)
    return q, k, v, cu.to(cuda)


def _check(out, ref):
    err = (out.float() - ref).abs()
    assert torch.isfinite(out.float()).all()
    assert err.max().item() <= MAX_ABS, f"max abs err {err.max().item()}"
    assert err.mean().item() <= MEAN_ABS, f"mean abs err {err.mean().item()}"


@pytest.mark.parametrize("D", [128, 64])
def test_ragged_attention_matches_fp32(cuda, D):
    from pyramidkv import _ops
    C, H, Lq = 2, 3, 1560                     # 1560 = 12 full 128-row tiles + a 24-row tail
    lens = [4680, 1560, 390, 9360, 4680 + 390, 777]   # frame / merge-anchor granular + ragged
    q, k, v, cu = _case(cuda, C, H, Lq, D, lens)
    scale = D ** -0.5
    out = _ops.ops().pkv_attention(q, k, v, cu, C, Lq, scale)
    _check(out, _reference(q, k, v, cu, C, H, Lq, scale))


def test_attention_rescale_path_and_empty_segment(cuda):
    """Large logits force the running-max rescale of O; an empty segment gives
    zeros (flash-attn's convention for seqlen_k = 0)."""
    from pyramidkv import _ops
    C, H, Lq, D = 1, 3, 200, 128
    lens = [3000, 0, 515]
    q, k, v, cu = _case(cuda, C, H, Lq, D, lens, seed=3, kv_scale=6.0)
    # ascending key magnitude so the row max keeps growing across tiles
    ramp = torch.linspace(0.2, 3.0, k.shape[0], device=cuda).unsqueeze(1)
    k = (k.float() * ramp).to(torch.bfloat16)
    out = _ops.ops().pkv_attention(q, k, v, cu, C, Lq, 0.088)
    ref = _reference(q, k, v, cu, C, H, Lq, 0.088)
    _check(out, ref)
    assert out[:, 1].abs().max().item() == 0.0


@pytest.mark.parametrize("seed", [0, 1])
def test_attention_max_jumps_between_tiles(cuda, seed):
    """Keys whose magnitude jumps from one 128-key tile to the next: a row
    maximum moving by 2^8..2^64 (log2 units) while P is formed from the old
    reference, by more than 2^64 (P redone from S), on the last full tile before a
    partial one, and on the last tile of a segment.  Query rows span two full
    tiles and a 24-row tail."""
    from pyramidkv import _ops
    C, H, Lq, D = 1, 4, 280, 128
    pattern = [[1, 6, 6, 40, 40, 1], [1, 1, 1, 6], [1, 1, 1, 1, 6, 6], [1, 1, 40]]
    tails = [7, 0, 100, 0]
    lens = [128 * (len(p_) - (1 if t else 0)) + t for p_, t in zip(pattern, tails)]
    q, k, v, cu = _case(cuda, C, H, Lq, D, lens, seed=seed)
    kf = k.float()
    cuh = cu.cpu()
    for i, pat in enumerate(pattern):
        a = int(cuh[i])
        for tile, f in enumerate(pat):
            kf[a + 128 * tile:min(a + 128 * (tile + 1), int(cuh[i + 1]))] *= f
    k = kf.to(torch.bfloat16)
    out = _ops.ops().pkv_attention(q, k, v, cu, C, Lq, 0.088)
    _check(out, _reference(q, k, v, cu, C, H, Lq, 0.088))


def test_attention_strided_q_layout(cuda):
    """Q as a non-contiguous view ([1, L_q, H, D] sliced from a wider tensor)."""
    from pyramidkv import _ops
    C, H, Lq, D = 3, 2, 320, 128
    lens = [1000, 2000, 640, 128, 1, 4000]
    q, k, v, cu = _case(cuda, C, H, Lq, D, lens, seed=7)
    wide = torch.zeros(C * Lq, H + 2, D, device=cuda, dtype=torch.bfloat16)
    wide[:, 1:H + 1] = q
    qv = wide[:, 1:H + 1]
    out = _ops.ops().pkv_attention(qv, k, v, cu, C, Lq, D ** -0.5)
    _check(out, _reference(q, k, v, cu, C, H, Lq, D ** -0.5))


def _ws(cuda, C, H, Lq):
    from pyramidkv import _ops
    n = int(_ops.ops().pkv_attention_ws_bytes(C, H, Lq))
    return torch.zeros(n, dtype=torch.uint8, device=cuda)


def _ws_counters(ws):
    """The workspace's arrival counters (after the 256-aligned partial slots)."""
    part = 160 * 4 * (130 * 128 + 32) * 4
    return ws[(part + 255) // 256 * 256:].view(torch.int32)


@pytest.mark.parametrize("seed", [0, 1])
def test_balanced_attention_c2_shape(cuda, seed):
    """The SM-balanced (persistent, split-unit) path at the C2 attend shape:
    3 chunks x 12 heads x 1560 queries over 4-19 frames of keys plus merge
    anchors, i.e. 252 units on the SMs, so units are cut between SMs and
    recombined.  Within tolerance of fp32; the workspace's counters are back
    at zero after every launch, and a second launch is bit-identical."""
    from pyramidkv import _ops
    C, H, Lq, D = 3, 12, 1560, 128
    g = torch.Generator().manual_seed(100 + seed)
    frames = torch.randint(4, 20, (C * H,), generator=g)
    lens = (frames * 1560 + (torch.rand(C * H, generator=g) < 0.3).long() * 390).tolist()
    q, k, v, cu = _case(cuda, C, H, Lq, D, lens, seed=seed)
    ws = _ws(cuda, C, H, Lq)
    scale = D ** -0.5
    out = _ops.ops().pkv_attention_ws(q, k, v, cu, C, Lq, scale, ws)
    torch.cuda.synchronize()
    assert int(_ws_counters(ws).abs().sum()) == 0
    _check(out, _reference(q, k, v, cu, C, H, Lq, scale))
    again = _ops.ops().pkv_attention_ws(q, k, v, cu, C, Lq, scale, ws)
    assert torch.equal(again.view(torch.int16), out.view(torch.int16))
    plain = _ops.ops().pkv_attention(q, k, v, cu, C, Lq, scale)
    err = (plain.float() - out.float()).abs()
    assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS


def test_balanced_attention_ragged_edges(cuda):
    """Split path with empty segments, one-key segments, lengths one off a
    128-key tile, very long and very short segments side by side, and a
    query count whose last tile has 1 row (so units hold one tile)."""
    from pyramidkv import _ops
    C, H, Lq, D = 2, 40, 257, 128            # 3 tiles: one pair + a lone 1-row tile
    g = torch.Generator().manual_seed(5)
    choices = [0, 1, 127, 128, 129, 390, 4000, 30000]
    lens = [choices[int(i)] for i in torch.randint(0, len(choices), (C * H,), generator=g)]
    lens[0], lens[1] = 60000, 0
    q, k, v, cu = _case(cuda, C, H, Lq, D, lens, seed=9)
    ws = _ws(cuda, C, H, Lq)
    out = _ops.ops().pkv_attention_ws(q, k, v, cu, C, Lq, 0.088, ws)
    torch.cuda.synchronize()
    assert int(_ws_counters(ws).abs().sum()) == 0
    ref = _reference(q, k, v, cu, C, H, Lq, 0.088)
    _check(out, ref)
    empty = [i for i, n in enumerate(lens) if n == 0]
    for i in empty:
        c, h = divmod(i, H)
        assert out[c * Lq:(c + 1) * Lq, h].abs().max().item() == 0.0


def test_balanced_attention_fewer_units_than_sms(cuda):
    """Fewer units than SMs (a head-parallel rank's share: 3 chunks x 3 heads x
    7 units = 63): every unit's keys are cut between the SMs and recombined."""
    from pyramidkv import _ops
    C, H, Lq, D = 3, 3, 1560, 128
    g = torch.Generator().manual_seed(31)
    frames = torch.randint(4, 20, (C * H,), generator=g)
    lens = (frames * 1560 + (torch.rand(C * H, generator=g) < 0.3).long() * 390).tolist()
    q, k, v, cu = _case(cuda, C, H, Lq, D, lens, seed=4)
    ws = _ws(cuda, C, H, Lq)
    scale = D ** -0.5
    out = _ops.ops().pkv_attention_ws(q, k, v, cu, C, Lq, scale, ws)
    torch.cuda.synchronize()
    assert int(_ws_counters(ws).abs().sum()) == 0
    _check(out, _reference(q, k, v, cu, C, H, Lq, scale))
    again = _ops.ops().pkv_attention_ws(q, k, v, cu, C, Lq, scale, ws)
    assert torch.equal(again.view(torch.int16), out.view(torch.int16))
