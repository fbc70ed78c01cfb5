"""The legacy all-layer plan (op pyramidkv_plan, M1.4) on the device.

The descriptors must equal the oracle's restatement of pyramidkv_plan.cc:48-173
bit for bit (random valid counts, some kinds empty), and planning then packing
must give the concatenation the reference's test expects
(tests/test_pyramidkv_plan.py:35-137): per (layer, head) the valid sink, recent
and middle slots, head-major.  Segments span several slots, so the packs (the
generic one at head_dim 16 and the warp-specialized one at 128) copy them
whole.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import pkv_oracle as O

pytestmark = pytest.mark.gpu


def _mgr(L, H, D, F, ms, mm, mr):
    return torch.classes.adahead.PyramidKVCacheManager(L, H, D, F, ms, mm, mr, "cuda:0",
                                                       "bfloat16", L)


def test_legacy_plan_matches_oracle(cuda):
    L, H, D, F, ms, mm, mr = 30, 12, 16, 8, 3, 24, 4
    mgr = _mgr(L, H, D, F, ms, mm, mr)
    rng = np.random.default_rng(11)
    vc = np.stack([rng.integers(0, ms + 1, (L, H)), rng.integers(0, mm + 1, (L, H)),
                   rng.integers(0, mr + 1, (L, H))], axis=-1).astype(np.int64)
    mgr.valid_count().copy_(torch.from_numpy(vc))
    got = torch.ops.adahead.pyramidkv_plan(mgr, 7, 1)
    torch.cuda.synchronize()
    want = O.legacy_plan(vc, F, ms, mm, mr)
    for name, g, w in zip(("cu", "sk", "sg", "sl", "dst"), got, want):
        assert g.dtype == torch.int32 and g.is_cuda
        np.testing.assert_array_equal(g.cpu().numpy(), w, err_msg=name)


@pytest.mark.parametrize("D,F,empty_kinds", [(16, 8, ()), (16, 8, (0, 2)), (16, 128, ()),
                                             (128, 8, ()), (128, 8, (1,))])
def test_legacy_plan_then_pack(cuda, D, F, empty_kinds):
    """F = 128 at head_dim 16: the 4-slot middle segments (512 tokens) are
    longer than the generic pack's per-segment unit span (max(F, 420))."""
    from pyramidkv import _ops
    L, H, ms, mm, mr = 2, 4, 2, 4, 2
    mgr = _mgr(L, H, D, F, ms, mm, mr)
    g = torch.Generator(device="cpu").manual_seed(42)
    for name in ("sink", "middle", "recent"):
        for kv in ("k", "v"):
            pool = getattr(mgr, f"{name}_{kv}_pool")()
            pool.copy_(torch.randn(pool.shape, generator=g).to(pool.dtype))
    counts = [ms, mm, mr]
    for k in empty_kinds:
        counts[k] = 0
    vc = mgr.valid_count()
    for kind, n in enumerate(counts):
        vc[..., kind] = n
    cu, sk, sg, sl, dst = torch.ops.adahead.pyramidkv_plan(mgr, 0, 0)
    _ops.pyramidkv_pack(mgr, sk, sg, sl, dst)
    torch.cuda.synchronize()
    assert int(torch.ops.adahead.pkv_status(mgr)) == 0
    per_head = sum(counts) * F
    assert (cu[1:] - cu[:-1] == per_head).all()
    ref = []
    for layer in range(L):
        for h in range(H):
            for name, n in (("sink", counts[0]), ("recent", counts[2]), ("middle", counts[1])):
                if n:
                    ref.append(getattr(mgr, f"{name}_k_pool")()[layer, h, :n].reshape(n * F, D))
    ref_k = torch.cat(ref, dim=0)
    total = L * H * per_head
    out_k = mgr.k_flat_out()[:total].reshape(total, D)
    assert torch.equal(out_k.view(torch.int16), ref_k.view(torch.int16))
