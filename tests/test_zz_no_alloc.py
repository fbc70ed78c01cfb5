"""The allocation-free attend entry point, called through the C ABI.

Some callers of this library cannot let it allocate device memory: a host
runtime that owns the device's memory pool and lends the library only the
cache and each call's inputs and outputs, or a serving loop where a cudaMalloc
could synchronise the device.  ``pkv_attend_noalloc`` serves them, with the
planner's scratch in a fixed device array inside libpkv.so.  This test builds a
cache through the normal API, then on consecutive calls (layer 0 and layer 1
over three chunks, then layer 0 over one chunk, so a smaller plan follows a
larger one in the shared array) compares the allocation-free entry point --
called with ctypes and a cache descriptor that has no scratch buffer -- with
the existing attend path.  At these sizes (at most 12 attention units, fewer
than the SMs) both run the same plan, pack and one-CTA-per-unit attention, so
cu_seqlens_k, the packed K/V/positions and the output must be bit-identical.
It also checks that a plan larger than the fixed array is refused before
anything launches.  The file sorts last, so a run that stops at the first
failure has already run every other test.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

LIBPKV = os.path.join(ROOT, "pyramid-forcing_b200", "pyramidkv", "lib", "libpkv.so")
P, I32, I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
PKV_ENOALLOC_LIMIT = 5


class PkvCache(ctypes.Structure):
    """ctypes mirror of pkv_cache_t (include/pkv.h)."""
    _fields_ = ([(n, I32) for n in ("num_layers", "num_heads", "head_dim", "frame_seqlen",
                                    "max_sink", "max_middle", "max_recent", "max_merge_blocks",
                                    "max_merge_active", "max_merge_tokens", "max_attend_chunks",
                                    "spatial_width")]
                + [("max_pack_tokens", I64)]
                + [(n, P) for n in ("sink_k", "sink_v", "middle_k", "middle_v", "recent_k",
                                    "recent_v", "sink_pos", "middle_pos", "recent_pos",
                                    "valid_count", "merge_k", "merge_v", "merge_pos",
                                    "merge_token_count", "accum_sum_k", "accum_sum_v",
                                    "accum_pos", "accum_group_ids", "accum_tokens_per_group",
                                    "accum_num_groups", "k_flat", "v_flat", "pos_flat",
                                    "cu_seqlens_k", "committed_vc", "committed_recent_k",
                                    "committed_recent_v", "committed_recent_pos", "sink_caps",
                                    "scratch")]
                + [("scratch_bytes", I64), ("status", P), ("first_t_dev", P)])


def _describe(ctx) -> PkvCache:
    """Descriptor of the cache that ``ctx`` owns, with no scratch buffer."""
    m = ctx.mgr
    c = PkvCache()
    c.num_layers, c.num_heads, c.head_dim, c.frame_seqlen = (
        m.num_layers(), m.num_heads(), m.head_dim(), m.frame_seqlen())
    c.max_sink, c.max_middle, c.max_recent = m.max_sink(), m.max_middle(), m.max_recent()
    c.max_merge_blocks, c.max_merge_active = m.max_merge_blocks(), m.max_merge_active()
    c.max_merge_tokens = m.max_merge_tokens_per_anchor()
    c.max_attend_chunks, c.spatial_width = m.max_attend_chunks(), ctx.spatial_width
    c.max_pack_tokens = m.max_pack_tokens()
    for name, t in (("sink_k", m.sink_k_pool()), ("sink_v", m.sink_v_pool()),
                    ("middle_k", m.middle_k_pool()), ("middle_v", m.middle_v_pool()),
                    ("recent_k", m.recent_k_pool()), ("recent_v", m.recent_v_pool()),
                    ("sink_pos", m.sink_pos_pool()), ("middle_pos", m.middle_pos_pool()),
                    ("recent_pos", m.recent_pos_pool()), ("valid_count", m.valid_count()),
                    ("merge_k", m.merge_k_pool()), ("merge_v", m.merge_v_pool()),
                    ("merge_pos", m.merge_pos_pool()), ("merge_token_count", m.merge_token_count()),
                    ("k_flat", m.k_flat_out()), ("v_flat", m.v_flat_out()),
                    ("pos_flat", m.pos_flat_out()), ("cu_seqlens_k", m.cu_seqlens_k()),
                    ("status", m.status_word())):
        setattr(c, name, t.data_ptr())
    c.scratch, c.scratch_bytes = None, 0       # the entry point must not need it
    return c


def _lib():
    lib = ctypes.CDLL(LIBPKV)
    f = lib.pkv_attend_noalloc
    f.restype = ctypes.c_int
    f.argtypes = ([ctypes.POINTER(PkvCache), P, ctypes.c_int, P, I64, I64, ctypes.c_int, I64]
                  + [ctypes.c_int] * 4 + [P, ctypes.c_int, ctypes.c_int] * 3
                  + [ctypes.c_float, P, I64, I64, P, P])
    return lib


def _caches(cuda):
    from oracle import pkv_oracle as O
    from pyramidkv import _mega_cache, policy
    _, full = O.rope_freq_tables(128)
    labels = np.array([[-1, 1, 2, 2], [2, 1, -1, 1]])
    return _mega_cache.build_mega_caches(
        2, 4, 128, 13 * 8, 3, 24, 4, policy.compositions_from_labels(labels), device="cuda:0",
        sink_time_mapping_mode="window_clamp", sink_time_clamp_min=18, sink_time_clamp_max=21,
        spatial_width=13, spatial_height=8, freqs=full)


def test_attend_noalloc_matches_attend_on_consecutive_calls(cuda):
    caches = _caches(cuda)
    ctx = caches[0].ctx
    FSEQ, H, D, F = 104, 4, 128, 3
    g = torch.Generator(device="cpu").manual_seed(5)
    rnd = lambda: torch.randn(1, F * FSEQ, H, D, generator=g).to(cuda, torch.bfloat16)  # noqa
    for blk in range(7):
        for mode in ("noisy", "clean"):
            for c in caches:
                c.update(rnd(), rnd(), blk * F * FSEQ, cache_update_mode=mode)
    lib = _lib()
    desc = _describe(ctx)
    stream = torch.cuda.current_stream().cuda_stream
    start = 7 * F * FSEQ
    mgr = ctx.mgr
    for call, (layer, chunks) in enumerate(((0, F), (1, F), (0, 1))):
        q = rnd()[:, :chunks * FSEQ]
        want = caches[layer].attend(q, start)      # existing entry point (allocating path)
        torch.cuda.synchronize()
        cu_want = mgr.cu_seqlens_k()[:chunks * H + 1].clone()
        total = int(cu_want[-1])
        packed_want = [t[:total].clone() for t in (mgr.k_flat_out(), mgr.v_flat_out(),
                                                   mgr.pos_flat_out())]
        for t in (mgr.k_flat_out(), mgr.v_flat_out(), mgr.pos_flat_out(), mgr.cu_seqlens_k()):
            t.zero_()                               # the entry point must rewrite them
        ft, fy, fx = ctx.freq_parts_flat
        got = torch.empty_like(q)
        rc = lib.pkv_attend_noalloc(
            ctypes.byref(desc), caches[layer].states_bytes_for_layer.data_ptr(), layer,
            q.data_ptr(), q.stride(1), q.stride(2), chunks, start // FSEQ, 1,
            ctx.sink_time_clamp_min, ctx.sink_time_clamp_max, ctx.decoupled_sink_time_lag,
            ft.data_ptr(), ft.shape[0], ft.shape[1] // 2, fy.data_ptr(), fy.shape[0],
            fy.shape[1] // 2, fx.data_ptr(), fx.shape[0], fx.shape[1] // 2, D ** -0.5,
            got.data_ptr(), got.stride(1), got.stride(2), None, stream)
        assert rc == 0, f"call {call}: rc={rc}"
        torch.cuda.synchronize()
        assert torch.equal(mgr.cu_seqlens_k()[:chunks * H + 1], cu_want), call
        for name, t, w in zip(("k", "v", "pos"), (mgr.k_flat_out(), mgr.v_flat_out(),
                                                   mgr.pos_flat_out()), packed_want):
            assert torch.equal(t[:total], w), (call, name)
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), call
    assert ctx.check_status() == 0


def test_attend_noalloc_refuses_oversize_plan(cuda):
    caches = _caches(cuda)
    lib = _lib()
    big = _describe(caches[0].ctx)
    big.num_heads = 4096            # 8 chunks x 4096 heads x its segments: far past the array
    big.max_attend_chunks = 8
    rc = lib.pkv_attend_noalloc(ctypes.byref(big), caches[0].states_bytes_for_layer.data_ptr(),
                                0, 16, 0, 0, 8, 0, 1, 18, 21, 0, None, 0, 0, None, 0, 0, None, 0,
                                0, 0.1, 16, 0, 0, None, None)
    assert rc == PKV_ENOALLOC_LIMIT     # returned before any launch
    err = lib.pkv_error_string
    err.restype, err.argtypes = ctypes.c_char_p, [ctypes.c_int]
    assert b"allocation-free" in err(rc)
