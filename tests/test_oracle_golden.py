"""The CPU oracle against the reference's own outputs (golden fixtures).

Fixtures come from tests/golden/make_golden.py, which drove the reference's
Python modules: the state-machine mirror (pyramidkv/_mega_state_ref.py), the
RoPE (pyramidkv/rope.py), the freq-table construction
(wan/modules/model.py:rope_params + pyramidkv/_mega_cache.py:715-731) and the
factory routing (pyramidkv/factory.py).
"""
from __future__ import annotations

import numpy as np
import torch

from conftest import golden
from oracle import pkv_oracle as O


def _mask(b, untracked):
    b = b.copy().reshape(-1, 600)
    for lo, hi in untracked:
        b[:, lo:hi] = 0
    return b.reshape(-1)


def test_state_record_size_and_offsets():
    from pyramidkv._mega_state_ops import PER_HEAD_STATE_DTYPE as DT
    assert O.state_size() == 600 == DT.itemsize
    names = ["cyclic_cursor", "tkey_slot", "tkey_count", "merge_completed_slot",
             "merge_completed_count", "merge_active_block_id", "merge_active_seen",
             "cached_num_groups"]
    for i, n in enumerate(names):
        assert O.lib().orc_state_offset(i) == DT.fields[n][1], n


def test_state_machine_matches_reference_sequences():
    g = golden("state_sequences.npz")
    unt = g["untracked"]
    for i in range(int(g["n_cases"])):
        H = int(g[f"c{i}_H"])
        st = g[f"c{i}_init"].copy()
        for j in range(g[f"c{i}_t"].shape[0]):
            d = O.state_update(st, g[f"c{i}_t"][j], int(g[f"c{i}_pk"][j]), H)
            np.testing.assert_array_equal(np.stack(d), g[f"c{i}_desc"][j], err_msg=f"case {i} call {j}")
            np.testing.assert_array_equal(_mask(st, unt), _mask(g[f"c{i}_after"][j], unt),
                                          err_msg=f"case {i} call {j}")


def test_sink_time_matches_reference():
    g = golden("sink_time.npz")
    for i, m in enumerate(g["modes"]):
        lo, hi, lag = (int(x) for x in g["params"][i])
        got = [O.map_sink_time(int(t), str(m), lo, hi, lag) for t in g["t"]]
        np.testing.assert_array_equal(got, g["table"][i])


def test_freq_tables_match_reference():
    g = golden("freq_tables.npz")
    (ft, fy, fx), _ = O.rope_freq_tables(128)
    rows = g["rows"]
    for mine, n in ((ft, "ft"), (fy, "fy"), (fx, "fx")):
        np.testing.assert_array_equal(mine[rows], g[n])


def _pack_rope(k, pos, tables, mode):
    T = k.shape[0]
    kout = np.zeros_like(k)
    vout = np.zeros_like(k)
    sk = np.array([1], np.int32)
    z = np.array([0], np.int32)
    ft, fy, fx = tables
    P = O._p
    O.lib().orc_pack(None, None, P(k), P(k), None, None, None, None, None,
                     P(np.ascontiguousarray(pos)), None, None, P(kout), P(vout), None, P(sk),
                     P(z), P(np.array([T], np.int32)), P(z), 1, P(np.array([-1], np.int64)),
                     P(ft), ft.shape[0], ft.shape[1] // 2, P(fy), fy.shape[0], fy.shape[1] // 2,
                     P(fx), fx.shape[0], fx.shape[1] // 2, T, 420, 128, mode)
    return kout


def test_rope_matches_reference_torch_rotation():
    """Unfused evaluation order == the reference's torch RoPE, bit for bit
    (clamped rows included); the FMA orders differ from it in <0.01% of
    elements by one bf16 ulp."""
    g = golden("rope_cases.npz")
    tables, _ = O.rope_freq_tables(128)
    out = _pack_rope(g["k"], g["pos"], tables, O.ROPE_NO_FMA)
    np.testing.assert_array_equal(out, g["out"])
    for mode in (O.ROPE_FMA_FIRST, O.ROPE_FMA_SECOND):
        o = _pack_rope(g["k"], g["pos"], tables, mode)
        assert (o != g["out"]).mean() < 1e-4
        diff = np.abs(O.bf16_to_f32(o) - O.bf16_to_f32(g["out"]))
        assert diff.max() <= np.abs(O.bf16_to_f32(g["out"])).max() * 2 ** -7


def test_policy_routing_matches_reference_factory():
    from pyramidkv import policy
    g = golden("compositions.npz")
    for r in ("yaml", "baseline"):
        s, c = policy.states_from_labels(g["labels"], r)
        np.testing.assert_array_equal(s, g[f"{r}_states"])
        np.testing.assert_array_equal(c, g[f"{r}_sink_caps"])


def test_bf16_rounding_helpers():
    x = np.random.default_rng(1).standard_normal(10000).astype(np.float32) * 7
    ours = O.f32_to_bf16(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(ours, ref)
    np.testing.assert_array_equal(O.bf16_to_f32(ours),
                                  torch.from_numpy(x).to(torch.bfloat16).float().numpy())


def test_build_mega_caches_state_bytes_match_reference_factory():
    """The state bytes build_mega_caches uploads, for the reference factory's
    compositions of a 30x12 label matrix (both routings)."""
    from pyramidkv import _mega_cache, policy
    g = golden("compositions.npz")
    for r in ("yaml", "baseline"):
        comps = policy.compositions_from_labels(g["labels"], r)
        raw, caps, any_merge = _mega_cache._states_from_compositions(comps, 30, 12)
        np.testing.assert_array_equal(raw, g[f"{r}_states"])
        np.testing.assert_array_equal(caps, g[f"{r}_sink_caps"])
        assert any_merge
