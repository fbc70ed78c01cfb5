"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py --reference /path/to/Pyramid-Forcing

It imports the reference's own Python modules (nothing is copied) and writes
small .npz files next to this script:

* ``state_sequences.npz`` -- the reference's state-machine mirror
  ``pyramidkv/_mega_state_ref.py:mega_state_update_ref`` (:239-333) driven
  over seeded strategies and frame sequences, with the reference's ABI packer
  ``pyramidkv/_mega_state_ops.py:pack_states`` (:104-136) producing the
  state bytes before and after every call.
* ``rope_cases.npz`` -- ``pyramidkv/rope.py:_pytorch_apply_rope_to_flat_k``
  (:18-68) on seeded bf16 keys and positions (including out-of-range rows that
  exercise the clamp) with the model's freq table
  (``wan/modules/causal_model.py:586-591``).
* ``sink_time.npz`` -- ``pyramidkv/rope.py:map_sink_time`` (:86-101).
* ``compositions.npz`` -- ``pyramidkv/factory.py:build_compositions``
  (:220-407) + ``pyramidkv/_mega_cache.py:_composition_to_perhead_state``
  (:572-628) + ``pack_states`` for a seeded 30x12 label matrix under the
  shipped yaml routing and under the BASELINE routing.

The fixtures are committed; tests read them without the reference present.
"""
from __future__ import annotations

import argparse

import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# Byte ranges of PerHeadState that the reference's Python dataclass does not
# carry (merge_completed_{start,end,median}_t and merge_active_slot); the
# reference's pack_states leaves them zero while the CUDA kernel writes them.
UNTRACKED = [(492, 564), (576, 584)]


def _mask_untracked(b: np.ndarray) -> np.ndarray:
    b = b.copy().reshape(-1, 600)
    for lo, hi in UNTRACKED:
        b[:, lo:hi] = 0
    return b.reshape(-1)


def gen_state_sequences(ref, ops, rng):
    """Seeded strategy mixes x frame sequences through the reference mirror."""
    cases = []

    def rand_state():
        k = int(rng.integers(0, 5))
        if k == ref.SK_CYCLIC:
            s = ref.make_cyclic(period=int(rng.integers(1, 7)), bucket_cap=int(rng.integers(1, 5)))
        elif k == ref.SK_STRIDE:
            s = ref.make_stride(interval=int(rng.integers(1, 9)), capacity=int(rng.integers(1, 25)))
        elif k == ref.SK_LAG:
            s = ref.make_lag(history_frames=int(rng.integers(1, 25)), offsets=[1, 3])
        elif k == ref.SK_MERGE:
            s = ref.make_merge(patch_size=int(rng.integers(1, 3)), capacity=int(rng.integers(1, 7)))
        else:
            s = ref.make_recent()
        s.sink_capacity = int(rng.integers(0, 4))
        return s

    for case in range(48):
        H = int(rng.integers(1, 13))
        F = int(rng.integers(1, 5))
        states = [rand_state() for _ in range(H)]
        init = ops.pack_states(states).view(np.uint8).reshape(-1).copy()
        n_blocks = int(rng.integers(3, 30))
        t = int(rng.integers(0, 3)) * F if case % 3 else 0
        calls_t, calls_pk, descs, after = [], [], [], []
        for _ in range(n_blocks):
            tv = list(range(t, t + F))
            for pk in ([0] * int(rng.integers(0, 2))) + [1]:
                d = ref.mega_state_update_ref(states, tv, pk)
                calls_t.append(tv)
                calls_pk.append(pk)
                descs.append(np.asarray(d, dtype=np.int32))
                after.append(ops.pack_states(states).view(np.uint8).reshape(-1).copy())
            t += F
        cases.append(dict(H=H, F=F, init=init, t=np.asarray(calls_t, np.int64),
                          pk=np.asarray(calls_pk, np.int32), desc=np.stack(descs),
                          after=np.stack(after)))

    # Out-of-order merge arrivals and a two-active-block interleave
    # (tests/test_mega_state_update_ref.py:226-330 exercise these forms).
    for order in ([3, 2, 1, 0, 7, 6, 5, 4], [0, 4, 1, 5, 2, 6, 3, 7, 8, 12, 9, 13],
                  [0, 1, 4, 5, 8, 9, 2, 3, 6, 7, 10, 11]):
        states = [ref.make_merge(patch_size=2, capacity=2)]
        init = ops.pack_states(states).view(np.uint8).reshape(-1).copy()
        calls_t, calls_pk, descs, after = [], [], [], []
        for i in range(0, len(order), 2):
            tv = order[i:i + 2]
            d = ref.mega_state_update_ref(states, tv, 1)
            calls_t.append(tv)
            calls_pk.append(1)
            descs.append(np.asarray(d, dtype=np.int32))
            after.append(ops.pack_states(states).view(np.uint8).reshape(-1).copy())
        cases.append(dict(H=1, F=2, init=init, t=np.asarray(calls_t, np.int64),
                          pk=np.asarray(calls_pk, np.int32), desc=np.stack(descs),
                          after=np.stack(after)))

    out = {}
    for i, c in enumerate(cases):
        for k, v in c.items():
            out[f"c{i}_{k}"] = np.asarray(v)
    out["n_cases"] = np.asarray(len(cases))
    out["untracked"] = np.asarray(UNTRACKED, np.int64)
    np.savez_compressed(os.path.join(HERE, "state_sequences.npz"), **out)
    return len(cases)


def gen_rope(rope, model_freqs, rng):
    import torch
    T = 768
    k = torch.from_numpy(rng.standard_normal((T, 128)).astype(np.float32)).to(torch.bfloat16)
    pos = np.stack([rng.integers(0, 48, T), rng.integers(0, 30, T), rng.integers(0, 52, T)], 1)
    # clamp coverage: rows below zero and past the table
    pos[:16, 0] = -3
    pos[16:32, 0] = 1500
    pos[32:48, 1] = 2000
    pos[48:64, 2] = -7
    pos_t = torch.from_numpy(pos.astype(np.int64))
    out = rope._pytorch_apply_rope_to_flat_k(k, pos_t, model_freqs)
    np.savez_compressed(os.path.join(HERE, "rope_cases.npz"),
                        k=k.view(torch.int16).numpy().view(np.uint16),
                        pos=pos.astype(np.int64),
                        out=out.view(torch.int16).numpy().view(np.uint16))


def gen_sink_time(rope):
    ts = np.arange(0, 320, dtype=np.int64)
    modes = [("window_clamp", 18, 21, 0), ("window_clamp", 0, 21, 0), ("lag", 0, 21, 0),
             ("lag", 0, 21, 3), ("window_clamp", 5, 9, 0)]
    table = np.zeros((len(modes), ts.size), np.int64)
    for i, (m, lo, hi, lag) in enumerate(modes):
        for j, t in enumerate(ts):
            table[i, j] = rope.map_sink_time(int(t), m, lo, hi, lag)
    np.savez_compressed(os.path.join(HERE, "sink_time.npz"), t=ts, table=table,
                        modes=np.asarray([m for m, *_ in modes]),
                        params=np.asarray([p[1:] for p in modes], np.int64))


def gen_compositions(factory, mega_cache, ops, rng):
    L, H = 30, 12
    labels = rng.choice(np.asarray([-1, 1, 2]), size=(L, H))
    common = dict(
        cyclic_enabled=True, cyclic_period=6, cyclic_bucket_cap=4,
        stride_enabled=True, stride_interval=6, stride_capacity=4,
        merge_enabled=True, merge_patch_size=2, merge_capacity=4,
        label_sink_frames_map={"-1": 1, "1": 3, "2": 3},
        label_recent_frames_map={"-1": 4, "1": 4, "2": 4},
        label_stride_interval_map={"1": 6},
        label_merge_patch_size_map={"-1": 2, "2": 2},
        label_merge_capacity_map={"-1": 4, "2": 4},
    )
    routings = {
        # configs/pyramid-forcing.yaml:112-131
        "yaml": dict(cyclic_osc_only=True,
                     label_phase_bucket_map={"-1": 4, "1": 0, "2": 0},
                     label_stride_enabled_map={"1": True, "2": False},
                     label_merge_enabled_map={"-1": False, "1": False, "2": True}),
        # BASELINE routing: stride for 1, periodic for 2, merge for -1
        "baseline": dict(cyclic_osc_only=False,
                         label_phase_bucket_map={"2": 4, "-1": 0, "1": 0},
                         label_stride_enabled_map={"1": True, "2": False},
                         label_merge_enabled_map={"-1": True, "1": False, "2": False}),
    }
    out = {"labels": labels.astype(np.int32)}
    with tempfile.TemporaryDirectory() as td:
        csv = os.path.join(td, "labels.csv")
        with open(csv, "w") as f:
            # one row per layer, no header (pyramidkv/factory.py:105-127)
            for l in range(L):
                f.write(",".join(str(int(x)) for x in labels[l]) + "\n")
        for name, r in routings.items():
            comps = factory.build_compositions(L, H, [[32760] * H] * L, csv, **common, **r)
            states = np.zeros((L, H * 600), np.uint8)
            caps = np.zeros((L, H), np.int64)
            for l in range(L):
                per = [mega_cache._composition_to_perhead_state(c) for c in comps[l]]
                states[l] = ops.pack_states(per).view(np.uint8).reshape(-1)
                caps[l] = [s.sink_capacity for s in per]
            out[f"{name}_states"] = states
            out[f"{name}_sink_caps"] = caps
    np.savez_compressed(os.path.join(HERE, "compositions.npz"), **out)


def model_freqs(reference: str, d: int):
    """The model's RoPE table, as wan/modules/causal_model.py:586-591 builds it.

    ``rope_params`` is taken from the reference's wan/modules/model.py source
    by AST (importing that module needs diffusers, absent here).
    """
    import ast
    import torch
    path = os.path.join(reference, "wan", "modules", "model.py")
    tree = ast.parse(open(path).read())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "rope_params")
    ns = {"torch": torch}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), path, "exec"), ns)
    rp = ns["rope_params"]
    return torch.cat([rp(1024, d - 4 * (d // 6)), rp(1024, 2 * (d // 6)),
                      rp(1024, 2 * (d // 6))], dim=1)


def gen_freq_tables(full):
    """fp32 flat (re, im) tables as pyramidkv/_mega_cache.py:715-731 builds them."""
    import torch
    c = full.shape[1]
    split = [c - 2 * (c // 3), c // 3, c // 3]
    parts = full.split(split, dim=1)
    flat = [torch.view_as_real(z.to(torch.complex64)).contiguous().view(z.shape[0], -1).numpy()
            for z in parts]
    rows = np.r_[0:96, 1023]
    np.savez_compressed(os.path.join(HERE, "freq_tables.npz"), rows=rows,
                        ft=flat[0][rows], fy=flat[1][rows], fx=flat[2][rows])


def gen_api(reference: str):
    """The reference's torch library surface (op schemas, class methods), read
    as text from pyramidkv/csrc/scatter_copy_bind.cpp:763-945."""
    import json
    import re
    src = open(os.path.join(reference, "pyramidkv", "csrc", "scatter_copy_bind.cpp")).read()
    body = src[src.index("TORCH_LIBRARY(adahead, m)"):src.index("TORCH_LIBRARY_IMPL(adahead, CUDA")]
    methods = re.findall(r'\.def\("([A-Za-z_0-9]+)"', body)
    schemas = []
    for block in re.findall(r'm\.def\(\s*((?:"[^"]*"\s*)+)\)', body):
        schemas.append("".join(re.findall(r'"([^"]*)"', block)))
    with open(os.path.join(HERE, "adahead_api.json"), "w") as f:
        json.dump({"class_methods": methods, "schemas": schemas}, f, indent=1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from pyramidkv import _mega_state_ref as ref
    from pyramidkv import _mega_state_ops as ops
    from pyramidkv import rope, factory
    from pyramidkv import _mega_cache as mega_cache
    import torch

    rng = np.random.default_rng(20261201)
    n = gen_state_sequences(ref, ops, rng)
    full = model_freqs(args.reference, 128)
    gen_freq_tables(full)
    gen_rope(rope, full, rng)
    gen_sink_time(rope)
    gen_compositions(factory, mega_cache, ops, rng)
    gen_api(args.reference)
    del torch
    print(f"wrote {n} state cases + rope, sink_time, compositions fixtures to {HERE}")


if __name__ == "__main__":
    main()
