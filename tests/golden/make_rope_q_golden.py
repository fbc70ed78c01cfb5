"""Golden vectors of the query RoPE from the reference's own functions.

Loads ``causal_rope_apply`` (wan/modules/causal_model.py) and ``rope_params``
(wan/modules/model.py) from a reference checkout -- only those two function
definitions, parsed out of the files with ``ast`` and executed with torch, since
the surrounding modules need packages this image does not have -- and records
their outputs on seeded bf16 inputs:

    python tests/golden/make_rope_q_golden.py /path/to/reference

Writes tests/golden/rope_q.npz (inputs and outputs as bf16 bit patterns).
"""
from __future__ import annotations

import ast
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(path: str, name: str, env: dict):
    tree = ast.parse(open(path).read())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == name)
    mod = ast.Module(body=[fn], type_ignores=[])
    exec(compile(mod, path, "exec"), env)
    return env[name]


def main(ref_root: str) -> None:
    env = {"torch": torch}
    rope_params = _load(os.path.join(ref_root, "wan/modules/model.py"), "rope_params", env)
    causal_rope_apply = _load(os.path.join(ref_root, "wan/modules/causal_model.py"),
                              "causal_rope_apply", env)
    d = 128
    freqs = torch.cat([rope_params(1024, d - 4 * (d // 6)), rope_params(1024, 2 * (d // 6)),
                       rope_params(1024, 2 * (d // 6))], dim=1)
    g = torch.Generator().manual_seed(7)
    out = {}
    # (frames, grid rows, grid cols, start frame, heads, tokens past the grid)
    cases = [(3, 8, 13, 0, 2, 0), (3, 8, 13, 21, 2, 5), (1, 30, 52, 1000, 1, 0)]
    for i, (F, Hg, Wg, start, heads, pad) in enumerate(cases):
        L = F * Hg * Wg + pad
        x = (torch.randn(1, L, heads, d, generator=g) * 2).to(torch.bfloat16)
        grid = torch.tensor([[F, Hg, Wg]])
        y = causal_rope_apply(x, grid, freqs, start_frame=start)
        out[f"c{i}_x"] = x.view(torch.int16).numpy().view(np.uint16)
        out[f"c{i}_y"] = y.view(torch.int16).numpy().view(np.uint16)
        out[f"c{i}_dims"] = np.array([F, Hg, Wg, start, heads, pad])
    out["n_cases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, "rope_q.npz"), **out)
    print("wrote", os.path.join(HERE, "rope_q.npz"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_rope_q_golden.py <path of the reference checkout>")
    main(sys.argv[1])
