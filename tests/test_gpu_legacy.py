"""The AdaptiveKVCache / CppStrategyManager ops on the GPU: product library vs
the CPU oracle and vs the reference's own compiled kernels
(oracle/_ref/adahead_ref.so, run in a child process by oracle/ref_runner.py),
bit for bit, on ragged segments with every flag combination of
refresh_readout_layout, both history mappings, unaligned row sizes and
skipped frames."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT
from oracle import pkv_oracle as O

pytestmark = pytest.mark.gpu
REF_SO = os.path.join(ROOT, "oracle", "_ref", "adahead_ref.so")


def _case(rng, D=128, mode="relative_softcap"):
    lens = [37, 0, 128, 5, 64, 17, 1, 90]
    n = len(lens)
    offs = np.cumsum([0] + lens[:-1]).astype(np.int64) + 3
    rows = int(offs[-1] + lens[-1] + 5)
    c = dict(op="legacy", nseg=n, D=D, rows=rows, off=offs, len=np.array(lens, np.int64),
             flags=np.array([i % 8 for i in range(n)], np.int64),
             rope_t=rng.integers(0, 40, n).astype(np.int64), cur=np.array(30),
             mode=np.array(mode), relmax=np.array(6), soft=np.array(0.37))
    for s, L in enumerate(lens):
        Lm = max(L, 1)
        c[f"sk{s}"] = O.f32_to_bf16(rng.standard_normal((Lm, D)).astype(np.float32))
        c[f"sv{s}"] = O.f32_to_bf16(rng.standard_normal((Lm, D)).astype(np.float32))
        c[f"sp{s}"] = np.stack([rng.integers(-3, 35, Lm), rng.integers(0, 30, Lm),
                                rng.integers(0, 52, Lm)], 1).astype(np.int64)
    F, nf, cap = 24, 5, 6
    c.update(F=np.array(F), cap=np.array(cap),
             kseq=O.f32_to_bf16(rng.standard_normal((nf * F, D)).astype(np.float32)),
             vseq=O.f32_to_bf16(rng.standard_normal((nf * F, D)).astype(np.float32)),
             pseq=rng.integers(0, 99, (nf * F, 3)).astype(np.int64),
             fdesc=np.array([[0, 2], [3, 0], [-1, 1], [4, -1], [1, 5]], np.int64))
    return c


def _bf(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)


def _u16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _mode_code(m):
    return {"relative_clamp": 1, "relative_softcap": 2}.get(m, 0)


def _ours(c, dev):
    from pyramidkv import _ops
    ops = _ops.ops()
    n, D, rows = int(c["nseg"]), int(c["D"]), int(c["rows"])
    sk = [_bf(c[f"sk{s}"], dev) for s in range(n)]
    sv = [_bf(c[f"sv{s}"], dev) for s in range(n)]
    sp = [torch.from_numpy(c[f"sp{s}"]).to(dev) for s in range(n)]
    t = lambda k: torch.from_numpy(np.asarray(c[k])).to(dev)  # noqa: E731
    dk = torch.zeros(rows, D, dtype=torch.bfloat16, device=dev)
    dv = torch.zeros_like(dk)
    dp = torch.full((rows, 3), -7, dtype=torch.int64, device=dev)
    df = torch.full((rows,), -7, dtype=torch.int64, device=dev)
    ptr = lambda: torch.empty(n, dtype=torch.int64, device=dev)  # noqa: E731
    ops.refresh_readout_layout(sk, sv, sp, ptr(), ptr(), ptr(), t("off"), t("len"), t("flags"),
                               t("rope_t"), dk, dv, dp, df, D, int(c["cur"]), str(c["mode"]),
                               int(c["relmax"]), float(c["soft"]))
    cap, F = int(c["cap"]), int(c["F"])
    stk = torch.zeros(cap, F, D, dtype=torch.bfloat16, device=dev)
    stv = torch.zeros_like(stk)
    stp = torch.zeros(cap, F, 3, dtype=torch.int64, device=dev)
    ops.anchor_store_write_frames(_bf(c["kseq"], dev), _bf(c["vseq"], dev), t("pseq"),
                                  t("fdesc"), stk, stv, stp)
    ws = torch.zeros(rows, D, dtype=torch.bfloat16, device=dev)
    ptrs = torch.tensor([x.data_ptr() for x in sk], dtype=torch.int64, device=dev)
    ops.scatter_copy(ptrs, t("len"), t("off"), ws, D)
    torch.cuda.synchronize()
    return dict(dk=_u16(dk), dv=_u16(dv), dp=dp.cpu().numpy(), df=df.cpu().numpy(),
                stk=_u16(stk), stv=_u16(stv), stp=stp.cpu().numpy(), ws=_u16(ws))


def _oracle(c):
    n, D, rows = int(c["nseg"]), int(c["D"]), int(c["rows"])
    sk = [c[f"sk{s}"] for s in range(n)]
    sv = [c[f"sv{s}"] for s in range(n)]
    sp = [c[f"sp{s}"] for s in range(n)]
    dk = np.zeros((rows, D), np.uint16); dv = np.zeros_like(dk)
    dp = np.full((rows, 3), -7, np.int64); df = np.full(rows, -7, np.int64)
    O.legacy_refresh(sk, sv, sp, c["off"], c["len"], c["flags"], c["rope_t"], dk, dv, dp, df,
                     int(c["cur"]), _mode_code(str(c["mode"])), int(c["relmax"]),
                     float(c["soft"]))
    cap, F = int(c["cap"]), int(c["F"])
    stk = np.zeros((cap, F, D), np.uint16); stv = np.zeros_like(stk)
    stp = np.zeros((cap, F, 3), np.int64)
    O.legacy_write_frames(c["kseq"], c["vseq"], c["pseq"], c["fdesc"], stk, stv, stp)
    ws = np.zeros((rows, D), np.uint16)
    O.legacy_scatter_copy(sk, c["len"], c["off"], ws)
    return dict(dk=dk, dv=dv, dp=dp, df=df, stk=stk, stv=stv, stp=stp, ws=ws)


@pytest.mark.parametrize("mode", ["relative_softcap", "relative_clamp", "none"])
def test_legacy_ops_match_oracle(cuda, mode):
    c = _case(np.random.default_rng(3), mode=mode)
    got, want = _ours(c, cuda), _oracle(c)
    for k in want:
        np.testing.assert_array_equal(got[k], want[k], err_msg=k)


def test_legacy_ops_unaligned_rows(cuda):
    c = _case(np.random.default_rng(4), D=7)        # 14-byte rows: word / byte copy paths
    got, want = _ours(c, cuda), _oracle(c)
    for k in want:
        np.testing.assert_array_equal(got[k], want[k], err_msg=k)


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference extension not built")
def test_legacy_ops_match_reference_kernels(cuda, tmp_path):
    c = _case(np.random.default_rng(5))
    flat = {"n_cases": np.array(1)}
    for k, v in c.items():
        flat[f"c0_{k}"] = np.asarray(v)
    inp, outp = str(tmp_path / "cases.npz"), str(tmp_path / "out.npz")
    np.savez(inp, **flat)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "oracle", "ref_runner.py"), inp, outp],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    ref = np.load(outp)
    got = _ours(c, cuda)
    for k in got:
        np.testing.assert_array_equal(got[k], ref[f"c0_{k}"], err_msg=k)
