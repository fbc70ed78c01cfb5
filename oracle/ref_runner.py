"""Run the reference's own CUDA extension on recorded inputs (test infrastructure).

    python oracle/ref_runner.py <cases.npz> <out.npz>

Loads ``oracle/_ref/adahead_ref.so`` -- the reference's pyramidkv/csrc built
from its sources by oracle/Makefile.ref -- and runs the ops named in the input
file through the reference's own ``torch.ops.adahead`` / manager class.  It
must run in its own process: the reference registers the same ``adahead``
namespace as the product library.  Only tests spawn it.

Input keys per case i (prefix ``c{i}_``): ``op`` plus the op's arrays;
outputs are written back under the same prefix.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "adahead_ref.so")


def _bf(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).astype(np.uint16).view(np.int16)) \
        .view(torch.bfloat16).to(dev)


def _u16(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _mgr(dims):
    L, H, D, F, ms, mm, mr, mac = (int(x) for x in dims)
    return torch.classes.adahead.PyramidKVCacheManager(L, H, D, F, ms, mm, mr, "cuda:0",
                                                       "bfloat16", mac)


def run_state(c, dev, out, p):
    st = torch.from_numpy(c[p + "states"].copy()).to(dev)
    H, F = int(c[p + "H"]), int(c[p + "F"])
    descs = []
    for j, tv in enumerate(c[p + "t"]):
        d = [torch.full((H * F,), 7, dtype=torch.int32, device=dev) for _ in range(8)]
        torch.ops.adahead.mega_state_update(st, torch.from_numpy(tv).to(dev), *d, H, F,
                                            int(c[p + "pk"][j]))
        descs.append(np.stack([x.cpu().numpy() for x in d]))
    out[p + "desc"] = np.stack(descs)
    out[p + "states"] = st.cpu().numpy()


def run_plan(c, dev, out, p):
    mgr = _mgr(c[p + "dims"])
    mgr.valid_count().copy_(torch.from_numpy(c[p + "vc"]))
    mgr.merge_token_count().copy_(torch.from_numpy(c[p + "mtc"]))
    args = [int(x) for x in c[p + "modes"]]  # sink_mode, cmin, cmax, lag
    res = torch.ops.adahead.mega_plan_multi(
        mgr, torch.from_numpy(c[p + "states"]).to(dev), int(c[p + "layer"]),
        torch.from_numpy(c[p + "ct"]), 1, args[0], args[1], args[2], args[3], 0, 21, 1.0)
    for name, t in zip(("cu", "sk", "sg", "sl", "dst", "traw", "tremap"), res):
        out[p + name] = t.cpu().numpy()


def _load_pools(mgr, c, p, dev):
    for name in ("sink", "middle", "recent"):
        getattr(mgr, f"{name}_k_pool")().copy_(_bf(c[p + name + "_k"], dev).view(
            getattr(mgr, f"{name}_k_pool")().shape))
        getattr(mgr, f"{name}_v_pool")().copy_(_bf(c[p + name + "_v"], dev).view(
            getattr(mgr, f"{name}_v_pool")().shape))
        getattr(mgr, f"{name}_pos_pool")().copy_(torch.from_numpy(c[p + name + "_pos"]))
    mgr.merge_k_pool().copy_(_bf(c[p + "merge_k"], dev).view(mgr.merge_k_pool().shape))
    mgr.merge_v_pool().copy_(_bf(c[p + "merge_v"], dev).view(mgr.merge_v_pool().shape))
    mgr.merge_pos_pool().copy_(torch.from_numpy(c[p + "merge_pos"]))


def run_pack(c, dev, out, p):
    mgr = _mgr(c[p + "dims"])
    _load_pools(mgr, c, p, dev)
    t = lambda k: torch.from_numpy(c[p + k]).to(dev)  # noqa: E731
    rope = int(c[p + "rope"])
    e64 = torch.empty(0, dtype=torch.int64, device=dev)
    e32 = torch.empty(0, dtype=torch.float32, device=dev)
    torch.ops.adahead.pyramidkv_pack(mgr, t("sk"), t("sg"), t("sl"), t("dst"),
                                     t("tremap") if rope else e64,
                                     t("ft") if rope else e32, t("fy") if rope else e32,
                                     t("fx") if rope else e32)
    total = int(c[p + "total"])
    out[p + "k"] = _u16(mgr.k_flat_out()[:total]).reshape(total, -1)
    out[p + "v"] = _u16(mgr.v_flat_out()[:total]).reshape(total, -1)
    out[p + "pos"] = mgr.pos_flat_out()[:total].cpu().numpy()


def run_merge(c, dev, out, p):
    mgr = _mgr(c[p + "dims"])
    st = torch.from_numpy(c[p + "states"].copy()).to(dev)
    H, Fb = int(c[p + "H"]), int(c[p + "Fb"])
    for j in range(c[p + "t"].shape[0]):
        tv = torch.from_numpy(c[p + "t"][j]).to(dev)
        d = [torch.full((H * Fb,), -1, dtype=torch.int32, device=dev) for _ in range(8)]
        torch.ops.adahead.mega_state_update(st, tv, *d, H, Fb, 1)
        dk = torch.where(d[0] == 5, d[0], torch.full_like(d[0], -1))
        nk = _bf(c[p + "nk"][j], dev)
        nv = _bf(c[p + "nv"][j], dev)
        pos = torch.from_numpy(c[p + "pos"][j]).to(dev)
        torch.ops.adahead.mega_merge_accum(
            st, nk, nv, pos, dk, d[4], d[6], d[7], mgr.merge_accum_sum_k()[0],
            mgr.merge_accum_sum_v()[0], mgr.merge_accum_pos()[0], mgr.merge_accum_group_ids()[0],
            mgr.merge_accum_tokens_per_group()[0], mgr.merge_accum_num_groups()[0],
            mgr.merge_k_pool()[0], mgr.merge_v_pool()[0], mgr.merge_pos_pool()[0],
            mgr.merge_token_count()[0])
    out[p + "states"] = st.cpu().numpy()
    out[p + "acc_k"] = mgr.merge_accum_sum_k()[0].cpu().numpy()
    out[p + "acc_v"] = mgr.merge_accum_sum_v()[0].cpu().numpy()
    out[p + "mk"] = _u16(mgr.merge_k_pool()[0])
    out[p + "mv"] = _u16(mgr.merge_v_pool()[0])
    out[p + "mpos"] = mgr.merge_pos_pool()[0].cpu().numpy()
    out[p + "mtc"] = mgr.merge_token_count()[0].cpu().numpy()
    out[p + "tpg"] = mgr.merge_accum_tokens_per_group()[0].cpu().numpy()


def run_legacy(c, dev, out, p):
    """refresh_readout_layout, anchor_store_write_frames and scatter_copy of the
    reference on the recorded sources (one call each)."""
    n = int(c[p + "nseg"])
    sk = [_bf(c[p + f"sk{s}"], dev) for s in range(n)]
    sv = [_bf(c[p + f"sv{s}"], dev) for s in range(n)]
    sp = [torch.from_numpy(c[p + f"sp{s}"]).to(dev) for s in range(n)]
    t = lambda k: torch.from_numpy(c[p + k]).to(dev)  # noqa: E731
    rows, D = int(c[p + "rows"]), int(c[p + "D"])
    dk = torch.zeros(rows, D, dtype=torch.bfloat16, device=dev)
    dv = torch.zeros_like(dk)
    dp = torch.full((rows, 3), -7, dtype=torch.int64, device=dev)
    df = torch.full((rows,), -7, dtype=torch.int64, device=dev)
    ptr = lambda: torch.empty(n, dtype=torch.int64, device=dev)  # noqa: E731
    torch.ops.adahead.refresh_readout_layout(
        sk, sv, sp, ptr(), ptr(), ptr(), t("off"), t("len"), t("flags"), t("rope_t"), dk, dv, dp,
        df, D, int(c[p + "cur"]), str(c[p + "mode"]), int(c[p + "relmax"]),
        float(c[p + "soft"]))
    out[p + "dk"], out[p + "dv"] = _u16(dk), _u16(dv)
    out[p + "dp"], out[p + "df"] = dp.cpu().numpy(), df.cpu().numpy()
    # anchor_store_write_frames
    kq, vq = _bf(c[p + "kseq"], dev), _bf(c[p + "vseq"], dev)
    pq = t("pseq")
    cap, F = int(c[p + "cap"]), int(c[p + "F"])
    stk = torch.zeros(cap, F, D, dtype=torch.bfloat16, device=dev)
    stv = torch.zeros_like(stk)
    stp = torch.zeros(cap, F, 3, dtype=torch.int64, device=dev)
    torch.ops.adahead.anchor_store_write_frames(kq, vq, pq, t("fdesc"), stk, stv, stp)
    out[p + "stk"], out[p + "stv"], out[p + "stp"] = _u16(stk), _u16(stv), stp.cpu().numpy()
    # scatter_copy of the same sources into a flat workspace
    ws = torch.zeros(rows, D, dtype=torch.bfloat16, device=dev)
    ptrs = torch.tensor([x.data_ptr() for x in sk], dtype=torch.int64, device=dev)
    torch.ops.adahead.scatter_copy(ptrs, t("len"), t("off"), ws, D)
    out[p + "ws"] = _u16(ws)


RUNNERS = {"state": run_state, "plan": run_plan, "pack": run_pack, "merge": run_merge,
           "legacy": run_legacy}


def main(inp: str, outp: str) -> None:
    torch.ops.load_library(REF_SO)
    dev = torch.device("cuda:0")
    c = np.load(inp)
    out = {}
    for i in range(int(c["n_cases"])):
        p = f"c{i}_"
        RUNNERS[str(c[p + "op"])](c, dev, out, p)
    torch.cuda.synchronize()
    np.savez(outp, **out)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2])
