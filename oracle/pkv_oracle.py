"""CPU oracle for the Pyramid Forcing MegaCache hot path.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, by ``__graft_entry__.smoke()``
and by ``bench.py``'s CPU-baseline leg, always as the checker.  The product
package never imports this module.

Layers:

* ``lib()`` -- ctypes handle on ``oracle/libpkv_oracle.so`` (built from
  ``oracle/pkv_oracle.c`` by ``oracle/Makefile``), the C restatement of the
  reference's state machine, planner, frame scatter, merge accumulation and
  pack+RoPE kernels.
* ``OracleMegaCache`` -- numpy restatement of the orchestration in
  ``pyramidkv/_mega_cache.py`` (``MegaCache.update`` :136-414 and
  ``MegaCache.attend`` :419-569), holding every pool of the reference's
  ``PyramidKVCacheManager`` (``pyramidkv/csrc/pyramidkv_manager.cc:36-137``)
  as numpy arrays.  bf16 tensors are stored as uint16 bit patterns.
* ``attention_fp32`` -- softmax(Q K^T * scale) V per (chunk, head) in fp32,
  standing in for ``flash_attn_varlen_func`` at ``_mega_cache.py:550-559``
  (the reference pins attention only against an fp32 softmax,
  ``tests/test_mega_readout.py:43-56``).
* ``rope_freq_tables`` -- the freq tables of ``wan/modules/causal_model.py``
  :586-591 (``rope_params`` at ``wan/modules/model.py:29-36``) split and
  flattened as ``_mega_cache.py:715-731`` does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libpkv_oracle.so")
_lib = None
_lock = threading.Lock()

# Bounds, kinds and modes restated from pyramidkv/csrc/anchor_store.cuh:39-45,
# :148 and pyramidkv/_mega_state_ref.py:23-50.
MAX_PHASE = 6
MAX_BUCKET = 4
MAX_T_KEYED = 24
MAX_LAG_OFFSETS = 4
MAX_MERGE_BLOCKS = 6
MAX_MERGE_ACTIVE = 2
MAX_MERGE_BLOCK_FRAMES = 4
MAX_MERGE_TOKENS = 420
SK_RECENT, SK_CYCLIC, SK_STRIDE, SK_LAG, SK_MERGE = 0, 1, 2, 3, 4
DST_SKIP, DST_SINK, DST_MIDDLE, DST_RECENT, DST_MERGE_ACCUM = -1, 0, 1, 2, 5
ROPE_FMA_FIRST, ROPE_FMA_SECOND, ROPE_NO_FMA = 0, 1, 2
SINK_MODE = {"lag": 0, "window_clamp": 1}


def build() -> str:
    """Compile the C restatement (plain gcc) if it is missing or stale."""
    src = os.path.join(_HERE, "pkv_oracle.c")
    if (not os.path.exists(_LIB_PATH)
            or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
        subprocess.check_call(["make", "-s", "-C", _HERE, "libpkv_oracle.so"])
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_LIB_PATH)
            P = ctypes.c_void_p
            I = ctypes.c_int
            L.orc_state_size.restype = ctypes.c_int64
            L.orc_state_offset.restype = ctypes.c_int64
            L.orc_state_offset.argtypes = [I]
            L.orc_map_sink_time.restype = ctypes.c_int64
            L.orc_map_sink_time.argtypes = [ctypes.c_int64, I, I, I, I]
            L.orc_state_update.argtypes = [P, P, I, I, I] + [P] * 8
            L.orc_plan_multi.restype = ctypes.c_int64
            L.orc_plan_multi.argtypes = [P, P, P] + [I] * 8 + [P, I, I, I, I, I] + [P] * 7
            L.orc_layer_offset.argtypes = [P, P, I, I, I, I, I, I, I]
            L.orc_update_frames.argtypes = [P] * 16 + [I] * 4
            L.orc_merge_accum.argtypes = [P] * 18 + [I] * 7
            L.orc_pack.argtypes = ([P] * 19 + [I, P] + [P, I, I] * 3 + [I] * 4)
            L.orc_f32_to_bf16.restype = ctypes.c_uint16
            L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
            L.orc_set_threads.argtypes = [I]
            _lib = L
    return _lib


def set_threads(n: int) -> None:
    """Threads for the C pack (OpenMP over segments); 1, the default, starts none.
    Only the timed CPU baseline raises it, to the host's core count."""
    lib().orc_set_threads(int(n))


def _p(a):
    """ctypes pointer to a contiguous numpy array (None -> NULL)."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------------------
# bf16 helpers (numpy, uint16 bit patterns)
# ---------------------------------------------------------------------------
def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits; NaN -> 0x7FC0.  In 32-bit
    arithmetic, in place: bits + 0x7FFF + lsb cannot pass 2^32 for any
    finite or infinite input, and NaNs are overwritten."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    r = u >> 16
    r &= 1
    r += 0x7FFF
    r += u
    r >>= 16
    out = r.astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = 0x7FC0
    return out


def state_size() -> int:
    return int(lib().orc_state_size())


# ---------------------------------------------------------------------------
# Thin wrappers over the C entry points
# ---------------------------------------------------------------------------
def state_update(states: np.ndarray, t_vals, pass_kind: int, H: int):
    """anchor_store_update.cu:233-313 on a uint8 [H*600] buffer (mutated).

    Returns the 8 descriptor arrays (int32 [H*F] each) in the kernel's order.
    """
    t = np.ascontiguousarray(np.asarray(list(t_vals), dtype=np.int64))
    F = int(t.shape[0])
    N = H * F
    d = [np.empty(N, dtype=np.int32) for _ in range(8)]
    assert states.dtype == np.uint8 and states.size >= H * state_size()
    lib().orc_state_update(_p(states), _p(t), H, F, int(pass_kind), *[_p(x) for x in d])
    return tuple(d)


def map_sink_time(t: int, mode: str, cmin: int, cmax: int, lag: int) -> int:
    return int(lib().orc_map_sink_time(int(t), SINK_MODE.get(mode, 0), cmin, cmax, lag))


def plan_multi(vc, mtc, states_layer, *, L, H, F, max_sink, max_middle, max_recent,
               layer, current_t_list, sink_mode="lag", cmin=0, cmax=21, lag=0,
               mmb=MAX_MERGE_BLOCKS):
    """mega_plan.cc:510-654.  Returns (cu, sk, sg, sl, dst, traw, tremap, total)."""
    C = len(current_t_list)
    S = max_sink + max_middle + max_recent + mmb
    N = C * H * S
    cu = np.empty(C * H + 1, np.int32)
    sk, sg, sl, dst = (np.empty(N, np.int32) for _ in range(4))
    traw, tremap = np.empty(N, np.int64), np.empty(N, np.int64)
    ct = np.ascontiguousarray(np.asarray(current_t_list, dtype=np.int64))
    total = lib().orc_plan_multi(
        _p(np.ascontiguousarray(vc, dtype=np.int64)),
        _p(np.ascontiguousarray(mtc, dtype=np.int32)),
        _p(np.ascontiguousarray(states_layer, dtype=np.uint8)),
        L, H, F, max_sink, max_middle, max_recent, mmb, layer, _p(ct), C,
        SINK_MODE.get(sink_mode, 0) if isinstance(sink_mode, str) else int(sink_mode),
        cmin, cmax, lag, _p(cu), _p(sk), _p(sg), _p(sl), _p(dst), _p(traw), _p(tremap))
    return cu, sk, sg, sl, dst, traw, tremap, int(total)


def layer_offset(sk, sg, layer, H, max_sink, max_middle, max_recent, mmb=MAX_MERGE_BLOCKS):
    out = np.ascontiguousarray(sg.copy())
    lib().orc_layer_offset(_p(np.ascontiguousarray(sk)), _p(out), int(sk.size), layer, H,
                           max_sink, max_middle, max_recent, mmb)
    return out


# ---------------------------------------------------------------------------
# RoPE tables (causal_model.py:586-591, model.py:29-36, _mega_cache.py:715-731)
# ---------------------------------------------------------------------------
def rope_freq_tables(head_dim: int = 128, max_len: int = 1024):
    """Return (ft, fy, fx) fp32 flat tables [max_len, cols*2] (re, im interleaved).

    torch is used only to evaluate cos/sin in float64 exactly as the reference
    builds its table; the result is plain numpy.
    """
    import torch

    d = head_dim

    def params(n, dim):
        freqs = torch.outer(
            torch.arange(n),
            1.0 / torch.pow(10000, torch.arange(0, dim, 2).to(torch.float64).div(dim)))
        return torch.polar(torch.ones_like(freqs), freqs)

    full = torch.cat([params(max_len, d - 4 * (d // 6)), params(max_len, 2 * (d // 6)),
                      params(max_len, 2 * (d // 6))], dim=1)
    c = d // 2
    split = [c - 2 * (c // 3), c // 3, c // 3]
    parts = full.split(split, dim=1)
    out = []
    for z in parts:
        out.append(torch.view_as_real(z.to(torch.complex64)).contiguous()
                   .view(z.shape[0], -1).numpy().copy())
    return tuple(out), full


# ---------------------------------------------------------------------------
# Attention reference (fp32)
# ---------------------------------------------------------------------------
def attention_fp32(q_f32: np.ndarray, k_f32: np.ndarray, v_f32: np.ndarray,
                   cu_k: np.ndarray, num_chunks: int, H: int, Lq: int,
                   scale: float | None = None) -> np.ndarray:
    """softmax(q k^T * scale) v, non-causal, per (chunk, head) segment.

    q_f32: [num_chunks*Lq, H, D] (the [B=1, L_q, H, D] layout of the caller);
    k_f32/v_f32: [T, D] packed flats; cu_k: [num_chunks*H + 1].
    Returns [num_chunks*Lq, H, D] fp32.
    """
    D = q_f32.shape[-1]
    if scale is None:
        scale = D ** -0.5
    out = np.zeros_like(q_f32, dtype=np.float32)
    for c in range(num_chunks):
        for h in range(H):
            i = c * H + h
            a, b = int(cu_k[i]), int(cu_k[i + 1])
            qh = q_f32[c * Lq:(c + 1) * Lq, h, :].astype(np.float32)
            if b <= a:
                continue
            s = (qh @ k_f32[a:b].T.astype(np.float32)) * np.float32(scale)
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=1, keepdims=True)
            out[c * Lq:(c + 1) * Lq, h, :] = p @ v_f32[a:b].astype(np.float32)
    return out


# ---------------------------------------------------------------------------
# Full MegaCache restatement
# ---------------------------------------------------------------------------
class OracleMegaCache:
    """numpy restatement of ``PyramidKVCacheManager`` + ``MegaCache`` (all layers).

    ``states``: uint8 [L, H*600] (as built by ``build_mega_caches``,
    ``_mega_cache.py:684-706``); ``sink_caps``: int64 [L, H].
    """

    def __init__(self, L, H, D, FSEQ, max_sink, max_middle, max_recent, states,
                 sink_caps, *, max_attend_chunks=8, spatial_width=52,
                 sink_time_mapping_mode="lag", sink_time_clamp_min=0,
                 sink_time_clamp_max=21, decoupled_sink_time_lag=0,
                 freq_tables=None, rope_mode=ROPE_FMA_FIRST, has_merge_head=None):
        self.L, self.H, self.D, self.FSEQ = L, H, D, FSEQ
        self.max_sink, self.max_middle, self.max_recent = max_sink, max_middle, max_recent
        self.mmb, self.mma, self.mtpa = MAX_MERGE_BLOCKS, MAX_MERGE_ACTIVE, MAX_MERGE_TOKENS
        self.max_attend_chunks = max_attend_chunks
        self.W = spatial_width
        self.sink_mode = sink_time_mapping_mode
        self.cmin, self.cmax, self.lag = (sink_time_clamp_min, sink_time_clamp_max,
                                          decoupled_sink_time_lag)
        self.freq_tables = freq_tables
        self.rope_mode = rope_mode
        u16, i64, i32, f32 = np.uint16, np.int64, np.int32, np.float32
        z = np.zeros
        # pyramidkv_manager.cc:80-137
        self.sink_k = z((L, H, max_sink, FSEQ, D), u16)
        self.sink_v = z_like = z((L, H, max_sink, FSEQ, D), u16)
        self.mid_k = z((L, H, max_middle, FSEQ, D), u16)
        self.mid_v = z((L, H, max_middle, FSEQ, D), u16)
        self.rec_k = z((L, H, max_recent, FSEQ, D), u16)
        self.rec_v = z((L, H, max_recent, FSEQ, D), u16)
        self.sink_pos = z((L, H, max_sink, FSEQ, 3), i64)
        self.mid_pos = z((L, H, max_middle, FSEQ, 3), i64)
        self.rec_pos = z((L, H, max_recent, FSEQ, 3), i64)
        self.vc = z((L, H, 3), i64)
        self.mg_k = z((L, H, self.mmb, self.mtpa, D), u16)
        self.mg_v = z((L, H, self.mmb, self.mtpa, D), u16)
        self.mg_pos = z((L, H, self.mmb, self.mtpa, 3), i64)
        self.mtc = z((L, H, self.mmb), i32)
        self.acc_k = z((L, H, self.mma, self.mtpa, D), f32)
        self.acc_v = z((L, H, self.mma, self.mtpa, D), f32)
        self.acc_pos = z((L, H, self.mma, self.mtpa, 3), i64)
        self.acc_gid = z((L, H, self.mma, FSEQ), i32)
        self.acc_tpg = z((L, H, self.mma, self.mtpa), f32)
        self.acc_ng = z((L, H, self.mma), i32)
        self.max_total = max_sink + max_middle + max_recent
        self.max_pack_tokens = max_attend_chunks * H * (self.max_total + self.mmb) * FSEQ
        self.states = np.ascontiguousarray(states, dtype=np.uint8).reshape(L, -1).copy()
        self.sink_caps = np.asarray(sink_caps, dtype=np.int64).reshape(L, H).copy()
        if has_merge_head is None:
            kinds = self.states.reshape(L, H, -1)[:, :, 0]
            has_merge_head = bool((kinds == SK_MERGE).any())
        self.has_merge_head = has_merge_head
        self.committed_vc = None
        self.committed_rec_k = None
        self.committed_rec_v = None
        self.committed_rec_pos = None
        del z_like

    # -- _mega_cache.py:136-414 ----------------------------------------------
    def update(self, layer, new_k, new_v, current_start, mode="clean"):
        if mode == "default":
            mode = "clean"
        if mode not in ("noisy", "clean"):
            return
        H, D, FSEQ = self.H, self.D, self.FSEQ
        L_in = new_k.shape[1]
        assert L_in % FSEQ == 0
        F = L_in // FSEQ
        t0 = current_start // FSEQ
        t_vals = np.arange(t0, t0 + F, dtype=np.int64)
        nk = np.ascontiguousarray(new_k.reshape(F, FSEQ, H, D).transpose(0, 2, 1, 3))
        nv = np.ascontiguousarray(new_v.reshape(F, FSEQ, H, D).transpose(0, 2, 1, 3))
        idx = np.arange(FSEQ, dtype=np.int64)
        pos = np.empty((F, H, FSEQ, 3), np.int64)
        pos[..., 0] = t_vals.reshape(F, 1, 1)
        pos[..., 1] = (idx // self.W).reshape(1, 1, FSEQ)
        pos[..., 2] = (idx % self.W).reshape(1, 1, FSEQ)

        vc = self.vc
        if self.committed_vc is None:
            self.committed_vc = vc.copy()
        else:
            vc[layer] = self.committed_vc[layer]
        if self.committed_rec_k is None:
            self.committed_rec_k = self.rec_k.copy()
            self.committed_rec_v = self.rec_v.copy()
            self.committed_rec_pos = self.rec_pos.copy()
        else:
            self.rec_k[layer] = self.committed_rec_k[layer]
            self.rec_v[layer] = self.committed_rec_v[layer]
            self.rec_pos[layer] = self.committed_rec_pos[layer]

        ms, mr = self.max_sink, self.max_recent
        for h in range(H):
            cap = min(int(self.sink_caps[layer, h]), ms)
            sc = int(vc[layer, h, 0])
            rc = int(vc[layer, h, 2])
            sw = max(0, min(F, cap - sc))
            rw = F - sw
            for i in range(sw):
                self.sink_k[layer, h, sc + i] = nk[i, h]
                self.sink_v[layer, h, sc + i] = nv[i, h]
                self.sink_pos[layer, h, sc + i] = pos[i, h]
            vc[layer, h, 0] = sc + sw
            if rw == 0:
                continue
            tot = rc + rw
            if tot <= mr:
                for i in range(rw):
                    self.rec_k[layer, h, rc + i] = nk[sw + i, h]
                    self.rec_v[layer, h, rc + i] = nv[sw + i, h]
                    self.rec_pos[layer, h, rc + i] = pos[sw + i, h]
                vc[layer, h, 2] = tot
            else:
                ev = tot - mr
                for arr in (self.rec_k, self.rec_v, self.rec_pos):
                    arr[layer, h, :mr - ev] = arr[layer, h, ev:mr].copy()
                for i in range(rw):
                    slot = mr - rw + i
                    self.rec_k[layer, h, slot] = nk[sw + i, h]
                    self.rec_v[layer, h, slot] = nv[sw + i, h]
                    self.rec_pos[layer, h, slot] = pos[sw + i, h]
                vc[layer, h, 2] = mr

        if mode == "clean":
            st = self.states[layer]
            dk, ds, dsf, dsh, dma, dml, dmf, dmn = state_update(st, t_vals, 1, H)
            dk_pool = np.where(dk == DST_MERGE_ACCUM, np.int32(-1), dk).astype(np.int32)
            sg = (ds.astype(np.int64) + (layer * H + dsh.astype(np.int64)) * self.max_middle)
            sg = sg.astype(np.int32)
            flat = lambda a: a.reshape(-1)  # noqa: E731
            lib().orc_update_frames(
                _p(nk), _p(nv), _p(pos),
                _p(flat(self.sink_k)), _p(flat(self.sink_v)), _p(flat(self.mid_k)),
                _p(flat(self.mid_v)), _p(flat(self.rec_k)), _p(flat(self.rec_v)),
                _p(flat(self.sink_pos)), _p(flat(self.mid_pos)), _p(flat(self.rec_pos)),
                _p(np.ascontiguousarray(dk_pool)), _p(sg), _p(dsf), _p(dsh),
                int(dk.size), H, FSEQ, D)
            if self.has_merge_head:
                dk_m = np.where(dk == DST_MERGE_ACCUM, dk, np.int32(-1)).astype(np.int32)
                lib().orc_merge_accum(
                    _p(st), _p(nk), _p(nv), _p(pos), _p(np.ascontiguousarray(dk_m)),
                    _p(dma), _p(dmf), _p(dmn),
                    _p(self.acc_k[layer]), _p(self.acc_v[layer]), _p(self.acc_pos[layer]),
                    _p(self.acc_gid[layer]), _p(self.acc_tpg[layer]), _p(self.acc_ng[layer]),
                    _p(self.mg_k[layer]), _p(self.mg_v[layer]), _p(self.mg_pos[layer]),
                    _p(self.mtc[layer]), H, F, FSEQ, D, self.mma, self.mmb, self.mtpa)
            self.committed_vc[layer] = vc[layer]
            self.committed_rec_k[layer] = self.rec_k[layer]
            self.committed_rec_v[layer] = self.rec_v[layer]
            self.committed_rec_pos[layer] = self.rec_pos[layer]

    # -- _mega_cache.py:419-524 (plan + layer offset + pack) -------------------
    def plan_and_pack(self, layer, current_start, num_chunks):
        H, D, FSEQ = self.H, self.D, self.FSEQ
        ct = [(current_start + c * FSEQ) // FSEQ for c in range(num_chunks)]
        cu, sk, sg, sl, dst, traw, tremap, total = plan_multi(
            self.vc, self.mtc, self.states[layer], L=self.L, H=H, F=FSEQ,
            max_sink=self.max_sink, max_middle=self.max_middle,
            max_recent=self.max_recent, layer=layer, current_t_list=ct,
            sink_mode=self.sink_mode, cmin=self.cmin, cmax=self.cmax, lag=self.lag)
        if total > self.max_pack_tokens:
            raise RuntimeError(
                f"mega_plan_multi: packed tokens ({total}) exceed pack-workspace "
                f"capacity ({self.max_pack_tokens})")
        sga = layer_offset(sk, sg, layer, H, self.max_sink, self.max_middle,
                           self.max_recent)
        k_out = np.zeros((max(total, 1), D), np.uint16)
        v_out = np.zeros((max(total, 1), D), np.uint16)
        pos_out = np.zeros((max(total, 1), 3), np.int64)
        ft = fy = fx = None
        fr = [0] * 6
        if self.freq_tables is not None:
            ft, fy, fx = (np.ascontiguousarray(t, dtype=np.float32) for t in self.freq_tables)
            fr = [ft.shape[0], ft.shape[1] // 2, fy.shape[0], fy.shape[1] // 2,
                  fx.shape[0], fx.shape[1] // 2]
        flat = lambda a: a.reshape(-1)  # noqa: E731
        lib().orc_pack(
            _p(flat(self.sink_k)), _p(flat(self.sink_v)), _p(flat(self.mid_k)),
            _p(flat(self.mid_v)), _p(flat(self.rec_k)), _p(flat(self.rec_v)),
            _p(flat(self.mg_k)), _p(flat(self.mg_v)), _p(flat(self.sink_pos)),
            _p(flat(self.mid_pos)), _p(flat(self.rec_pos)), _p(flat(self.mg_pos)),
            _p(k_out), _p(v_out), _p(pos_out), _p(sk), _p(sga), _p(sl), _p(dst),
            int(sk.size), _p(tremap) if ft is not None else None,
            _p(ft), fr[0], fr[1], _p(fy), fr[2], fr[3], _p(fx), fr[4], fr[5],
            FSEQ, self.mtpa, D, int(self.rope_mode))
        return dict(cu=cu, sk=sk, sg=sg, sg_adj=sga, sl=sl, dst=dst, traw=traw,
                    tremap=tremap, total=total, k=k_out[:total], v=v_out[:total],
                    pos=pos_out[:total], current_t=ct)

    # -- _mega_cache.py:419-569 -------------------------------------------------
    def attend(self, layer, q_bf16, current_start, softmax_scale=None):
        """q_bf16: uint16 [1, L_q, H, D].  Returns (out_f32 [1, L_q, H, D], packed)."""
        L_q = q_bf16.shape[1]
        num_chunks = L_q // self.FSEQ
        pk = self.plan_and_pack(layer, current_start, num_chunks)
        qf = bf16_to_f32(q_bf16[0])
        out = attention_fp32(qf, bf16_to_f32(pk["k"]), bf16_to_f32(pk["v"]), pk["cu"],
                             num_chunks, self.H, self.FSEQ, softmax_scale)
        return out[None], pk


def make_states(kinds_params, H=None) -> np.ndarray:
    """Build one layer's uint8 PerHeadState buffer from dicts.

    Each dict: {"kind": SK_*, "sink_capacity": int, "period", "bucket_cap",
    "interval", "capacity", "patch_size"} (missing fields default as in
    ``pyramidkv/_mega_state_ref.py:59-113``: slots -1, times 0).
    """
    n = len(kinds_params)
    buf = np.zeros(n * 600, np.uint8)
    for h, kp in enumerate(kinds_params):
        b = buf[h * 600:(h + 1) * 600]
        i32 = b[4:].view(np.int32)  # offset 4 onwards is 4-byte aligned
        b[0] = np.uint8(np.int8(kp.get("kind", 0)).view(np.uint8))
        b[1] = np.uint8(np.int8(kp.get("sink_capacity", 0)).view(np.uint8))
        ps = int(kp.get("patch_size", 0))
        vals = [kp.get("period", 0), kp.get("bucket_cap", 0), kp.get("interval", 0),
                kp.get("capacity", 0), ps,
                kp.get("block_frames", ps * ps if kp.get("kind") == SK_MERGE else 0)]
        i32[0:6] = vals
        # cyclic_slot @48 (i32 idx 11), 24 entries = -1
        i32[11:35] = -1
        # tkey_slot @248 -> idx (248-4)/4 = 61
        i32[61:85] = -1
        # merge_completed_slot @444 -> idx 110 (6), block_id @468 -> 116 (6)
        i32[110:116] = -1
        i32[116:122] = -1
        # merge_active_block_id @568 -> idx 141 (2)
        i32[141:143] = -1
    return buf


# ---------------------------------------------------------------------------
# AdaptiveKVCache / CppStrategyManager ops (pyramidkv/csrc/scatter_copy.cu)
# ---------------------------------------------------------------------------
def legacy_map_t(src_t: int, current_t: int, mode: int, rel_max: int, soft: float) -> int:
    """History time mapping of one stored time (scatter_copy.cu:138-163):
    mode 1 clamps current_t - t at rel_max, mode 2 compresses the excess by
    ``soft`` (float32 product rounded to nearest even, as llrintf); never < 0."""
    if rel_max <= 0:
        return int(src_t)
    rel = max(int(current_t) - int(src_t), 0)
    t = int(src_t)
    if mode == 1:
        rel = min(rel, int(rel_max))
        t = int(current_t) - rel
    elif mode == 2:
        if rel > rel_max:
            rel = int(rel_max) + int(np.rint(np.float32(rel - rel_max) * np.float32(soft)))
        t = int(current_t) - rel
    return max(t, 0)


def legacy_refresh(srcs_k, srcs_v, srcs_pos, offsets, lengths, flags, rope_t, dst_k, dst_v,
                   dst_pos, dst_frame, current_t, mode, rel_max, soft):
    """refresh_readout_layout (scatter_copy.cu:77-168) on numpy arrays, in place."""
    for s, (sk, sv, sp) in enumerate(zip(srcs_k, srcs_v, srcs_pos)):
        n, off, fl = int(lengths[s]), int(offsets[s]), int(flags[s])
        if n <= 0:
            continue
        dst_k[off:off + n] = sk[:n]
        dst_v[off:off + n] = sv[:n]
        for r in range(n):
            t = int(sp[r, 0])
            if fl & 4:
                mt = int(rope_t[s])
            elif fl & 1:
                mt = legacy_map_t(t, current_t, mode, rel_max, soft)
            else:
                mt = t
            dst_pos[off + r] = (mt, sp[r, 1], sp[r, 2])
            dst_frame[off + r] = t if fl & 2 else mt


def legacy_scatter_copy(srcs, lengths, offsets, dst):
    """scatter_copy (scatter_copy.cu:13-47): rows of each source into dst, in place."""
    for s, src in enumerate(srcs):
        n, off = int(lengths[s]), int(offsets[s])
        if n > 0:
            dst[off:off + n] = src[:n]


def legacy_write_frames(k_seq, v_seq, pos_seq, frame_desc, store_k, store_v, store_pos):
    """anchor_store_write_frames (scatter_copy.cu:170-225): whole frames into slots."""
    F = store_k.shape[1]
    for src_frame, slot in np.asarray(frame_desc).reshape(-1, 2):
        if src_frame < 0 or slot < 0:
            continue
        store_k[slot] = k_seq[src_frame * F:(src_frame + 1) * F]
        store_v[slot] = v_seq[src_frame * F:(src_frame + 1) * F]
        store_pos[slot] = pos_seq[src_frame * F:(src_frame + 1) * F]


def legacy_plan(vc, F: int, max_sink: int, max_middle: int, max_recent: int):
    """The M1.4 all-layer plan (pyramidkv_plan.cc:48-173): vc [L, H, 3] int64
    valid counts -> (cu [L*H+1], sk, sg, sl, dst [L*H*3]) int32.  Per (layer,
    head) the kinds sink (0), recent (2), middle (1) in that order; an active
    kind is one segment from the head's slot 0 over valid_count frames, an
    inactive one kind -1 with zero slot, length and offset."""
    vc = np.asarray(vc, dtype=np.int64)
    L, H = vc.shape[:2]
    n = L * H
    max_slots = (max_sink, max_middle, max_recent)
    cu = np.zeros(n + 1, np.int32)
    sk = np.full(n * 3, -1, np.int32)
    sg = np.zeros(n * 3, np.int32)
    sl = np.zeros(n * 3, np.int32)
    dst = np.zeros(n * 3, np.int32)
    run = 0
    for i in range(n):
        layer, head = divmod(i, H)
        for kp, kind in enumerate((0, 2, 1)):
            nv = int(vc[layer, head, kind])
            if nv <= 0:
                continue
            d = i * 3 + kp
            sk[d] = kind
            sg[d] = i * max_slots[kind]
            sl[d] = nv * F
            dst[d] = run
            run += nv * F
        cu[i + 1] = run
    return cu, sk, sg, sl, dst


# ---------------------------------------------------------------------------
# Query RoPE (wan/modules/causal_model.py:30-63)
# ---------------------------------------------------------------------------
def rope_q(x_bf16: np.ndarray, freqs_full, start_frame: int, F: int, Hg: int, Wg: int):
    """One sample: x uint16 [L, n, D] -> rotated uint16 [L, n, D] (complex128
    products a*c - b*d, a*d + b*c, rounded to float32 then bf16; tokens past
    F*Hg*Wg copied).  wan/modules/causal_model.py:30-63."""
    import torch
    L, n, D = x_bf16.shape
    c = D // 2
    z = freqs_full.detach().cpu().numpy() if isinstance(freqs_full, torch.Tensor) else freqs_full
    parts = np.split(z, [c - 2 * (c // 3), c - (c // 3)], axis=1)
    S = F * Hg * Wg
    f_idx = np.arange(S) // (Hg * Wg)
    h_idx = (np.arange(S) // Wg) % Hg
    w_idx = np.arange(S) % Wg
    fr = np.concatenate([parts[0][start_frame + f_idx], parts[1][h_idx], parts[2][w_idx]], axis=1)
    xf = bf16_to_f32(x_bf16[:S]).astype(np.float64).reshape(S, n, c, 2)
    a, b = xf[..., 0], xf[..., 1]
    cr, ci = fr.real[:, None, :], fr.imag[:, None, :]
    re = a * cr - b * ci
    im = a * ci + b * cr
    out = x_bf16.copy()
    # torch casts float64 -> bf16 through float32 (two roundings), as the
    # reference's .type_as(x) does
    out[:S] = f32_to_bf16(np.stack([re, im], -1).reshape(S, n, D).astype(np.float32))
    return out
