"""The drop-in boundary, checked without a GPU.

* libpkv.so loads and exports every entry point include/pkv.h declares;
* the torch glue registers the reference's 12 op schemas and the
  PyramidKVCacheManager class with all 46 of its methods
  (pyramidkv/csrc/scatter_copy_bind.cpp:763-945, fixture
  tests/golden/adahead_api.json), plus Meta kernels;
* the manager allocates the reference's pool shapes and dtypes
  (pyramidkv/csrc/pyramidkv_manager.cc:80-137) and keeps reset() semantics.
No compute kernel is launched here.
"""
from __future__ import annotations

import ctypes
import json
import os
import re

import pytest
import torch

from conftest import GOLDEN, ROOT

LIB = os.path.join(ROOT, "pyramid-forcing_b200", "pyramidkv", "lib")


def _header_functions():
    src = open(os.path.join(ROOT, "include", "pkv.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(pkv_[a-z_0-9]+)\s*\(", src)))


def test_header_symbols_exported():
    lib = ctypes.CDLL(os.path.join(LIB, "libpkv.so"))
    names = _header_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), f"libpkv.so does not export {n}"
    lib.pkv_state_perhead_size.restype = ctypes.c_int64
    assert lib.pkv_state_perhead_size() == 600
    lib.pkv_error_string.restype = ctypes.c_char_p
    assert lib.pkv_error_string(0) == b"ok"


@pytest.fixture(scope="module")
def adahead():
    from pyramidkv import _scatter_ext
    _scatter_ext.load_library()
    return torch.ops.adahead


def _norm(s: str) -> str:
    s = s.split("::", 1)[1] if s.startswith("adahead::") else s
    return re.sub(r"\s+", " ", s).strip()


def test_reference_schemas_registered(adahead):
    api = json.load(open(os.path.join(GOLDEN, "adahead_api.json")))
    for sch in api["schemas"]:
        name = sch.split("(", 1)[0]
        op = getattr(adahead, name)
        got = _norm(str(op.default._schema))
        assert got == _norm(sch), f"{name}: {got} != {sch}"


def test_manager_methods_and_shapes(adahead):
    api = json.load(open(os.path.join(GOLDEN, "adahead_api.json")))
    L, H, D, F, ms, mm, mr, mac = 2, 3, 16, 4, 3, 8, 4, 2
    mgr = torch.classes.adahead.PyramidKVCacheManager(L, H, D, F, ms, mm, mr, "cpu",
                                                      "bfloat16", mac)
    for m in api["class_methods"]:
        assert hasattr(mgr, m), m
    assert mgr.sink_k_pool().shape == (L, H, ms, F, D)
    assert mgr.middle_v_pool().shape == (L, H, mm, F, D)
    assert mgr.recent_pos_pool().shape == (L, H, mr, F, 3)
    assert mgr.recent_pos_pool().dtype == torch.int64
    assert mgr.head_t_table().shape == (L, H, ms + mm + mr)
    assert int(mgr.head_t_table().min()) == -1
    assert mgr.valid_count().shape == (L, H, 3) and mgr.valid_count().dtype == torch.int64
    assert mgr.strategy().dtype == torch.int8
    P = mac * H * (ms + mm + mr + 6) * F
    assert mgr.max_pack_tokens() == P == mgr.max_total_tokens()
    assert mgr.k_flat_out().shape == (P, 1, D) and mgr.pos_flat_out().shape == (P, 3)
    assert mgr.cu_seqlens_k().shape == (mac * H + 1,)
    assert mgr.merge_k_pool().shape == (L, H, 6, 420, D)
    assert mgr.merge_accum_sum_k().dtype == torch.float32
    assert mgr.merge_accum_group_ids().shape == (L, H, 2, F)
    assert mgr.merge_token_count().shape == (L, H, 6)
    assert (mgr.max_merge_blocks(), mgr.max_merge_active(), mgr.max_merge_tokens_per_anchor()) == (6, 2, 420)
    mgr.valid_count().fill_(3)
    mgr.recent_pos_pool().fill_(7)
    mgr.reset()
    assert int(mgr.valid_count().abs().sum()) == 0 and int(mgr.recent_pos_pool().abs().sum()) == 0
    mgr.set_strategy(1, 2, 4, torch.tensor([6, 4], dtype=torch.int8))
    assert mgr.strategy()[1, 2].tolist() == [4, 6, 4, 0, 0, 0, 0, 0]
    with pytest.raises(RuntimeError):
        torch.classes.adahead.PyramidKVCacheManager(L, H, D, F, ms, mm, mr, "cpu", "int8", mac)


def test_meta_dispatch(adahead):
    q = torch.empty(3 * 8, 2, 128, device="meta", dtype=torch.bfloat16)
    out = adahead.pkv_attention(q, q[:, 0], q[:, 0], torch.empty(7, dtype=torch.int32,
                                                                   device="meta"), 3, 8, 0.1)
    assert out.shape == q.shape and out.device.type == "meta"


def test_loader_without_cuda_reports_unavailable(monkeypatch):
    from pyramidkv import _ops, _scatter_ext
    monkeypatch.setattr(_scatter_ext, "_available", None)
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    assert _ops.available() is False
    with pytest.raises(RuntimeError, match="not available"):
        _ops.ops()
