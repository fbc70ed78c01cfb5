"""Failure detection on the GPU without a fault: a bounded wait that runs out.

The kernels' waits on mbarriers are bounded; on expiry they OR
PKV_ST_TIMEOUT into the status word and return instead of spinning forever.
``pkv_wait_selftest`` runs that wait helper on a barrier nothing completes,
with a 50 ms limit.  The test checks the status bit, the "not completed"
result, and that the CUDA context still runs ordinary work afterwards.
"""
from __future__ import annotations

import ctypes
import os
import time

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu
LIBPKV = os.path.join(ROOT, "pyramid-forcing_b200", "pyramidkv", "lib", "libpkv.so")
PKV_ST_TIMEOUT = 0x40


def test_bounded_wait_times_out_and_reports(cuda):
    lib = ctypes.CDLL(LIBPKV)
    f = lib.pkv_wait_selftest
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    result = torch.full((1,), 7, dtype=torch.int32, device=cuda)
    t0 = time.time()
    rc = f(status.data_ptr(), 50_000_000, result.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert time.time() - t0 < 5.0
    assert int(status.item()) & PKV_ST_TIMEOUT
    assert int(result.item()) == 0
    x = torch.arange(1 << 20, device=cuda, dtype=torch.int64)       # context still usable
    assert int(x.sum().item()) == (1 << 20) * ((1 << 20) - 1) // 2
    assert f(status.data_ptr(), 0, result.data_ptr(), None) != 0     # bad limit refused
