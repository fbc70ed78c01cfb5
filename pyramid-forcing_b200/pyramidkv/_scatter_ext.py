"""Loader of the prebuilt ``adahead`` extension (``lib/_adahead.so``).

Drop-in for the reference's JIT loader (pyramidkv/_scatter_ext.py:34-77):
``_try_load()`` returns True once ``torch.ops.adahead`` and
``torch.classes.adahead.PyramidKVCacheManager`` are registered, False when no
CUDA device is visible (as the reference does).  There is no JIT build and no
fallback: a missing or unloadable library on a CUDA machine is reported on
stderr and every op call then raises.

Build the library with ``python pyramid-forcing_b200/build.py``.
"""
from __future__ import annotations

import os
import sys

import torch

_LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib")
GLUE_PATH = os.path.join(_LIB_DIR, "_adahead.so")
KERNEL_PATH = os.path.join(_LIB_DIR, "libpkv.so")

_loaded = False
_available: bool | None = None


def load_library() -> None:
    """Register the adahead library in this process (no GPU needed).

    Raises if the prebuilt library is missing.
    """
    global _loaded
    if _loaded:
        return
    if not os.path.exists(GLUE_PATH):
        raise RuntimeError(
            f"pyramidkv: {GLUE_PATH} is missing; build it with "
            "`python pyramid-forcing_b200/build.py`")
    torch.ops.load_library(GLUE_PATH)
    _loaded = True


def _try_load() -> bool:
    global _available
    if _available is not None:
        return _available
    if not torch.cuda.is_available():
        _available = False
        return False
    try:
        load_library()
        _available = True
    except Exception as exc:  # reported, never silently replaced
        print(f"[pyramidkv] failed to load the adahead library: {exc!r}", file=sys.stderr)
        _available = False
    return _available


def _ops():
    if not _try_load():
        raise RuntimeError("CUDA scatter extension not available")
    return torch.ops.adahead


def scatter_available() -> bool:
    """The legacy scatter_copy path stays opt-in (PYRAMIDKV_FORCE_SCATTER=1)."""
    if os.environ.get("PYRAMIDKV_FORCE_SCATTER") != "1":
        return False
    return _try_load()


def cuda_refresh_available() -> bool:
    return _try_load()


def scatter_copy(src_ptrs, lengths, offsets, dst, col_dim):
    _ops().scatter_copy(src_ptrs, lengths, offsets, dst, int(col_dim))


def apply_pos_override(pos, starts, ends, vals):
    _ops().apply_pos_override(pos, starts, ends, vals)


def anchor_store_write_frames(k_seq, v_seq, pos_seq, frame_desc, store_k, store_v, store_pos):
    _ops().anchor_store_write_frames(k_seq, v_seq, pos_seq, frame_desc, store_k, store_v,
                                     store_pos)


def refresh_readout_layout(*args):
    _ops().refresh_readout_layout(*args)
