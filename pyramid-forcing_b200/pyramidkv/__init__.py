"""B200-native MegaCache path of Pyramid Forcing (drop-in ``pyramidkv`` modules).

This package provides the modules of the reference ``pyramidkv`` package that
sit on the per-step KV-cache hot path -- ``_mega_cache``, ``_mega_state_ops``,
``_mega_attention``, ``_ops``, ``_scatter_ext`` and the ``PerHeadState``
mirror ``_mega_state_ref`` -- with the same names, signatures and behaviour,
backed by the sm_100a kernels of ``lib/libpkv.so`` through the ``adahead``
torch library in ``lib/_adahead.so``.

The rest of the reference package (``factory``, ``base``, ``config``, the
strategy classes, ``cpp_strategy``, ...) is not part of this path.  To run the
reference pipeline on top of this package, point ``PYRAMIDKV_REFERENCE_ROOT``
at the reference checkout: its ``pyramidkv`` directory is then appended to
this package's search path, so ``pyramidkv.factory`` etc. resolve to the
reference's modules while the hot-path modules resolve here first.
"""
from __future__ import annotations

import os as _os

_ref_root = _os.environ.get("PYRAMIDKV_REFERENCE_ROOT")
if _ref_root:
    _ref_pkg = _os.path.join(_ref_root, "pyramidkv")
    if _os.path.isdir(_ref_pkg) and _ref_pkg not in __path__:
        __path__.append(_ref_pkg)

LIB_DIR = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "lib")
