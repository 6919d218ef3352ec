"""lmcache_b200: LMCache's paged KV-cache transfer ops on NVIDIA B200 (sm_100a).

Importing the package loads the native extension ``lmcache_b200.c_ops`` (the
reference's c_ops surface: same names, positional argument order and tensor
layouts) and installs it as ``lmcache.c_ops``, the way LMCache-Ascend does at
lmcache_ascend/__init__.py:6-8, so upstream LMCache callers reach these
kernels unchanged. There is no CPU fallback: if the extension was not built
the import fails.
"""

from __future__ import annotations

import os
import sys

import torch  # noqa: F401  (loads libtorch / libc10 before the extension)

try:
    from . import c_ops  # type: ignore[attr-defined]
except ImportError as exc:  # pragma: no cover - exercised only on broken installs
    raise ImportError(
        "lmcache_b200.c_ops is not built (run `python lmcache-ascend_b200/build.py` "
        "or __graft_entry__.build()): " + str(exc)
    ) from exc

LIBRARY_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "liblmcache_b200.so")

sys.modules["lmcache.c_ops"] = c_ops
_lmcache = sys.modules.get("lmcache")
if _lmcache is not None:
    setattr(_lmcache, "c_ops", c_ops)

__all__ = ["c_ops", "LIBRARY_PATH"]
