"""Builds and loads the C part of the oracle (oracle/*.c -> oracle/_build/liboracle.so).

Test infrastructure only (see oracle/__init__.py). Compiled with gcc on the
host; nothing here touches a GPU.
"""

from __future__ import annotations

import ctypes
import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle.so")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "*.c")))


def build(force: bool = False) -> str | None:
    srcs = sources()
    if not srcs:
        return None
    os.makedirs(OUT_DIR, exist_ok=True)
    if not force and os.path.exists(LIB):
        t = os.path.getmtime(LIB)
        if all(os.path.getmtime(s) <= t for s in srcs + glob.glob(os.path.join(HERE, "*.h"))):
            return LIB
    cmd = [shutil.which("gcc") or "gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-Wall",
           "-Werror", *srcs, "-o", LIB]
    subprocess.run(cmd, check=True)
    return LIB


_LIB = None


def load() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        build()
        _LIB = ctypes.CDLL(LIB)
    return _LIB
