"""Builds the lmcache_b200 native libraries in-tree.

Outputs (next to the Python package, so they travel with a source snapshot):
  lmcache_b200/liblmcache_b200.so   CUDA kernels + C ABI (include/lmcache_b200.h),
                                    sm_100a only, static CUDA runtime
  lmcache_b200/c_ops<EXT_SUFFIX>    PyTorch/pybind11 surface (the reference's
                                    c_ops names), linked against the library

Objects go to _build/ (git-ignored). A target is rebuilt only when one of its
inputs is newer than it. Usage: python build.py [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PKG = os.path.join(HERE, "lmcache_b200")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(REPO, "_build")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

CU_SOURCES = ["common.cu", "kv_transfer.cu", "host_mem.cu", "cachegen.cu", "noalloc.cu",
              "pos_kernels.cu"]
HEADERS = [os.path.join(CSRC, "common.cuh"), os.path.join(INCLUDE, "lmcache_b200.h")]
LIB = os.path.join(PKG, "liblmcache_b200.so")
EXT = os.path.join(PKG, "c_ops" + sysconfig.get_config_var("EXT_SUFFIX"))

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-I" + INCLUDE,
    "-I" + CSRC,
]


def _stale(target: str, inputs: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(i) > t for i in inputs)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stdout.write(res.stdout)
        sys.stderr.write(res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"build step failed ({res.returncode}): {' '.join(cmd)}")


def build_library(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    jobs = []
    for src in CU_SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, [path] + HEADERS):
            flags = list(NVCC_FLAGS)
            if ptxas_verbose:
                flags += ["-Xptxas", "-v"]
            jobs.append([NVCC, *flags, "-c", path, "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=max(1, len(jobs))) as ex:
        list(ex.map(lambda c: _run(c, verbose or ptxas_verbose), jobs))
    if force or jobs or _stale(LIB, objs):
        _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs,
              "-o", LIB, "-Xlinker", "-soname=liblmcache_b200.so"], verbose)
    return LIB


def build_extension(force: bool = False, verbose: bool = False) -> str:
    import torch  # noqa: F401  (only for paths)
    from torch.utils import cpp_extension

    src = os.path.join(CSRC, "c_ops.cpp")
    if not (force or _stale(EXT, [src, LIB] + HEADERS)):
        return EXT
    torch_lib = cpp_extension.library_paths()[0]
    includes = cpp_extension.include_paths() + [
        sysconfig.get_paths()["include"],
        os.path.join(CUDA_HOME, "include"),
        INCLUDE,
    ]
    import torch as _t
    abi = int(bool(_t._C._GLIBCXX_USE_CXX11_ABI))
    cmd = [
        # The system g++ (not $CXX): the extension must link libstdc++
        # dynamically, sharing torch's copy; a second, static copy breaks
        # iostream/locale state across the boundary.
        shutil.which("g++") or "g++",
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        "-DTORCH_EXTENSION_NAME=c_ops",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        *["-I" + i for i in includes],
        src,
        "-o",
        EXT,
        "-L" + PKG,
        "-llmcache_b200",
        "-L" + torch_lib,
        "-lc10",
        "-lc10_cuda",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_cuda",
        "-ltorch_python",
        "-Wl,-rpath,$ORIGIN",
        "-Wl,-rpath," + torch_lib,
    ]
    _run(cmd, verbose)
    return EXT


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_extension(force=force, verbose=verbose)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    build_library(force=a.force or a.ptxas, verbose=a.verbose, ptxas_verbose=a.ptxas)
    build_extension(force=a.force, verbose=a.verbose)


if __name__ == "__main__":
    main()
