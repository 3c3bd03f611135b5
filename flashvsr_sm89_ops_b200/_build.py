"""Build the sm_100a C-ABI library in-tree: ``python -m flashvsr_sm89_ops_b200._build``.

One nvcc invocation compiles ``csrc/fvb_lib.cu`` (a unity translation unit of
every kernel) into ``libflashvsr_b200.so`` next to this file.  The library has
no torch dependency; Python reaches it through ctypes (``_lib.py``).  Rebuilds
only when a source is newer than the library unless ``force`` is set.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(os.path.dirname(PKG_DIR), "include")
LIB_NAME = "libflashvsr_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found (set NVCC=...)")
    return cand


def _sources():
    out = []
    for d in (CSRC, INCLUDE):
        for name in sorted(os.listdir(d)):
            if name.endswith((".cu", ".cuh", ".h")):
                out.append(os.path.join(d, name))
    return out


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(s) > t for s in _sources())


def nvcc_command(out_path: str = LIB_PATH, extra=()):
    return [
        _nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
        "--shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "-Xptxas", "-v" if os.environ.get("FVB_PTXAS_VERBOSE") else "-O3",
        "-I", INCLUDE, "-o", out_path, os.path.join(CSRC, "fvb_lib.cu"), *extra,
    ]


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = nvcc_command(tmp)
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
