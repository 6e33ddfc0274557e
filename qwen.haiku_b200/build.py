# SPDX-License-Identifier: MIT
"""Builds libqh200.so (CUDA kernels for sm_100a + the C-ABI + the C host
layer) in place, next to this file.

    python qwen.haiku_b200/build.py [-v] [--force]

nvcc compiles every csrc/*.cu for sm_100a only (-gencode
arch=compute_100a,code=sm_100a -lineinfo); gcc compiles csrc/*.c as C17;
nvcc links them into one shared library with a static CUDA runtime, so the
library does not depend on whichever libcudart another component loads.
Objects go to _build/ under the repository root (git-ignored).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build", "qh200")
LIB = os.path.join(HERE, "libqh200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "-Xptxas", "-warn-spills", "--expt-relaxed-constexpr",
    f"-I{INCLUDE}", f"-I{CSRC}",
]
CC_FLAGS = ["-O2", "-std=c17", "-ffp-contract=off", "-fPIC", "-Wall", "-Wextra", "-I/usr/local/cuda/include",
            f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libqh200.so")


def _sources():
    cu = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    c = sorted(f for f in os.listdir(CSRC) if f.endswith(".c"))
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return cu, c, headers


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    if verbose and (r.stdout or r.stderr):
        sys.stdout.write(r.stdout + r.stderr)
    return r


def build(verbose: bool = False, force: bool = False) -> str:
    """Compile and link libqh200.so; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    cu, c, headers = _sources()
    objs = []
    for f in cu:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        if force or _stale(obj, [src] + headers):
            _run([nvcc, *NVCC_FLAGS, "-c", src, "-o", obj], verbose)
        objs.append(obj)
    cc = os.environ.get("CC", "gcc")
    for f in c:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        if force or _stale(obj, [src] + headers):
            _run([cc, *CC_FLAGS, "-c", src, "-o", obj], verbose)
        objs.append(obj)
    if force or _stale(LIB, objs):
        _run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-lm", "-lpthread", "-ldl"], verbose)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="--force" in sys.argv)
    print(LIB)
