"""Builds kore_b200/libkore_cuda.so (the C-ABI library) with nvcc for sm_100a.

Usage: ``python -m kore_b200.build [--force] [--verbose] [--trace]``. The
library is built in-tree so that it travels with the repository to the GPU
machine. ``--trace`` builds kore_b200/libkore_cuda_trace.so instead: the same
library compiled with KORE_TRACE, whose decode and merge CTAs record
%globaltimer stamps (read by ``python -m kore_b200.trace_decode``).
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libkore_cuda.so")
TRACE_LIB = os.path.join(PKG, "libkore_cuda_trace.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O2",
              "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, trace: bool = False, out: str | None = None,
          defines: tuple[str, ...] = ()) -> str:
    """Compiles every .cu under csrc/ into one shared library; returns its path.
    `out` and `defines` (NAME=VALUE, e.g. KORE_ROWS_WARPS=12) build a variant
    with other compile-time shapes elsewhere (loaded through $KORE_CUDA_LIB)."""
    lib = out or (TRACE_LIB if trace else LIB)
    if not force and not out and not _stale(lib):
        return lib
    objdir = os.path.join(os.path.dirname(lib), "_build_" + os.path.basename(lib)) if out else \
        os.path.join(PKG, "_build_trace" if trace else "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *(["-DKORE_TRACE"] if trace else []), *("-D" + d for d in defines),
               "-I", INCLUDE, "-c", src, "-o", obj]
        if verbose:
            cmd += ["-Xptxas", "-v"]
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = lib + ".tmp"
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-lrt", "-ldl", "-lpthread"],
                   check=True)
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--trace", action="store_true")
    ap.add_argument("--out", default=None, help="build a variant library at this path")
    ap.add_argument("-D", dest="defines", action="append", default=[], help="NAME=VALUE for a variant build")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, trace=a.trace, out=a.out, defines=tuple(a.defines)))
