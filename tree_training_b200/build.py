"""Build the C-ABI shared library ``libtt_sm100.so`` in-tree.

    python -m tree_training_b200.build            # compile changed sources
    python -m tree_training_b200.build --force    # recompile everything

Every CUDA source is compiled for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``); the CUDA runtime is linked statically so the
library does not depend on which libcudart torch happens to load.  Objects go
to ``_build/`` (git-ignored); the .so lands next to this file so that it
travels with the repository snapshot.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libtt_sm100.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-Xptxas", "-v"] + ARCH
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-Wall"]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")
    return cand


def _sources():
    out = []
    for f in sorted(os.listdir(CSRC)):
        if f.endswith((".cu", ".cpp")):
            out.append(os.path.join(CSRC, f))
    return out


def _headers_mtime() -> float:
    m = 0.0
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh", ".hpp")):
                m = max(m, os.path.getmtime(os.path.join(d, f)))
    return m


def _compile(src: str, force: bool, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if (not force and os.path.exists(obj)
            and os.path.getmtime(obj) >= max(os.path.getmtime(src), _headers_mtime())):
        return obj
    if src.endswith(".cu"):
        cmd = [_nvcc(), *NVCC_FLAGS, "-c", src, "-o", obj]
    else:
        cmd = [os.environ.get("CXX", "g++"), *CXX_FLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log = os.path.join(BUILD, os.path.basename(src) + ".log")
    with open(log, "w") as fh:
        fh.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{r.stderr[-6000:]}")
    if verbose:
        print(f"compiled {os.path.basename(src)}", file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        tmp = LIB + ".tmp"
        cmd = [_nvcc(), "-shared", *ARCH, "-cudart", "static", "-o", tmp, *objs, "-ldl",
               "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr[-6000:]}")
        os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=True))


if __name__ == "__main__":
    main()
