"""Build the breccia_b200 CUDA library in-tree.

``python -m breccia_b200.build`` compiles every ``csrc/*.cu`` for sm_100a with
nvcc and links ``breccia_b200/libbreccia_b200.so`` (C ABI declared in
``include/breccia_b200.h``). The CUDA runtime is linked statically, and the
driver API is reached through ``cudaGetDriverEntryPoint``, so the library
loads on a machine without a GPU (for the export checks) and needs only the
driver on a GPU machine. nvcc cross-compiles: no GPU is needed to build.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libbreccia_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                 "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC,
                 "-Xptxas", "-v", "-Xptxas", "-warn-spills"]
# The cast kernels rely on exact IEEE rounding of every multiply and add:
# no contraction into FMA except where written explicitly.
PER_FILE = {"cast.cu": ["-fmad=false"]}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) > max(
            os.path.getmtime(p) for p in _deps(src)):
        return obj
    cmd = [nvcc()] + COMMON + PER_FILE.get(os.path.basename(src), []) + ["-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    log = os.path.join(BUILD, os.path.basename(src) + ".log")
    with open(log, "w") as f:
        f.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stderr[-6000:]}")
    if verbose:
        print(f"compiled {os.path.basename(src)}")
    return obj


def _deps(src):
    hdrs = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
    return [src, os.path.join(INCLUDE, "breccia_b200.h"), __file__] + hdrs


def build(verbose: bool = True) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    with ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), sources))
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr[-6000:]}")
        os.replace(tmp, LIB)
        if verbose:
            print("linked", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
