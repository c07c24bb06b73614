"""Build libmea.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m memory_efficient_attn_layer_b200.build        # or build() from Python

Objects go to ``_build/`` at the repository root; the shared library is written
next to this file so it travels with the package.  nvcc cross-compiles for
sm_100a without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libmea.so")

SOURCES = ["api.cu", "gemm.cu", "attn_fwd.cu", "attn_bwd.cu", "elementwise.cu", "noalloc.cu", "optim.cu", "selftest.cu", "tma.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + INCLUDE, "-I" + CSRC]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _compile(src: str, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    path = os.path.join(CSRC, src)
    deps = [path] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    deps.append(os.path.join(INCLUDE, "mea.h"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [_nvcc(), *ARCH, *FLAGS, *extra, "-c", path, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [_nvcc(), *FLAGS, "-x", "c++", "-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and "-Xptxas" in " ".join(extra):
        sys.stderr.write(r.stderr)
    return obj


def build(verbose_ptxas: bool = False) -> str:
    """Compile every source for sm_100a and link libmea.so; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), SOURCES))
    newest = max(os.path.getmtime(o) for o in objs)
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= newest:
        return LIB
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp, "-lcudart_static", "-ldl", "-lrt",
           "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose_ptxas="-v" in sys.argv))
