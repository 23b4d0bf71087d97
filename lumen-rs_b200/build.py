"""Build liblumen_cuda.so (the C-ABI library) in-tree for sm_100a.

    python lumen-rs_b200/build.py [--force] [-j N]

Every .cu/.cpp under csrc/ is compiled with nvcc for
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared
library next to this file, so the built .so travels with the source tree.
Objects are cached in csrc/_build/ and rebuilt when a source or header is
newer.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJDIR = os.path.join(CSRC, "_build")
LIB = os.path.join(HERE, "liblumen_cuda.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "-I", INCLUDE, "-I", CSRC]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers_mtime():
    hs = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src: str, force: bool, verbose_ptxas: bool) -> str:
    obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
    if not force and os.path.exists(obj):
        m = os.path.getmtime(obj)
        if m >= os.path.getmtime(src) and m >= _headers_mtime():
            return obj
    cmd = [NVCC, *ARCH, *COMMON, "-c", src, "-o", obj]
    if src.endswith(".cu") and verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    if src.endswith(".cpp"):
        cmd += ["-x", "cu"] if False else []
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int = 8, verbose_ptxas: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose_ptxas), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-lnccl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage per kernel")
    a = ap.parse_args()
    print(build(a.force, a.j, a.ptxas_v))
