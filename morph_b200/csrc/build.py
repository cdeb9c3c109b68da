"""Build libmorph_b200.so (the C-ABI library) in place with nvcc for sm_100a.

    python -m morph_b200.csrc.build [--force]

Every ``*.cu`` in this directory is compiled to an object under ``_build/``
(in parallel, skipped when up to date) and linked into
``morph_b200/libmorph_b200.so`` against the shared CUDA runtime.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
OUT = os.path.join(PKG, "libmorph_b200.so")
BUILD = os.path.join(HERE, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-fvisibility=hidden",
          "-I" + os.path.join(REPO, "include")]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build morph_b200")
    return path


def _deps(src: str):
    return [src] + glob.glob(os.path.join(HERE, "*.cuh")) + [os.path.join(REPO, "include", "morph_b200.h")]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def compile_one(src: str, force: bool, extra=()) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if force or _stale(obj, _deps(src)):
        cmd = [nvcc(), *ARCH, *CFLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
        if extra:
            print(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(HERE, "*.cu")))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force or verbose_ptxas, extra), sources))
    if force or _stale(OUT, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "shared", "-o", OUT + ".tmp", *objs,
               "-Xlinker", "-rpath,/usr/local/cuda/lib64"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register/smem usage")
    a = ap.parse_args()
    print(build(a.force, a.ptxas))
