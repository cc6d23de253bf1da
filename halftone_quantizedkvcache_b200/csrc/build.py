"""Build ``libhalftone_b200.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m halftone_quantizedkvcache_b200.csrc.build [--force] [--jobs N]

Each ``.cu`` file here is compiled to an object under ``_build/`` (skipped when
the object is newer than its sources), then linked with the CUDA runtime
(static) into ``halftone_quantizedkvcache_b200/libhalftone_b200.so``.  No torch
headers are involved: the library's interface is ``include/halftone_b200.h``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
BUILD = os.path.join(ROOT, "_build", "csrc")
LIB = os.path.join(PKG, "libhalftone_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libhalftone_b200.so")


def sources():
    return sorted(glob.glob(os.path.join(HERE, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(HERE, "*.cuh"))) + [os.path.join(ROOT, "include", "halftone_b200.h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, force):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if not force and not _stale(obj, [src] + headers()):
        return obj, None
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    return obj, None


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=jobs or min(len(srcs), os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, force), srcs))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    objs = [o for o, _ in results]
    # the exported symbols are the hq_* entry points (default visibility via extern "C")
    if force or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static", *objs, "-o", LIB]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose:
            print("linked", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.jobs, verbose=True))
    sys.exit(0)
