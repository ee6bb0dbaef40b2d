"""Build libmlrec.so (the C-ABI scan library) for sm_100a, in-tree.

    python mlx-recurrence_b200/csrc/build.py [--force] [-v]

Each ``.cu`` file under this directory is compiled by nvcc for
``arch=compute_100a,code=sm_100a`` (with ``-lineinfo``) into ``_build/``,
then linked into ``mlx-recurrence_b200/libmlrec.so``. Rebuilds only what
changed (by modification time of sources and headers).
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
OUT = os.path.join(PKG, "libmlrec.so")
BUILD = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC=...)")


def _flags():
    f = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-I", HERE]
    return ARCH + f


def _headers():
    return glob.glob(os.path.join(HERE, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def build(force=False, verbose=False, jobs=None):
    srcs = sorted(glob.glob(os.path.join(HERE, "*.cu")))
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    hdr_mtime = max([os.path.getmtime(h) for h in _headers()] + [0])
    flags = _flags()

    def obj_of(s):
        return os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")

    todo = [s for s in srcs if force or not os.path.exists(obj_of(s))
            or os.path.getmtime(obj_of(s)) < max(os.path.getmtime(s), hdr_mtime)]

    def compile_one(s):
        cmd = [nvcc] + flags + ["-c", s, "-o", obj_of(s)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {s}:\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        for msg in ex.map(compile_one, todo):
            if verbose and msg:
                print(msg)

    objs = [obj_of(s) for s in srcs]
    if force or todo or not os.path.exists(OUT) or os.path.getmtime(OUT) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", OUT] + objs + ["-lcudart", "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)
