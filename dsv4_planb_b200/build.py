"""Build the sas_b200 CUDA library in-tree for sm_100a.

``build()`` compiles every ``csrc/*.cu`` with nvcc (``-gencode
arch=compute_100a,code=sm_100a -lineinfo``) into object files under
``dsv4_planb_b200/_build/`` and links ``dsv4_planb_b200/_lib/libsas_b200.so``.
Sources are recompiled only when they (or a header) are newer than their object.
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libsas_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the sas_b200 CUDA library cannot be built")
    return path


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _compile(src: str, obj: str, extra) -> str:
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    jobs = []
    objs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        stale = force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), newest_header)
        if stale:
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, list(extra_flags)): s for s, o in jobs}
            for f in cf.as_completed(futs):
                msg = f.result()
                if verbose and msg.strip():
                    print(f"[{os.path.basename(futs[f])}]\n{msg}")
    if jobs or not os.path.exists(LIB):
        tmp = LIB + f".tmp{os.getpid()}"
        cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose=True))
