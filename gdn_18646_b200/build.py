"""Build libgdn_b200.so (sm_100a) in-tree with nvcc.

    python -m gdn_18646_b200.build [--verbose-ptxas] [--force]

Objects go to gdn_18646_b200/_build/, the shared library to
gdn_18646_b200/lib/libgdn_b200.so.  Rebuilds only what changed (source or
header mtimes).  The library links the CUDA runtime statically and needs no
libcuda at link time (the TMA encoder is fetched from the driver at run time).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libgdn_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                     "-Xcompiler", "-fPIC,-O3", "-I" + INCLUDE]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (CUDA 12.9 toolkit required to build libgdn_b200.so)")


def _deps_mtime() -> float:
    files = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(f) for f in files), default=0.0)


def _compile(src: str, obj: str, verbose_ptxas: bool) -> str:
    cmd = [nvcc(), *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = True) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr_t = _deps_mtime()
    jobs = []
    for src in srcs:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        stale = force or verbose_ptxas or not os.path.exists(obj) or \
            os.path.getmtime(obj) < max(os.path.getmtime(src), hdr_t)
        jobs.append((src, obj, stale))
    logs = {}
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        futs = {ex.submit(_compile, s, o, verbose_ptxas): s for s, o, stale in jobs if stale}
        for f in cf.as_completed(futs):
            logs[os.path.basename(futs[f])] = f.result()
    objs = [o for _, o, _ in jobs]
    if logs or force or not os.path.exists(LIB) or \
            os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if not quiet or verbose_ptxas:
        for name, log in sorted(logs.items()):
            if log.strip():
                print(f"== {name}\n{log}")
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args(argv)
    path = build(force=a.force, verbose_ptxas=a.verbose_ptxas, quiet=False)
    print(path)


if __name__ == "__main__":
    sys.exit(main())
