"""Test infrastructure: the reference repository's own CUDA kernels, built for
B200 as same-box GPU comparators.

Compiles ``kernels/rmsnorm.cu``, ``kernels/decode.cu``,
``kernels/fused_proj_conv_silu.cu`` and ``kernels/prefill_chunked.cu`` of the
reference checkout (read in place, never copied) into torch extension modules
under ``oracle/_ref/``, with the reference's own flags (bench_gdn.py:28-42:
-O3 --use_fast_math, and --expt-relaxed-constexpr for the projection) and the
B200 architecture in place of sm_80.  Only the tests load them (``load``), to
check the library's kernels against them and time both on the same GPU;
nothing in the library or in bench.py's timed legs does.  The prefill kernel
hard-codes H=16, dk=128, dv=256 (kernels/prefill_chunked.cu:15-18), so it is
compared at that head shape only.

Usage (where the reference checkout exists; the built modules then travel with
the repository):  python oracle/build_ref_kernels.py <reference checkout>
"""
from __future__ import annotations

import glob
import importlib.util
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
BUILD_TIMEOUT_S = 1200                          # per module compile

# module name -> (source under kernels/, extra nvcc flags of the reference's bench)
KERNELS = {
    "gdn_ref_rmsnorm": ("rmsnorm.cu", ()),
    "gdn_ref_decode": ("decode.cu", ()),
    "gdn_ref_proj": ("fused_proj_conv_silu.cu", ("--expt-relaxed-constexpr",)),
    "gdn_ref_prefill": ("prefill_chunked.cu", ()),
}


def default_reference_dir() -> str | None:
    """The reference checkout: $GDN_REFERENCE_DIR, else a ``reference`` directory
    beside this repository."""
    cand = os.environ.get("GDN_REFERENCE_DIR") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isfile(os.path.join(cand, "kernels", "decode.cu")) else None


def build(ref_dir: str, only: str | None = None) -> list[str]:
    """Compile the comparator modules into oracle/_ref/<name>/ (skipping those already
    built), one compiler process per module in parallel; returns the .so paths."""
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    os.environ.setdefault("MAX_JOBS", "4")
    names = [only] if only else list(KERNELS)
    missing = [n for n in names if so_path(n) is None]
    if only is None and len(missing) > 1:
        procs = [subprocess.Popen([sys.executable, os.path.abspath(__file__), ref_dir, "--only", n])
                 for n in missing]
        rcs = []
        for p in procs:
            try:
                rcs.append(p.wait(timeout=BUILD_TIMEOUT_S))
            except subprocess.TimeoutExpired:
                p.kill()
                rcs.append("timeout")
        if any(rcs):
            raise RuntimeError(f"comparator build failed: {dict(zip(missing, rcs))}")
    elif missing:
        from torch.utils.cpp_extension import load
        name = missing[0]
        src, extra = KERNELS[name]
        bdir = os.path.join(OUT, name)
        os.makedirs(bdir, exist_ok=True)
        stale = os.path.join(bdir, "lock")         # left by an interrupted build; torch would wait on it
        if os.path.exists(stale):
            os.remove(stale)
        load(name=name, sources=[os.path.join(ref_dir, "kernels", src)], build_directory=bdir,
             extra_cuda_cflags=["-O3", "--use_fast_math", "-lineinfo", *extra], verbose=False)
    return [so_path(n) for n in names]


def so_path(name: str) -> str | None:
    hits = glob.glob(os.path.join(OUT, name, f"{name}*.so"))
    return hits[0] if hits else None


def load(name: str):
    """Import a built comparator module (torch must be imported first); None if absent."""
    path = so_path(name)
    if path is None:
        return None
    import torch  # noqa: F401  (the module links against libtorch)
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    args = sys.argv[1:]
    only = None
    if "--only" in args:
        i = args.index("--only")
        only = args[i + 1]
        del args[i:i + 2]
    ref = args[0] if args else default_reference_dir()
    if not ref:
        sys.exit("usage: python oracle/build_ref_kernels.py <reference checkout> [--only <module>]")
    for p in build(ref, only):
        print(p)
