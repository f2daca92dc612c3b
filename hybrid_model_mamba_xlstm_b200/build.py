"""Build libhxm.so (the sm_100a kernels behind include/hxm.h) in-tree.

    python -m hybrid_model_mamba_xlstm_b200.build [--force] [-j N]

Each ``csrc/*.cu`` is compiled separately with nvcc for sm_100a and the
objects are linked into ``hybrid_model_mamba_xlstm_b200/lib/libhxm.so``
(static CUDA runtime, so the library needs only the driver).  Objects are
rebuilt when their source or any header is newer.
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
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
OBJDIR = os.path.join(LIBDIR, "obj")
LIB = os.path.join(LIBDIR, "libhxm.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, extra) -> str:
    obj = os.path.join(OBJDIR, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, extra=()) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = _headers()
    todo = [s for s in srcs if force or _stale(os.path.join(OBJDIR, os.path.basename(s)[:-3] + ".o"), [s, *hdrs])]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            for obj in ex.map(lambda s: _compile(s, list(extra)), todo):
                if verbose:
                    print("compiled", os.path.relpath(obj, ROOT))
    objs = [os.path.join(OBJDIR, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if force or todo or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose:
            print("linked", os.path.relpath(LIB, ROOT))
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills per kernel")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    if a.ptxas_verbose:
        os.makedirs(OBJDIR, exist_ok=True)
        for s in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", s, "-o", os.devnull]
            r = subprocess.run(cmd, capture_output=True, text=True)
            sys.stdout.write(r.stderr)
        return
    print(build(force=a.force, jobs=a.j, verbose=True))


if __name__ == "__main__":
    main()
