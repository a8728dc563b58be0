"""Build libpesti_kq.so (sm_100a) in-tree with nvcc.

    python -m pesti_b200.build          # or: python pesti_b200/build.py

The library is a plain C-ABI shared object (include/pesti_kq.h): no torch
types cross the boundary, so it is built directly with nvcc rather than as a
torch extension.  The CUDA runtime is linked statically.
"""
from __future__ import annotations

import concurrent.futures
import glob
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libpesti_kq.so")
STAMP = LIB + ".stamp"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC,-O2,-Wall", "-Xptxas", "-warn-spills"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libpesti_kq.so")


def _sources():
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
                  + glob.glob(os.path.join(ROOT, "include", "*.h")))
    return srcs, hdrs


def _digest(files) -> str:
    h = hashlib.sha256()
    h.update(" ".join(ARCH + NVCC_FLAGS).encode())
    for f in files:
        h.update(f.encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def _compile(nvcc, src, obj, deps_digest, verbose):
    """Compile one source unless its object was built from the same source,
    headers and flags (a digest beside the object)."""
    stamp = obj + ".stamp"
    want = _digest([src]) + deps_digest
    if os.path.exists(obj) and os.path.exists(stamp):
        with open(stamp) as fh:
            if fh.read().strip() == want:
                return obj
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    with open(stamp, "w") as fh:
        fh.write(want)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    srcs, hdrs = _sources()
    digest = _digest(srcs + hdrs)
    if not force and os.path.exists(LIB) and os.path.exists(STAMP):
        with open(STAMP) as fh:
            if fh.read().strip() == digest:
                return LIB
    nvcc = _nvcc()
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    if force:
        for f in glob.glob(os.path.join(objdir, "*.stamp")):
            os.remove(f)
    deps = _digest(hdrs)
    objs = [os.path.join(objdir, os.path.basename(src) + ".o") for src in srcs]
    # one nvcc per translation unit, in parallel (each is single-threaded)
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 1))) as ex:
        for f in [ex.submit(_compile, nvcc, s, o, deps, verbose) for s, o in zip(srcs, objs)]:
            f.result()
    tmp = LIB + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-lpthread", "-ldl", "-lrt"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    with open(STAMP, "w") as fh:
        fh.write(digest)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
