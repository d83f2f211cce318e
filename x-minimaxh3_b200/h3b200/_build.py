"""Build the sm_100a shared library ``libh3b200.so`` in-tree with nvcc.

Every ``csrc/*.cu`` file is compiled for ``sm_100a`` only and linked into one
shared object next to this file (static CUDA runtime, no libcuda link: the TMA
descriptor encoder is resolved at run time through the runtime's driver entry
point, so the library also loads on machines without a GPU driver).
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(HERE)
CSRC = os.path.join(PKG_ROOT, "csrc")
REPO = os.path.dirname(PKG_ROOT)
LIB = os.path.join(HERE, "libh3b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the h3b200 library needs the CUDA 12.9 toolchain to build")
    return cand


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        [os.path.join(REPO, "include", "h3b200.h")]
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    objdir = os.path.join(PKG_ROOT, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-I", os.path.join(REPO, "include"), "-rdc=true", "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-rdc=true", "-cudart", "static", "-o", tmp, *objs, "-Xlinker", "--exclude-libs,ALL"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_verbose="--ptxas-v" in sys.argv)
    print(LIB)
