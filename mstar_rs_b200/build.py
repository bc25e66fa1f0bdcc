"""Build the sampler's CUDA library in-tree for sm_100a.

`python -m mstar_rs_b200.build` compiles csrc/sampler.cu with nvcc into
mstar_rs_b200/_lib/libmstar_sampler.so (C ABI declared in
include/mstar_sampler.h).  The library links the CUDA runtime statically, so
it needs only the driver at load time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
SRC = [os.path.join(PKG, "csrc", "sampler.cu")]
DEPS = SRC + [os.path.join(PKG, "csrc", "spec.cuh"), os.path.join(PKG, "csrc", "lmhead.cuh"), os.path.join(ROOT, "include", "mstar_sampler.h")]
OUT = os.path.join(PKG, "_lib", "libmstar_sampler.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the sampler needs the CUDA toolkit to build")
    return cand


def stale() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(d) > t for d in DEPS)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not stale():
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-I", os.path.join(ROOT, "include"), "-o", OUT + ".tmp", *SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.check_call(cmd)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
