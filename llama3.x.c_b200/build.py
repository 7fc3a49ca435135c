"""Builds libllama3x_cuda.so (the sm_100a kernels and their C-ABI) in this directory with nvcc.

    python llama3.x.c_b200/build.py          # rebuild when a source is newer than the library

Flags: -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo, relocatable device code (the kernels share one device
error word), position-independent host code, static CUDA runtime. No JIT cache is involved: the library is built in
the tree so it travels with the checkout.
"""
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libllama3x_cuda.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [HERE.parent / "include" / "kernels_cuda.h"])


def stale():
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources() + headers() + [Path(__file__)])


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    obj_dir = HERE / "_build"
    obj_dir.mkdir(exist_ok=True)
    objs = []
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-rdc=true", "-shared", "-Xcompiler", "-fPIC", *objs, "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
