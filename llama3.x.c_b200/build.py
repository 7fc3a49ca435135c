"""Builds the two shared libraries of the package in this directory.

    python llama3.x.c_b200/build.py [--force]

- libllama3x_cuda.so: the sm_100a kernels and their C-ABI (csrc/*.cu, include/kernels_cuda.h, include/device_cuda.h),
  nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo, relocatable device code (the kernels share one device
  error word), position-independent host code, static CUDA runtime.
- libllama3x_engine.so: the C11 engine (host/engine.c, include/engine_cuda.h), gcc -std=c11, linked against
  libllama3x_cuda.so through $ORIGIN.

Objects are rebuilt when their source, a header or this script is newer. No JIT cache is involved: the libraries are
built in the tree so they travel with the checkout.
"""
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
INCLUDE = HERE.parent / "include"
CSRC = HERE / "csrc"
HOST = HERE / "host"
LIB = HERE / "libllama3x_cuda.so"
ENGINE_LIB = HERE / "libllama3x_engine.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr"]
CFLAGS = ["-std=c11", "-O2", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter", "-pthread"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _newer(target, deps):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in deps)


def stale():
    deps = sources() + headers() + [Path(__file__)]
    return _newer(LIB, deps) or _newer(ENGINE_LIB, deps + sorted(HOST.glob("*.c")))


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)


def build(force=False, verbose=False):
    obj_dir = HERE / "_build"
    obj_dir.mkdir(exist_ok=True)
    common = headers() + [Path(__file__)]
    objs, relink = [], force or not LIB.exists()
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        if force or _newer(obj, [src] + common):
            _run([nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)], verbose)
            relink = True
        objs.append(str(obj))
    if relink or _newer(LIB, [Path(o) for o in objs]):
        tmp = LIB.with_suffix(".so.tmp")
        _run([nvcc(), *ARCH, "-rdc=true", "-shared", "-Xcompiler", "-fPIC", *objs, "-o", str(tmp), "-ldl"], verbose)
        os.replace(tmp, LIB)
    host = sorted(HOST.glob("*.c"))
    if force or _newer(ENGINE_LIB, host + common + [LIB]):
        gcc = shutil.which("gcc") or "cc"
        tmp = ENGINE_LIB.with_suffix(".so.tmp")
        _run([gcc, *CFLAGS, "-shared", *map(str, host), "-o", str(tmp), f"-L{HERE}", "-lllama3x_cuda",
              "-Wl,-rpath,$ORIGIN", "-lm", "-pthread"], verbose)
        os.replace(tmp, ENGINE_LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
