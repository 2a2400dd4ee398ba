"""Build the engine's shared library, in-tree, for sm_100a.

``python -m gemmkit_b200._build`` (or ``__graft_entry__.build()``) compiles every CUDA
source under ``gemmkit_b200/csrc`` with nvcc into ``gemmkit_b200/_lib/libgemmkit_cuda.so``
(C ABI of ``include/gemmkit_cuda.h``). The CUDA runtime is linked statically; the driver's
tensor-map encoder is looked up at run time, so the library needs no libcuda at link time.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT_DIR = os.path.join(PKG, "_lib")
LIB = os.path.join(OUT_DIR, "libgemmkit_cuda.so")
OBJ_DIR = os.path.join(ROOT, "_build", "obj")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
           "--expt-relaxed-constexpr", "-Xptxas", "-O3", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _newest(paths: list[str]) -> float:
    return max(os.path.getmtime(p) for p in paths)


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    deps = [os.path.join(CSRC, s) for s in sources()] + headers() + [os.path.abspath(__file__)]
    return os.path.getmtime(LIB) >= _newest(deps)


def _compile(src: str, extra: list[str]) -> str:
    obj = os.path.join(OBJ_DIR, src.replace(".cu", ".o"))
    deps = [os.path.join(CSRC, src)] + headers() + [os.path.abspath(__file__)]
    if os.path.exists(obj) and os.path.getmtime(obj) >= _newest(deps):
        return obj
    cmd = [nvcc(), *ARCH, *NVFLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
    subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    if force:
        for f in os.listdir(OBJ_DIR):
            os.remove(os.path.join(OBJ_DIR, f))
    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), sources()))
    tmp = LIB + ".tmp"
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-Xcompiler", "-fPIC"],
                   check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
