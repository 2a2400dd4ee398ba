"""Build recipe for the CPU oracle (test infrastructure only).

Compiles ``gk_oracle.c`` (scalar restatement of gemmkit's semantics) and
``gk_cpu_baseline.c`` (threaded restatement of gemmkit's AVX-512 VNNI / BF16 path) into
``oracle/_build/libgk_oracle.so``. The strict floating-point flags keep every f64 step a
single IEEE-754 operation, as in the Rust reference. Runs in seconds with gcc; needs no
GPU and no reference sources.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libgk_oracle.so")
SOURCES = ["gk_oracle.c", "gk_cpu_baseline.c"]
CFLAGS = ["-O2", "-std=gnu11", "-fPIC", "-shared", "-fopenmp", "-fno-fast-math",
          "-ffp-contract=off", "-Wall", "-Wno-unused-function"]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    deps = SOURCES + ["gk_oracle.h", "build.py"]
    return all(os.path.getmtime(os.path.join(HERE, s)) <= t for s in deps)


def build(force: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = ["gcc", *CFLAGS, "-o", LIB + ".tmp", *[os.path.join(HERE, s) for s in SOURCES], "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
