"""Build recipe of the CPU oracle (test infrastructure): oracle.c -> oracle/_build/liboracle.so.

The reference (huppiflupp/wgpu-ocr) is Rust + WGSL; no C or C++ part of it can be compiled
here, so there is no `oracle/_ref` build.  Usage: `python oracle/build.py` or `build()`.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle.so")
SRC = os.path.join(HERE, "oracle.c")

# x86-64-v3 (AVX2 + FMA): runs on this container and on the GPU hosts alike.
CFLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-std=c11", "-Wall",
          "-Wno-unused-function"]


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB + f".tmp{os.getpid()}"
    subprocess.run(["gcc", *CFLAGS, SRC, "-o", tmp, "-lm"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
