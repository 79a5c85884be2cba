"""Build recipe for the CPU oracle (test infrastructure only).

Compiles oracle.c into oracle/_build/liboracle.so with strict IEEE float
semantics (-ffp-contract=off, no fast-math) so each value is computed in the
same order and rounding as the reference's scalar x86 path.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle.so")
SRCS = [os.path.join(HERE, "oracle.c")]


def build(force: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    newest = max(os.path.getmtime(p) for p in SRCS + [os.path.join(HERE, "oracle.h")])
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= newest:
        return LIB
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC", "-shared",
           "-std=c11", "-Wall", "-Wno-unused-function", "-Wno-psabi", "-o", LIB] + SRCS + ["-lm"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
