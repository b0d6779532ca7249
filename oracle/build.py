"""Build recipe for the CPU oracle (test infrastructure only).

Compiles oracle/reels_oracle.c with gcc into oracle/_build/libreels_oracle.so.
No -ffast-math: the quantiser relies on IEEE fp32 division and round-to-even.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libreels_oracle.so")
SRC = os.path.join(HERE, "reels_oracle.c")


def build(force: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-fno-fast-math",
           "-ffp-contract=off", "-o", LIB, SRC, "-lm"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
