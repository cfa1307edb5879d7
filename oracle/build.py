"""Compile the C oracle (oracle/kq_oracle.c) into oracle/liboracle.so (test infrastructure)."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "kq_oracle.c")
LIB = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-fopenmp",
                        "-std=gnu11", SRC, "-o", LIB, "-lm"], check=True)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
