"""Build the CPU oracle library (test infrastructure; see lq_oracle.c's header).

    python oracle/build.py        ->  oracle/_build/liblq_oracle.so

The reference (Generated-Computers/Locals) is Python + Metal over MLX; none of its hot-path
code is C or C++, so there is no ``oracle/_ref`` build: the restatement in lq_oracle.c is the
oracle and the timed CPU baseline ("kind": "port").
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liblq_oracle.so")
SRC = os.path.join(HERE, "lq_oracle.c")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = ["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-std=c11", "-Wall", "-o", LIB, SRC, "-lm"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
