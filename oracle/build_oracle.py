"""Builds the C part of the oracle (test infrastructure) with gcc into
oracle/_build/liboracle.so.  Only the checker is built here; nothing under
oracle/ is part of the product.

    python oracle/build_oracle.py [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "oracle_c.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB + f".{os.getpid()}.tmp"
    cmd = ["gcc", "-O3", "-mfma", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC", SRC, "-o", tmp,
           "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
