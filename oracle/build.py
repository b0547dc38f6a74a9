"""Build recipe for the C oracle (test infrastructure, never part of the product).

Compiles oracle/w4_oracle.c with gcc into oracle/libw4oracle.so (OpenMP,
x86-64-v3 so the object runs on any AVX2 host). The reference itself is a
Python package, so there is no oracle/_ref build: golden vectors come from
importing the reference's packer (tests/golden/make_golden.py).
"""
from __future__ import annotations

import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
SRC = ORACLE_DIR / "w4_oracle.c"
LIB = ORACLE_DIR / "libw4oracle.so"


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-std=c11",
           str(SRC), "-o", str(LIB), "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"gcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force=True))
