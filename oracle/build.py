"""Builds the CPU oracle (test infrastructure) into oracle/_build/liboracle.so.

    python oracle/build.py

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
the result; the product library never does.
"""
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_build"
LIB = OUT_DIR / "liboracle.so"
SRC = HERE / "attn_oracle.c"


def build(force: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared", "-std=c11",
           "-fvisibility=hidden", "-o", str(tmp), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
