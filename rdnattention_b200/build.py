"""Builds librdnattention.so for sm_100a in-tree (rdnattention_b200/lib/).

    python -m rdnattention_b200.build [--force] [--verbose-ptxas]

Plain nvcc, no torch extension machinery: the product is a C-ABI shared
library that links only the CUDA runtime (the driver entry point for TMA
tensor maps is resolved at run time through cudaGetDriverEntryPoint).
"""
import hashlib
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "librdnattention.so"
STAMP = LIB_DIR / ".build_stamp"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["forward.cu"]
CPP_SOURCES = ["c_api.cpp"]


def _sources():
    files = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.cpp"))
    files += sorted(INCLUDE.rglob("*.h")) + sorted(INCLUDE.rglob("*.hpp"))
    return files


def _digest(extra=()):
    h = hashlib.sha256()
    for f in _sources():
        h.update(f.name.encode())
        h.update(f.read_bytes())
    for e in extra:
        h.update(e.encode())
    return h.hexdigest()


def build(force: bool = False, ptxas_verbose: bool = False) -> Path:
    LIB_DIR.mkdir(exist_ok=True)
    flags = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
             f"-I{INCLUDE}", f"-I{CSRC}"]
    digest = _digest(flags + ARCH)
    if not force and LIB.exists() and STAMP.exists() and STAMP.read_text() == digest:
        return LIB
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    for src in CU_SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [NVCC, *ARCH, *flags, "-c", str(CSRC / src), "-o", str(obj)]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        subprocess.run(cmd, check=True)
        objs.append(obj)
    for src in CPP_SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        subprocess.run([NVCC, *flags, "-x", "cu", "-c", str(CSRC / src), "-o", str(obj), *ARCH], check=True)
        objs.append(obj)
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    subprocess.run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"], check=True)
    os.replace(tmp, LIB)
    STAMP.write_text(digest)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, ptxas_verbose="--verbose-ptxas" in sys.argv))
