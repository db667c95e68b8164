"""Builds liblaya_b200.so in-tree with nvcc for sm_100a (B200).

    python -m laya_cuda.build            # from laya-cuda_b200/
"""
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE.parent / "csrc"
INCLUDE = PACKAGE.parents[1] / "include"
TARGET = PACKAGE / "liblaya_b200.so"
SOURCES = [CSRC / "laya_b200.cu"]
DEPENDS = SOURCES + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "laya_b200.h"]
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-shared", "-cudart", "static"]


def nvcc():
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found")
    return found


def up_to_date():
    if not TARGET.exists():
        return False
    built = TARGET.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in DEPENDS)


def build(force=False, verbose=False):
    if not force and up_to_date():
        return TARGET
    tmp = TARGET.with_suffix(".so.tmp")
    cmd = [nvcc(), *FLAGS, "-I", str(INCLUDE), "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, TARGET)
    return TARGET


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
