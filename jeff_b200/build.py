"""Builds libjeffb200.so in-tree (jeff_b200/libjeffb200.so) with nvcc for sm_100a.

    python -m jeff_b200.build [--verbose]

One translation unit (csrc/lib.cu includes the kernel files), the CUDA runtime linked statically, so the library
loads anywhere the driver exists (and, without a GPU, still loads and exports its symbols)."""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc"
LIB = HERE / "libjeffb200.so"
INCLUDE = HERE.parent / "include"


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def sources() -> list[Path]:
    return sorted(SRC.glob("*.cu")) + sorted(SRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    built = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in sources())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
           "-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
           f"-I{INCLUDE}", "-o", str(LIB) + ".tmp", str(SRC / "lib.cu")]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or ptxas_info:
        print(res.stderr, file=sys.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info))


if __name__ == "__main__":
    main()
