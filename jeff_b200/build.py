"""Builds libjeffb200.so in-tree (jeff_b200/libjeffb200.so) with nvcc for sm_100a.

    python -m jeff_b200.build [--verbose] [--trace]

One translation unit (csrc/lib.cu includes the kernel files), the CUDA runtime linked statically, so the library
loads anywhere the driver exists (and, without a GPU, still loads and exports its symbols). --trace builds
libjeffb200_trace.so beside it, with the shared-memory product kernel's stage trace compiled in (-DJB_TRACE, read out
by its extra entry jb_stage_trace_read, a measurement aid outside the product header); the library the package loads
is always the one without. Without --force an up-to-date library (newer than every source) is kept."""

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
TRACE_LIB = HERE / "libjeffb200_trace.so"
INCLUDE = HERE.parent / "include"


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def sources() -> list[Path]:
    return sorted(SRC.glob("*.cu")) + sorted(SRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date(lib: Path = LIB) -> bool:
    if not lib.exists():
        return False
    built = lib.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in sources())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False, trace: bool = False) -> Path:
    lib = TRACE_LIB if trace else LIB
    if not force and up_to_date(lib):
        return lib
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
           "-shared", "-Xcompiler", "-fPIC", "-cudart", "static", *(["-DJB_TRACE"] if trace else []),
           f"-I{INCLUDE}", "-o", str(lib) + ".tmp", str(SRC / "lib.cu")]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or ptxas_info:
        print(res.stderr, file=sys.stderr)
    os.replace(str(lib) + ".tmp", lib)
    return lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--trace", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info, trace=args.trace))


if __name__ == "__main__":
    main()
