"""Build the sm_100a C-ABI library in-tree: attention_lab_b200/libattention_lab_b200.so.

    python -m attention_lab_b200.build [--verbose]

One nvcc invocation over csrc/al_capi.cu (which includes every kernel header), static CUDA runtime, position
independent code. `--verbose` adds `-Xptxas -v` (registers, spills and shared memory per kernel).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
SRC = PKG / "csrc"
LIB = PKG / "libattention_lab_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(SRC.glob("*.cu")) + sorted(SRC.glob("*.cuh")) + [PKG.parent / "include" / "attention_lab_b200.h"]


def up_to_date() -> bool:
    return LIB.exists() and all(LIB.stat().st_mtime >= s.stat().st_mtime for s in sources())


def build(verbose: bool = False, force: bool = False) -> Path:
    if up_to_date() and not force:
        return LIB
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
           "--expt-relaxed-constexpr", "-I", str(PKG.parent / "include"), str(SRC / "al_capi.cu"),
           "-o", str(LIB) + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed with exit code {res.returncode}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
