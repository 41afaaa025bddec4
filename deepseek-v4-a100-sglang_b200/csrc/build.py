"""Build the C-ABI shared library libdsv4_b200.so for sm_100a, in-tree.

    python build.py            # -> ../dsv4_b200/libdsv4_b200.so
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent / "dsv4_b200"
INCLUDE = HERE.parent.parent / "include"
LIB = PKG / "libdsv4_b200.so"
SOURCES = [HERE / "dsv4_b200.cu"]
DEPS = SOURCES + sorted(HERE.glob("*.cuh")) + [INCLUDE / "dsv4_b200.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    PKG.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(HERE), *map(str, SOURCES), "-o", str(tmp)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libdsv4_b200.so")
    if verbose:
        sys.stderr.write(res.stderr)
    (HERE.parent / "ptxas_report.txt").write_text(res.stderr) if verbose else None
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
