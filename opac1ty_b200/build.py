"""In-tree build of ``libopc_b200.so`` for sm_100a with nvcc (no JIT cache, no Triton)."""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
SOURCES = [CSRC / "opc_lib.cu", CSRC / "opc_engine.cu"]
DEPENDS = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
OUTPUT = PKG / "libopc_b200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not OUTPUT.exists():
        return False
    t = OUTPUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in DEPENDS)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUTPUT
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", str(INCLUDE), "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    print(build_library(force=True, verbose=True))
