"""Build libpalu_b200.so in-tree with nvcc for sm_100a (no JIT cache: the .so travels with the tree)."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
OUT = PKG / "libpalu_b200.so"
SOURCES = ["palu_abi.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def command(verbose_ptxas: bool = False) -> list:
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "--expt-relaxed-constexpr", "-o", str(OUT)] + [str(CSRC / s) for s in SOURCES]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    return cmd


def stale() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list((PKG.parent.parent / "include").glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    if force or stale():
        subprocess.run(command(verbose_ptxas), check=True, cwd=str(CSRC))
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
    print(OUT)
