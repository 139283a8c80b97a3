"""Build ``libffnrm.so`` (the C-ABI CUDA library) in-tree for sm_100a.

    python -m ffn_residual_mesh_b200.build

nvcc cross-compiles without a GPU. The shared library links the CUDA runtime
statically, so it needs only the driver at run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libffnrm.so"
SOURCES = [CSRC / "ffnrm.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "ffnrm.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def command(out: Path = LIB, extra: list[str] | None = None) -> list[str]:
    return [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
            "-cudart", "static", "-I", str(ROOT / "include"), "-I", str(CSRC),
            *(extra or []), *map(str, SOURCES), "-o", str(out)]


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if force or stale():
        LIB_DIR.mkdir(exist_ok=True)
        cmd = command()
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
