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
SOURCES = [CSRC / "ffnrm.cu", PKG / "host" / "base_producer.cpp"]
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted((PKG / "host").glob("*.hpp")) + [ROOT / "include" / "ffnrm.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def command(out: Path = LIB, extra: list[str] | None = None) -> list[str]:
    return [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
            "-cudart", "static", "-Xcompiler", "-mavx2", "-I", str(ROOT / "include"), "-I", str(CSRC), "-I", str(PKG / "host"),
            *(extra or []), *map(str, SOURCES), "-o", str(out)]


# Drop-in runner executables (same argv / exit codes / JSON as the reference's runners),
# host C++ over the C ABI; they find libffnrm.so through an $ORIGIN-relative rpath.
HOST = PKG / "host"
BIN_DIR = PKG / "bin"
RUNNERS = ["exact_residual_cuda_runner", "exact_main_residual_cuda_runner", "exact_cpu_base_gpu_full_ffn_runner"]
HOST_HEADERS = sorted(HOST.glob("*.hpp"))


def runner_command(name: str) -> list[str]:
    return [nvcc(), *ARCH, "-O3", "-std=c++17", "-Xcompiler", "-mavx2,-pthread", "-I", str(ROOT / "include"), "-I", str(HOST),
            str(HOST / f"{name}.cpp"), "-L", str(LIB_DIR), "-lffnrm", "-Xlinker", "-rpath,$ORIGIN/../lib",
            "-o", str(BIN_DIR / name)]


def stale(target: Path = LIB, deps: list[Path] | None = None) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in (deps if deps is not None else SOURCES + HEADERS))


def build_runners(force: bool = False, verbose: bool = False) -> list[Path]:
    BIN_DIR.mkdir(exist_ok=True)
    out = []
    for name in RUNNERS:
        exe = BIN_DIR / name
        if force or stale(exe, [HOST / f"{name}.cpp", LIB, ROOT / "include" / "ffnrm.h", *HOST_HEADERS]):
            cmd = runner_command(name)
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
        out.append(exe)
    return out


def build(force: bool = False, verbose: bool = False, runners: bool = True) -> Path:
    if force or stale():
        LIB_DIR.mkdir(exist_ok=True)
        cmd = command()
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    if runners:
        build_runners(force, verbose)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
