"""Build libfaber_gpu.so in-tree for sm_100a (nvcc cross-compiles without a GPU)."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "libfaber_gpu.so"
SOURCES = [CSRC / "faber_gpu.cu", CSRC / "synth.cpp"]
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + [ROOT / "include" / "faber_gpu.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs() -> tuple[Path, Path]:
    """Headers and library of the NCCL that ships with torch (2.28)."""
    import importlib.util
    spec = importlib.util.find_spec("nvidia.nccl")
    if spec and spec.submodule_search_locations:
        base = Path(list(spec.submodule_search_locations)[0])
        if (base / "include" / "nccl.h").exists():
            return base / "include", base / "lib"
    return Path("/usr/include"), Path("/usr/lib/x86_64-linux-gnu")


def needs_build() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    if not force and not needs_build():
        return OUT
    inc, lib = nccl_dirs()
    cmd = ["nvcc", *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC,-fvisibility=hidden,-ffp-contract=off,-O2",
           "-I", str(ROOT / "include"), "-I", str(inc),
           *[str(s) for s in SOURCES],
           "-L", str(lib), "-l:libnccl.so.2", "-Xlinker", f"-rpath,{lib}",
           "-o", str(OUT)]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force=True, verbose_ptxas="-v" in sys.argv))
