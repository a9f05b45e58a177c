"""Build recipe for the CPU oracle (test infrastructure).

g++ with -ffp-contract=off and no fast-math so every f32 operation is a
separate IEEE round-to-nearest step, as in the Rust reference. OpenMP
parallelizes across output rows/heads only, never inside a sum.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

_HERE = Path(__file__).resolve().parent
SRC = _HERE / "faber_oracle.cpp"
OUT = _HERE / "_build" / "libfaber_oracle.so"


def build(force: bool = False) -> Path:
    if OUT.exists() and not force and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off",
           "-fno-fast-math", "-fno-finite-math-only", "-fopenmp", "-fvisibility=hidden",
           str(SRC), "-o", str(OUT)]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
