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
# The seeded input generator (plain C++, no GPU code) is linked in as well,
# so that a CPU-only user of the oracle (the benchmark's reference leg)
# draws the same synthetic weights without loading the GPU library.
ROOT = _HERE.parent
SYNTH = ROOT / "faber_runtime_b200" / "csrc" / "synth.cpp"
OUT = _HERE / "_build" / "libfaber_oracle.so"


def build(force: bool = False) -> Path:
    srcs = [SRC, SYNTH]
    if OUT.exists() and not force and all(OUT.stat().st_mtime >= s.stat().st_mtime for s in srcs):
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off",
           "-fno-fast-math", "-fno-finite-math-only", "-fopenmp", "-fvisibility=hidden",
           "-I", str(ROOT / "include"), *[str(s) for s in srcs], "-o", str(OUT), "-lpthread"]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
