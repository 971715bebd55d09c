"""Build recipe for the oracle restatement (test infrastructure only).

Compiles ``oracle/imi_oracle.cpp`` with ``g++ -O2 -ffp-contract=off`` into
``oracle/_build/libimi_oracle.so``.  ``-ffp-contract=off`` keeps every
multiply-add that the restatement writes as two operations as two operations;
the fused ones are written with ``std::fma`` explicitly.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "imi_oracle.cpp"
OUT = HERE / "_build" / "libimi_oracle.so"


def build(force: bool = False) -> Path:
    OUT.parent.mkdir(exist_ok=True)
    if OUT.exists() and OUT.stat().st_mtime >= SRC.stat().st_mtime and not force:
        return OUT
    cmd = ["g++", "-O3", "-march=x86-64-v3", "-std=c++17", "-ffp-contract=off", "-fPIC", "-shared", str(SRC), "-o", str(OUT)]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
