"""Build recipe for the product library ``adaptiveimi_b200/lib/libimi_b200.so``.

``nvcc -gencode arch=compute_100a,code=sm_100a`` on the CUDA sources in this
directory, statically linked against the CUDA runtime, exporting only the C ABI
of ``include/imi_b200.h``.  The object files are cached next to the library so
that an unchanged source is not recompiled.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
ROOT = PKG.parent
OUT = PKG / "lib" / "libimi_b200.so"
OBJ = PKG / "lib" / "obj"
SOURCES = ["decode.cu", "select.cu", "attention.cu", "build.cu", "peer.cu", "capi.cu"]
HEADERS = ["common.cuh", "imi_internal.h", "select_core.cuh", "attn_core.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}"]


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(parents=True, exist_ok=True)
    hdrs = [HERE / h for h in HEADERS] + [ROOT / "include" / "imi_b200.h"]
    objs = []
    for src in SOURCES:
        obj = OBJ / (src + ".o")
        objs.append(obj)
        if force or _stale(obj, [HERE / src] + hdrs):
            cmd = [NVCC] + FLAGS + ["-c", str(HERE / src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            print("[imi_b200] nvcc", src, flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(OUT, objs):
        cmd = [NVCC, "-shared", "-cudart", "static", "-gencode", "arch=compute_100a,code=sm_100a"] + \
              [str(o) for o in objs] + ["-o", str(OUT)]
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
