"""Build recipe for ``oracle/_ref/libref_scorer.so``: the reference's own CUDA
decode scorer, compiled in place for sm_100a.

Test infrastructure only.  ``nvcc`` compiles, straight from the reference
checkout (never copied into this repository),
``library/AdaptiveIMI/cpp_extensions/cuda/compute_impl.cu`` (the
``fused_query_group_similarity_kernel`` of lines 62-103 and its launcher) with
the reference's nvcc flags (``cpp_extensions/setup.py``: ``-O3 -std=c++17
--expt-relaxed-constexpr -lineinfo``, so fma contraction stays at nvcc's
default), together with ``oracle/ref_scorer_shim.cu``, a C entry point without
torch types.  The output goes to ``oracle/_ref/`` (git-ignored, carried to the
GPU box).  Does nothing (and says so) when the reference checkout is absent.

Usage: ``python oracle/build_ref_cuda.py [REFERENCE_ROOT]``.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "libref_scorer.so"
DEFAULT_REF = Path("/root/reference")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def build(ref_root: Path | None = None, force: bool = False) -> bool:
    ref_root = Path(ref_root or os.environ.get("IMI_REFERENCE_ROOT", DEFAULT_REF))
    src = ref_root / "library" / "AdaptiveIMI" / "cpp_extensions" / "cuda" / "compute_impl.cu"
    if not src.exists():
        print(f"[oracle/_ref] reference CUDA sources not found under {ref_root}; skipping")
        return False
    OUT.parent.mkdir(exist_ok=True)
    shim = HERE / "ref_scorer_shim.cu"
    if OUT.exists() and not force and OUT.stat().st_mtime >= max(src.stat().st_mtime, shim.stat().st_mtime):
        return True
    cmd = [NVCC, "-O3", "-std=c++17", "--expt-relaxed-constexpr", "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
           "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static", str(src), str(shim), "-o", str(OUT)]
    print("[oracle/_ref] nvcc compute_impl.cu ->", OUT.name)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        print(r.stderr[-4000:])
        return False
    return True


if __name__ == "__main__":
    sys.exit(0 if build(sys.argv[1] if len(sys.argv) > 1 else None, force="--force" in sys.argv) else 1)
