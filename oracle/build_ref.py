"""Build recipe for ``oracle/_ref``: the reference's own CPU code, compiled in place.

Test infrastructure only.  Compiles, straight from the reference checkout (never
copied into this repository):

* ``library/AdaptiveIMI/cpp_extensions/src/kmeans_core.cpp`` and
  ``reorganize_core.cpp`` plus ``oracle/ref_shim.cpp`` -> ``oracle/_ref/imi_ref*.so``
  (k-means + CSR reorganize, the reference's index build);
* ``library/AdaptiveIMI/cpp_extensions/src/wave_buffer_cpu_hotcold.cpp`` ->
  ``oracle/_ref/AdpIMI_Index*.so`` (the page-cache manager whose ``batch_access``
  defines the page truncation of the selected cells).

The flags are the reference's host flags (``cpp_extensions/setup.py:42-48``:
``-O3 -std=c++17 -fPIC -fopenmp -march=native``).  This runs ``g++`` directly on
those files; the reference's own ``setup.py`` / ``build.sh`` are not used.  The
outputs go to ``oracle/_ref/`` (git-ignored, but carried to the GPU box), so the
GPU box never needs the reference checkout.

Usage: ``python oracle/build_ref.py [REFERENCE_ROOT]``.  Does nothing (and says
so) when the reference checkout is absent.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
DEFAULT_REF = Path("/root/reference")


def _torch_flags():
    import torch.utils.cpp_extension as ce

    inc = [f"-I{p}" for p in ce.include_paths()]
    libdir = ce.library_paths()[0]
    libs = [f"-L{libdir}", f"-Wl,-rpath,{libdir}", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python"]
    return inc, libs


def build(ref_root: Path | None = None, force: bool = False) -> bool:
    ref_root = Path(ref_root or os.environ.get("IMI_REFERENCE_ROOT", DEFAULT_REF))
    src = ref_root / "library" / "AdaptiveIMI" / "cpp_extensions"
    if not (src / "src" / "kmeans_core.cpp").exists():
        print(f"[oracle/_ref] reference sources not found under {ref_root}; skipping")
        return False
    OUT.mkdir(exist_ok=True)
    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    inc, libs = _torch_flags()
    py_inc = f"-I{sysconfig.get_paths()['include']}"
    flags = ["-O3", "-std=c++17", "-fPIC", "-fopenmp", "-march=native", "-shared",
             "-DTORCH_API_INCLUDE_EXTENSION_H", "-D_GLIBCXX_USE_CXX11_ABI=1", py_inc,
             f"-I{src / 'include'}", "-I/usr/local/cuda/include"] + inc
    jobs = [
        ("imi_ref", [HERE / "ref_shim.cpp", src / "src" / "kmeans_core.cpp", src / "src" / "reorganize_core.cpp"],
         ["-DTORCH_EXTENSION_NAME=imi_ref"]),
        ("AdpIMI_Index", [src / "src" / "wave_buffer_cpu_hotcold.cpp"], ["-DTORCH_EXTENSION_NAME=AdpIMI_Index"]),
    ]
    ok = True
    for name, files, extra in jobs:
        target = OUT / f"{name}{suffix}"
        newest = max(f.stat().st_mtime for f in files)
        if target.exists() and target.stat().st_mtime >= newest and not force:
            continue
        cmd = ["g++"] + flags + extra + [str(f) for f in files] + ["-o", str(target)] + libs + ["-fopenmp"]
        print("[oracle/_ref]", " ".join(cmd[:3]), "...", target.name)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            print(r.stderr[-4000:])
            ok = False
    return ok


if __name__ == "__main__":
    sys.exit(0 if build(sys.argv[1] if len(sys.argv) > 1 else None, force="--force" in sys.argv) else 1)
