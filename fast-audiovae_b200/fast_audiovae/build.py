"""Build the sm_100a CUDA library in-tree (``nvcc`` target of the package).

``python -m fast_audiovae.build`` (with ``fast-audiovae_b200`` on ``sys.path``)
compiles ``csrc/*.cu`` into ``fast_audiovae/libfav_cuda.so``. The library is
built for ``sm_100a`` only; it contains no CPU fallback.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
ROOT = PACKAGE_DIR.parent
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
LIBRARY = PACKAGE_DIR / "libfav_cuda.so"
SOURCES = ("fav_kernels.cu", "fav_tail.cu", "fav_stage.cu", "fav_prepass.cu", "fav_api.cu")
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden"]


def nvcc():
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build the decoder")
    return found


def inputs():
    return [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + \
        sorted(INCLUDE.glob("*.h"))


def up_to_date():
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in inputs())


def build(force=False, verbose=False):
    """Compile the library unless it is newer than every source. Returns its path."""
    if not force and up_to_date():
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), *[str(CSRC / s) for s in SOURCES], "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + result.stdout + result.stderr)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
