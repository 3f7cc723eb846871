"""Build the sm_100a C-ABI library ``libcimekv.so`` in-tree.

    python -m isa_b200.build        (or isa_b200.build.build_library())

nvcc cross-compiles for sm_100a without a GPU.  The library lands next to this
file in ``_lib/`` so it travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
SRC_DIR = PKG_DIR.parent / "csrc"
REPO_ROOT = PKG_DIR.parent.parent
INCLUDE_DIR = REPO_ROOT / "include"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libcimekv.so"
DEBUG_LIB_PATH = LIB_DIR / "libcimekv_debug.so"  # table-index bounds checks (CIMEKV_DEBUG_BOUNDS=1)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libcimekv")
    return cand


def sources() -> list[Path]:
    return sorted(SRC_DIR.glob("*.cu"))


def build_library(force: bool = False, verbose: bool = False, debug: bool = False) -> Path:
    """Compile csrc/*.cu into _lib/libcimekv.so (or the bounds-checking
    libcimekv_debug.so with debug=True); skipped when up to date."""
    srcs = sources()
    deps = srcs + sorted(INCLUDE_DIR.glob("*.h")) + sorted(SRC_DIR.glob("*.cuh"))
    out = DEBUG_LIB_PATH if debug else LIB_PATH
    if not force and out.exists():
        mtime = out.stat().st_mtime
        if all(p.stat().st_mtime <= mtime for p in deps):
            return out
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, f"-I{INCLUDE_DIR}", f"-I{SRC_DIR}", *map(str, srcs), "-o", str(tmp)]
    if debug:
        cmd.insert(1, "-DCIMEKV_DEBUG_BOUNDS=1")
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv, debug="--debug" in sys.argv))
