"""Compile the CUDA sources of this package into ``libcce_b200.so`` (in-tree).

The library is built for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``)
with nvcc; it links the CUDA runtime statically and resolves the driver's
tensor-map encoder at run time, so it loads on a machine without a GPU and
needs nothing at run time but the NVIDIA driver.

    python mlx-cross-entropy_b200/mlx_cce/build.py           # rebuild if stale
    python mlx-cross-entropy_b200/mlx_cce/build.py --force

(Run it as a script: importing the package itself loads the library.)
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent                     # mlx-cross-entropy_b200/
CSRC = ROOT / "csrc"
REPO = ROOT.parent
INCLUDE = REPO / "include"
LIB_NAME = "libcce_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

SOURCES = ["cce_abi.cu", "aux_kernels.cu", "simt_kernels.cu", "tc_kernels.cu", "noalloc.cu", "peer.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-shared",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set $NVCC or put the CUDA toolkit on PATH")


def _deps():
    deps = [CSRC / s for s in SOURCES]
    deps += sorted(CSRC.glob("*.cuh"))
    deps += sorted(INCLUDE.glob("*.h"))
    return deps


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the shared library if missing or stale; return its path."""
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-o", str(tmp)]
    cmd += [str(CSRC / s) for s in SOURCES]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True)
    print(p)
