"""Build the in-tree CUDA library ``avqa_b200/libavqa_b200.so`` for sm_100a.

``python -m avqa_b200.build_ext`` (or ``__graft_entry__.build()``) compiles
every ``csrc/*.cu`` with nvcc into one shared library exporting the C ABI of
``include/avqa_b200.h``.  Objects are rebuilt only when a source or header is
newer than the library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libavqa_b200.so"
BUILD = ROOT / "_build"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and not shutil.which(cand):
        raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _newest_input() -> float:
    files = list(CSRC.glob("*")) + [ROOT / "include" / "avqa_b200.h"]
    return max(f.stat().st_mtime for f in files if f.is_file())


def build(force: bool = False, verbose: bool = False) -> Path:
    if LIB.exists() and not force and LIB.stat().st_mtime >= _newest_input():
        return LIB
    BUILD.mkdir(exist_ok=True)
    objs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *map(str, objs), "-o", str(tmp),
           "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
