"""Build the sm_100a shared library ``libmaple_b200.so`` in-tree with nvcc.

The library is a plain C ABI (``include/maple_b200.h``) loaded with ctypes,
so it carries no torch or Python types and is built straight by nvcc:

    python -m maple_flash_dgx_spark_b200.build
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libmaple_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--fmad=false",          # canonical numerics: no implicit mul+add contraction
    "-Xcompiler", "-fPIC",
    "-shared",
    f"-I{REPO / 'include'}",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build maple-b200")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + [REPO / "include" / "maple_b200.h"]
    return any(p.stat().st_mtime > t for p in deps)


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *map(str, sources()), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
    print(LIB)
