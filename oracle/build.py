"""Build recipe for the CPU oracle ``oracle/liboracle.so`` (test infrastructure).

    python -m oracle.build

``-ffp-contract=off`` keeps every multiply and add a separate IEEE rounding
unless the source calls fmaf(), matching the CUDA library's ``--fmad=false``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
SRC = [HERE / "oracle.c"]

CFLAGS = ["-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
          "-fopenmp"]


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and all(s.stat().st_mtime <= LIB.stat().st_mtime for s in SRC):
        return LIB
    cc = shutil.which("gcc") or "cc"
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([cc, *CFLAGS, *map(str, SRC), "-o", str(tmp), "-lm"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
