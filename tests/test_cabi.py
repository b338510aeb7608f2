"""The C-ABI library loads and exports every symbol include/maple_b200.h declares (no GPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def declared_symbols() -> list[str]:
    text = (REPO / "include" / "maple_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(maple_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_declared_symbols():
    from maple_flash_dgx_spark_b200 import _lib
    from maple_flash_dgx_spark_b200.build import build

    build()
    L = ctypes.CDLL(str(_lib.LIB_PATH))
    syms = declared_symbols()
    assert syms, "header declares no entry points"
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    # every declared symbol has a ctypes signature in the Python binding
    assert set(syms) <= set(_lib.exported_symbols()), set(syms) - set(_lib.exported_symbols())


def test_pure_shape_queries():
    from maple_flash_dgx_spark_b200 import _lib

    L = _lib.lib()
    assert L.maple_router_topk_workspace_bytes(1, 64) > 0
    assert L.maple_decode_gqa_workspace_bytes(1, 32, 128, 4096, 64) > 0
    assert L.maple_ternary_gemv_workspace_bytes(1, 5120, 2048) >= 0
