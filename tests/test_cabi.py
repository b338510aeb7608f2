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


def test_decode_layers_host_checks():
    """Shape checks of the whole-stack decode entry run before any CUDA call."""
    from maple_flash_dgx_spark_b200 import _lib

    L = _lib.lib()
    assert L.maple_decode_layers_workspace_bytes(2048, 32, 4, 128, 64, 8, 1024, 4096, 64) > 0
    assert L.maple_decode_layers_workspace_bytes(2048, 32, 4, 128, 64, 8, 1024, 4096, 0) < 0
    args = dict(hidden=2048, heads=32, kv=4, hd=128, rot=128, E=64, topk=8, inter=1024)

    def call(n_layers=1, **kw):
        a = {**args, **kw}
        dummy = ctypes.c_void_p(16)
        return L.maple_decode_layers(dummy, n_layers, dummy, dummy, None, dummy, dummy, 1, 128, 4096, a["hidden"],
                                     a["heads"], a["kv"], a["hd"], a["rot"], a["E"], a["topk"], a["inter"], 1, 4096,
                                     4 * 4096 * 128, 4096 * 128, 64, 1, 0, 1, 1e-6, 0.088, dummy, 1 << 30,
                                     dummy, None)

    assert call(n_layers=0) == 0
    assert call(hd=96) == 1          # head_dim 64 or 128 only
    assert call(heads=48, kv=4) == 1  # more than 8 query heads per KV head
    assert call(topk=9) == 1
    assert call(inter=4096) == 1      # down K halves exceed the register tiles
