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


def test_tc_attention_host_checks():
    """The tensor-core attention entry refuses what it cannot run before any launch."""
    from maple_flash_dgx_spark_b200 import _lib

    L = _lib.lib()
    assert L.maple_decode_gqa_attn_tc_workspace_bytes(64, 32, 128, 8192) > 0
    d = ctypes.c_void_p(256)

    def call(x_dtype=1, heads=32, kv=4, hd=128):
        return L.maple_decode_gqa_attn_tc(d, x_dtype, 2, heads, heads * hd, hd, d, d, 2, kv, kv * 4096 * hd,
                                          4096 * hd, 4096, hd, d, None, 0.088, 0, d, heads * hd, hd, d, 1 << 30, d,
                                          None)

    assert call(x_dtype=0) == 2        # fp32 caches: the canonical kernel's job
    assert call(hd=256) == 1           # head_dim 64 or 128
    assert call(heads=48, kv=4) == 1   # more than 8 query heads per KV head
