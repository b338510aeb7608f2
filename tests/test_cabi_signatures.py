"""Every entry point's ctypes signature in the Python binding matches its
declaration in include/maple_b200.h parameter by parameter (pointer, int64,
int32, float) and in its return type (no GPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]

_KINDS = {ctypes.c_void_p: "ptr", ctypes.c_int64: "i64", ctypes.c_int: "i32", ctypes.c_float: "f32"}


def _kind(c_type: str) -> str:
    c_type = c_type.strip()
    if "*" in c_type:
        return "ptr"
    base = re.sub(r"\b(const|unsigned)\b", "", c_type).split()
    base = base[0] if base else ""
    return {"int64_t": "i64", "int": "i32", "int32_t": "i32", "float": "f32"}.get(base, f"?{c_type}")


def declarations() -> dict[str, tuple[str, list[str]]]:
    text = (REPO / "include" / "maple_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    out = {}
    for m in re.finditer(r"\b(int64_t|int)\s+(maple_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        ret, name, params = m.group(1), m.group(2), m.group(3).strip()
        kinds = [] if params in ("", "void") else [_kind(re.sub(r"\w+$", "", p.strip()))
                                                   for p in params.split(",")]
        out[name] = (_kind(ret), kinds)
    return out


def test_header_parses():
    decl = declarations()
    assert len(decl) > 40
    assert not [n for n, (_, ks) in decl.items() if any(k.startswith("?") for k in ks)]


def test_binding_matches_header():
    from maple_flash_dgx_spark_b200 import _lib

    decl = declarations()
    bad = []
    for name, (ret, kinds) in decl.items():
        sig = _lib._SIGS.get(name)
        if sig is None:
            bad.append(f"{name}: no binding")
            continue
        rtype, argtypes = sig
        got = [_KINDS.get(a, f"?{a}") for a in argtypes]
        if got != kinds:
            bad.append(f"{name}: header {kinds} binding {got}")
        if _KINDS.get(rtype) != ret:
            bad.append(f"{name}: returns {ret}, binding {rtype}")
    assert not bad, "\n".join(bad)
