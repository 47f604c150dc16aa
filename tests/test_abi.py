"""The C-ABI library loads and exports every symbol include/*.h declares (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(?:int|size_t|void)\s*\*?\s*(sb_\w+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "sb_router_forward" in names and "sb_ternary_moe_swiglu" in names


def test_library_exports_every_declared_symbol():
    from sb200 import _lib
    lib = _lib.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"
    assert lib.sb_abi_version() == 1


def test_binding_table_covers_header():
    from sb200 import _lib
    assert set(declared_symbols()) <= set(_lib.exported_symbols())


def test_host_validation_without_gpu():
    """Argument checks run on the host and report through sb_last_error."""
    from sb200 import _lib
    lib = _lib.load()
    desc = _lib.RouterDesc()
    desc.hidden, desc.spectral, desc.n_levels = 30, 16, 3   # hidden not a multiple of 8
    for i in range(3):
        desc.branching[i] = 4
    h = ctypes.c_void_p()
    rc = lib.sb_router_create(ctypes.byref(desc), 0, ctypes.byref(h))
    assert rc == -1
    assert "hidden" in _lib.last_error()
    desc.hidden = 64
    rc = lib.sb_router_create(ctypes.byref(desc), 0, ctypes.byref(h))
    assert rc == 0 and h.value
    assert lib.sb_router_workspace_bytes(h, 256, 0) > 0
    rc = lib.sb_router_forward(h, None, 1, 4, 0, 0, 8, None, None, 0, None)
    assert rc == -1
    assert lib.sb_router_destroy(h) == 0
