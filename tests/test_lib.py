"""The C-ABI library loads and exports every entry point include/pkv_b200.h declares (no GPU calls)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

from tests.conftest import ROOT


def _declared() -> set[str]:
    header = (ROOT / "include" / "pkv_b200.h").read_text()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    return set(re.findall(r"\b(pkv_[a-z0-9_]+)\s*\(", header))


def test_library_exports_every_declared_symbol():
    from randomrepo_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    declared = _declared()
    assert len(declared) >= 20
    missing = [name for name in sorted(declared) if not hasattr(lib, name)]
    assert not missing, missing
    assert set(_lib.exported_symbols()) <= declared


def test_library_is_built_for_sm100a():
    from randomrepo_b200 import _lib

    assert _lib.lib.pkv_version().decode().endswith("sm_100a")
    assert Path(_lib.LIB_PATH).stat().st_size > 0


def test_pool_bytes_formula():
    from randomrepo_b200 import _lib

    g = _lib.PoolGeom(28, 1000, 2, 16, 128, _lib.PKV_BF16)
    # layers x blocks x (K, V) x kv_heads x block_size x head_dim x 2 bytes
    assert _lib.lib.pkv_pool_bytes(ctypes.byref(g)) == 28 * 1000 * 2 * 2 * 16 * 128 * 2
