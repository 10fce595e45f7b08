"""The C-ABI library loads and exports every symbol include/b200q.h declares
(no GPU needed: nothing here launches a kernel)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols() -> list[str]:
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = h.read_text()
        names += re.findall(r"^B200Q_API\s+[\w\s\*]+?\b((?:simd|b200q)_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_reference_entry_points():
    names = set(_declared_symbols())
    for q in ("q4k", "q4k_r4", "q6k", "q6k_r4", "q6k_lm", "q8_0"):
        assert f"simd_matvec_{q}" in names
    for q in ("q4k", "q4k_r4", "q6k", "q6k_r4", "q8_0"):
        assert f"simd_matmul_{q}" in names


def test_library_exports_every_declared_symbol():
    from cybel_b200 import _native

    if not _native.LIB_PATH.exists():
        from cybel_b200 import build

        build.build()
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    missing = [n for n in _declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"
    # every declared symbol also has a ctypes signature in the loader
    assert set(_declared_symbols()) <= set(_native.SIGNATURES)


def test_controls_without_gpu():
    from cybel_b200 import _native

    L = _native.lib()
    assert L.b200q_version().startswith(b"b200q")
    assert L.b200q_status_string(-7) == b"kernel pipeline wait timed out"
    prev = L.b200q_set_act_mode(1)
    assert L.b200q_get_act_mode() == 1
    L.b200q_set_act_mode(prev)
    assert L.b200q_weight_cache_bytes() == 0
