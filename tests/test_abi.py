"""The C-ABI library loads and exports exactly what include/aios_b200.h declares
(no compute calls: this runs without a GPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

from aios_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "aios_b200.h"


def _declared() -> set[str]:
    return set(re.findall(r"AIOSB_API\s+(?:int|int64_t)\s+(aiosb_\w+)\s*\(", HEADER.read_text()))


def test_library_exports_every_declared_symbol() -> None:
    lib = _lib.load()
    declared = _declared()
    assert declared, "no declarations parsed from the header"
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(_lib.EXPORTED)


def test_version_and_error_reporting_without_gpu() -> None:
    lib = _lib.load()
    assert lib.aiosb_version() >= 100
    # argument validation happens before any CUDA call, so it works on a CPU box
    rc = lib.aiosb_linear(None, 4, 100, None, 128, None, 128, 0, None, 0, None, None)
    assert rc == _lib.ERR_UNSUPPORTED
    assert "multiple of 64" in _lib.last_error()
    rc = lib.aiosb_attnres_mix(None, 0, 1, 8, None, None, ctypes.c_float(1e-6), None, None, None)
    assert rc == _lib.ERR_INVALID_ARG
    assert "positive" in _lib.last_error()


def test_group_structs_match_header_layout() -> None:
    text = HEADER.read_text()
    state_fields = re.findall(r"^\s+(?:int32_t|int64_t|float)\s+(\w+);", text.split("typedef struct aiosb_group_state")[1].split("}")[0], re.M)
    assert state_fields == [f[0] for f in _lib.GroupState._fields_]
    ptr_block = text.split("typedef struct aiosb_group_ptrs")[1].split("} aiosb_group_ptrs")[0]
    ptr_fields = re.findall(r"(?:\*\s*|\bint64_t\s+)(\w+);", ptr_block)
    assert ptr_fields == [f[0] for f in _lib.GroupPtrs._fields_]
