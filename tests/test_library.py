"""The C-ABI library loads and exports exactly what include/dtree_b200.h declares.

No GPU needed: only symbol lookup and the host-side argument validation that
every entry point performs before touching CUDA.
"""
from __future__ import annotations

import ctypes as C
import re

import pytest

from dtree_mlx_b200 import _lib

ROOT = _lib.LIB_PATH.parents[1]


def header_symbols() -> list[str]:
    names = []
    for h in (ROOT / "include").glob("*.h"):
        names += re.findall(r"DTREE_API\s+[\w\s\*]+?\b(dtree_\w+)\s*\(", h.read_text())
    return sorted(set(names))


def test_header_declares_entry_points():
    names = header_symbols()
    assert "dtree_tree_build" in names and "dtree_qwen3_forward_tree" in names
    assert len(names) >= 20


def test_every_declared_symbol_is_exported(lib):
    for name in header_symbols():
        assert hasattr(lib, name), f"libdtree_b200.so does not export {name}"


def test_bindings_cover_header():
    assert set(header_symbols()) <= set(_lib.PROTOTYPES)


def test_version(lib):
    assert lib.dtree_version() == 100


def test_argument_validation_without_gpu(lib):
    st = C.c_void_p(1)
    # budget out of range is rejected before any CUDA call
    rc = lib.dtree_tree_build(None, 4, 16, 500, st, None, 0, st, st, st, st, st, None, None, None)
    assert rc == -1 and "budget" in _lib.last_error()
    rc = lib.dtree_kv_compact(st, 1, 1, 16, 7, st, st, None)
    assert rc == -1 and "head_dim" in _lib.last_error()
    rc = lib.dtree_gather_rows(st, 15, st, st, st, 4, None)
    assert rc == -1 and "row_bytes" in _lib.last_error()
    with pytest.raises(_lib.DTreeError):
        _lib.call("dtree_linear_bf16", st, 24, 64, st, 128, st, st, 1 << 30, 0, None)


def test_step_state_layout():
    assert C.sizeof(_lib.StepState) == 32
    assert _lib.STEP_STATE_FIELDS[:2] == ["start", "root_token"]
