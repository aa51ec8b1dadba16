"""Shared pytest configuration.

``-m gpu`` tests need a CUDA device and the in-tree ``libdtree_b200.so``;
everything else runs on CPU.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built library")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return ROOT / "tests" / "golden"


def pytest_collection_modifyitems(config, items):
    """GPU tests are skipped (not failed) on a machine without CUDA."""
    try:
        import torch

        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def lib():
    """The in-tree C-ABI library (built here if it is missing)."""
    from dtree_mlx_b200 import _lib, build

    if not _lib.LIB_PATH.exists():
        build.build()
    return _lib.load()
