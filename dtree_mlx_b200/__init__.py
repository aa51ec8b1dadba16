"""B200-native DTree/DFlash speculative-decoding step (drop-in for dtree_mlx).

The public names match dtree_mlx/__init__.py:9-22.  Heavy modules (torch,
the CUDA library) load lazily on first attribute access.
"""
from __future__ import annotations

import importlib

__all__ = [
    "DFlashGenerator",
    "DFlashResult",
    "Generator",
    "DFlashDraftModel",
    "LoadedTargetModel",
    "adapter_for_model_type",
    "dflash_generate",
    "dtree_generate",
    "load_draft_model",
    "load_target_model",
    "longest_prefix_match",
    "sample_tokens",
]

_WHERE = {
    "DFlashGenerator": "api",
    "DFlashResult": "api",
    "Generator": "api",
    "DFlashDraftModel": "draft",
    "load_draft_model": "draft",
    "LoadedTargetModel": "adapters",
    "adapter_for_model_type": "adapters",
    "load_target_model": "adapters",
    "dflash_generate": "runtime",
    "longest_prefix_match": "runtime",
    "sample_tokens": "runtime",
    "dtree_generate": "dtree_runtime",
}


def __getattr__(name: str):
    mod = _WHERE.get(name)
    if mod is None:
        raise AttributeError(name)
    return getattr(importlib.import_module(f".{mod}", __name__), name)
