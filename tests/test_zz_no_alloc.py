"""dtree_tree_build_noalloc: the tree build for callers that cannot allocate.

Some callers of this library cannot allocate device memory while they decode:
a serving loop that runs under a fixed memory budget and must not call
cudaMalloc (or any routine that allocates), or a host runtime that only hands
the library buffers it already owns.  ``dtree_tree_build_noalloc`` serves them
with the scratch held in a fixed device array inside the library instead of a
caller workspace.  These tests call it through the C ABI and check that it
builds exactly the tree ``dtree_tree_build`` (the workspace version) builds,
on two calls in a row, and that oversized requests are rejected.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from dtree_mlx_b200 import _lib

DEV = "cuda"


def _outputs():
    z = lambda *s, dt=torch.int32: torch.zeros(*s, dtype=dt, device=DEV)  # noqa: E731
    return {"tokens": z(128), "parents": z(128), "depths": z(128), "positions": z(128),
            "anc": z(128, 2, dt=torch.int64)}


def _state(start, root):
    s = torch.zeros(8, dtype=torch.int32, device=DEV)
    s[0], s[1] = start, root
    return s


def _args(o):
    return [o["tokens"].data_ptr(), o["parents"].data_ptr(), o["depths"].data_ptr(), o["positions"].data_ptr(),
            o["anc"].data_ptr()]


@pytest.mark.gpu
def test_noalloc_matches_workspace_build_twice(lib):
    rng = np.random.default_rng(2024)
    rows, vocab, budget = 15, 151936, 24
    stream = torch.cuda.current_stream().cuda_stream
    ws_bytes = int(lib.dtree_tree_build_workspace_bytes(rows, vocab, budget))
    assert ws_bytes <= int(lib.dtree_tree_build_noalloc_max_bytes())
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=DEV)
    for call in range(2):  # two calls in a row share (and reuse) the fixed scratch
        logits = rng.standard_normal((rows, vocab)).astype(np.float32)
        logits[:, rng.integers(vocab, size=6)] += 7.0
        lg = torch.from_numpy(logits).to(DEV)
        ref, got = _outputs(), _outputs()
        s_ref, s_got = _state(300 + call, 11), _state(300 + call, 11)
        _lib.call("dtree_tree_build", lg.data_ptr(), rows, vocab, budget, s_ref.data_ptr(), ws.data_ptr(), ws_bytes,
                  *_args(ref), None, None, stream)
        _lib.call("dtree_tree_build_noalloc", lg.data_ptr(), rows, vocab, budget, s_got.data_ptr(), *_args(got),
                  stream)
        torch.cuda.synchronize()
        assert torch.equal(s_ref, s_got)
        n = int(s_ref[6].item())
        assert n == budget + 1
        for key in ref:
            assert torch.equal(ref[key][:n], got[key][:n]), (call, key)
    assert _lib.device_error() == 0


def test_noalloc_rejects_oversized_requests(lib):
    """Sizes beyond the fixed scratch are refused before any GPU work."""
    st = C.c_void_p(1)
    rc = lib.dtree_tree_build_noalloc(st, 65, 1000, 8, st, st, st, st, st, st, None)
    assert rc == -1 and "rows" in _lib.last_error()
    assert int(lib.dtree_tree_build_noalloc_max_bytes()) == 1 << 20


def test_noalloc_rejects_vocab_beyond_the_scratch(lib):
    """The fixed scratch bounds the vocabulary (per draft-row count); a larger
    one is refused with DTREE_ERR_CAPACITY before any GPU work."""
    st = C.c_void_p(1)
    vmax = int(lib.dtree_tree_build_noalloc_max_vocab(64))
    assert 300_000 < vmax < 400_000
    assert int(lib.dtree_tree_build_noalloc_max_vocab(16)) > vmax
    rc = lib.dtree_tree_build_noalloc(st, 64, vmax + 1, 24, st, st, st, st, st, st, None)
    assert rc == -4 and "vocab" in _lib.last_error()
