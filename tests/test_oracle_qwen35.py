"""The Qwen3.5 DeltaNet tree-kernel oracle against the reference's own
known-answer tests (inputs and NumPy reference outputs captured from
tests/test_qwen35_tree_kernels.py of the reference by
tests/golden/make_qwen35_golden.py; tolerance atol = rtol = 1e-5 as there)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import qwen35 as Q
from oracle import tree as OT


@pytest.fixture(scope="module")
def kat(golden_dir):
    return dict(np.load(golden_dir / "qwen35_tree_kernels.npz"))


def test_conv1d_matches_reference_kat(kat):
    out, states = Q.tree_conv1d(kat["conv_qkv"][0], kat["conv_base"][0], kat["conv_weight"], kat["conv_parents"])
    np.testing.assert_allclose(out, kat["conv_out"][0], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(states, kat["conv_states"][0], atol=1e-5, rtol=1e-5)


def test_gated_delta_matches_reference_kat(kat):
    y, states = Q.tree_gated_delta(kat["delta_q"][0], kat["delta_k"][0], kat["delta_v"][0], kat["delta_g"][0],
                                   kat["delta_beta"][0], kat["delta_state"][0], kat["delta_parents"])
    np.testing.assert_allclose(y, kat["delta_out"][0], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(states, kat["delta_states"][0], atol=1e-5, rtol=1e-5)


def test_commit_takes_deepest_accepted_node(kat):
    parents = kat["delta_parents"]
    _, states = Q.tree_gated_delta(kat["delta_q"][0], kat["delta_k"][0], kat["delta_v"][0], kat["delta_g"][0],
                                   kat["delta_beta"][0], kat["delta_state"][0], parents)
    _, cstates = Q.tree_conv1d(kat["conv_qkv"][0], kat["conv_base"][0], kat["conv_weight"], kat["conv_parents"])
    lineages = OT.build_node_lineages([int(p) for p in parents])
    accepted = lineages[3] + [3]  # root -> node 3 (parents [-1, 0, 0, 1, 2])
    assert accepted == [0, 1, 3]
    s, c = Q.commit_path(states, cstates, accepted)
    assert np.array_equal(s, states[3]) and np.array_equal(c, cstates[3])


def test_bf16_rounding_of_states():
    rng = np.random.default_rng(7)
    x = rng.standard_normal(1000).astype(np.float32)
    r = Q._round(x, "bf16")
    assert np.all((r.view(np.uint32) & 0xFFFF) == 0)
    assert np.max(np.abs(r - x) / np.abs(x)) <= 2.0 ** -8
