"""Oracle tree/walk/lineage/compaction restatement vs the reference's own outputs.

The fixtures were produced by ``tests/golden/make_golden.py``, which runs the
reference functions (dtree_runtime.py:82-208, qwen35_tree.py:41-123,
adapters.py:635-668, runtime.py:33-39) unchanged.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from oracle import tree as T


@pytest.fixture(scope="module")
def golden(golden_dir):
    data = json.loads((golden_dir / "tree_golden.json").read_text())
    logits = np.load(golden_dir / "tree_logits.npz")
    return data, logits


def test_reference_unit_kat(golden):
    """tests/test_dtree_runtime.py:15-40 input; answer produced by the reference."""
    data, logits = golden
    case = data["trees"][0]
    assert case["name"] == "ref_unit_3x3_b4"
    tokens, depths, parents, child_maps, vis = T.build_dtree_tree(logits[case["name"]], 4)
    assert tokens == [0, 0, 0, 1]
    assert depths == [1, 2, 3, 1]
    assert parents == [-1, 0, 1, 2, 0]
    assert child_maps == [{0: 1, 1: 4}, {0: 2}, {0: 3}, {}, {}]
    assert vis.shape == (5, 5) and bool(vis[0, 0])


def test_heap_bit_exact_on_reference_log_probs(golden):
    """Given the reference's own top-k log-probs, the heap is bit-exact."""
    data, _ = golden
    for case in data["trees"]:
        if case["budget"] <= 0:
            continue
        ids = np.asarray(case["top_ids"], dtype=np.int64)
        lps = np.asarray(case["top_log_probs"], dtype=np.float32)
        tokens, depths, parents, child_maps = T.heap_build(ids, lps, case["budget"])
        assert tokens == case["node_token_ids"], case["name"]
        assert depths == case["node_depths"], case["name"]
        assert parents == case["parents"], case["name"]
        assert child_maps == [{int(k): v for k, v in cm.items()} for cm in case["child_maps"]]
        vis = T.visibility_matrix(parents)
        assert vis.astype(np.uint8).tolist() == case["visibility"], case["name"]


def test_full_build_matches_reference(golden):
    """Oracle top-k + log-softmax + heap end to end vs the reference."""
    data, logits = golden
    for case in data["trees"]:
        tokens, depths, parents, child_maps, vis = T.build_dtree_tree(
            logits[case["name"]], case["budget"]
        )
        assert tokens == case["node_token_ids"], case["name"]
        assert parents == case["parents"], case["name"]
        if case["budget"] > 0:
            k = min(case["budget"], logits[case["name"]].shape[1])
            ids, lps = T.topk_log_probs(logits[case["name"]], k)
            ref_ids = np.asarray(case["top_ids"])
            # exactly-equal logits have no specified order in the reference
            # (argpartition + argsort); compare ids only where the value is unique
            row_vals = np.take_along_axis(logits[case["name"]], ref_ids, axis=1)
            for r in range(row_vals.shape[0]):
                vals, counts = np.unique(row_vals[r], return_counts=True)
                unique = set(vals[counts == 1].tolist())
                for j in range(row_vals.shape[1]):
                    if row_vals[r, j] in unique:
                        assert ids[r, j] == ref_ids[r, j], (case["name"], r, j)
            np.testing.assert_allclose(lps, np.asarray(case["top_log_probs"]), rtol=0, atol=2e-6)


def test_tree_invariants(golden):
    data, _ = golden
    for case in data["trees"]:
        parents = case["parents"]
        for i in range(1, len(parents)):
            assert 0 <= parents[i] < i
        anc = T.ancestor_masks(parents)
        vis = T.visibility_matrix(parents)
        for i in range(len(parents)):
            for j in range(len(parents)):
                bit = (int(anc[i, j // 64]) >> (j % 64)) & 1
                assert bit == int(vis[i, j])


def test_walks_match_reference(golden):
    data, _ = golden
    for w in data["walks"]:
        cm = T.child_maps_from(w["parents"], w["tree_tokens"])
        acc, nxt = T.follow_verified_tree(cm, w["posterior"])
        assert acc == w["accepted"] and nxt == w["next_token"]
    acc, nxt = T.follow_verified_tree([{11: 1, 12: 2}, {21: 3}, {}, {}], [11, 21, 99, 0])
    assert acc == data["unit_walk"]["accepted"] == [0, 1, 3]
    assert nxt == data["unit_walk"]["next_token"] == 0


def test_lineages_and_depth_groups(golden):
    data, _ = golden
    for item in data["lineages"]:
        assert T.build_node_lineages(item["parents"]) == item["lineages"]
        assert T.tree_depth_groups(item["parents"]) == item["depth_groups"]
    with pytest.raises(ValueError):
        T.build_node_lineages([-1, 1])
    with pytest.raises(ValueError):
        T.tree_depth_groups([0, 0])


def test_prefix_match(golden):
    data, _ = golden
    for item in data["prefix_match"]:
        assert T.longest_prefix_match(item["draft"], item["verifier"]) == item["matched"]


def test_compaction_matches_reference(golden_dir):
    z = np.load(golden_dir / "compact_golden.npz")
    for c in range(int(z["count"])):
        meta = z[f"c{c}_meta"].tolist()
        past, t, nkeep = meta[:3]
        keep = meta[3:3 + nkeep]
        for li in range(2):
            k = z[f"c{c}_k_in_{li}"].copy()
            v = z[f"c{c}_v_in_{li}"].copy()
            off = T.compact_kv(k, v, past + t, past, keep)
            assert off == int(z[f"c{c}_offset_{li}"])
            np.testing.assert_array_equal(k, z[f"c{c}_k_out_{li}"])
            np.testing.assert_array_equal(v, z[f"c{c}_v_out_{li}"])
