"""The reference's runtime tests (tests/test_dtree_runtime.py) against this
package's functions of the same names.

* lazy_follow_tree_exact walks only the taken branch (the fake-model test of
  test_dtree_runtime.py:67-106: a fake text model whose norm hidden is the
  input token and a fake LM head mapping 10 -> 100, 11 -> 300, 21 -> 999);
  host logic, runs on the CPU;
* build_dtree_tree returns prefix-closed visibility (:15-44) and
  follow_verified_tree walks matching children (:47-56), on the GPU.
"""
from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch


def test_lazy_follow_tree_exact_walks_only_the_taken_branch():
    from dtree_mlx_b200.dtree_runtime import lazy_follow_tree_exact

    class FakeTextModel:
        def forward_dflash(self, inputs, cache, layer_ids):
            del cache, layer_ids
            token = int(inputs[0, 0].item())
            return torch.tensor([[[token]]], dtype=torch.float32), torch.tensor([[[token + 1000]]], dtype=torch.float32)

    class FakeTarget:
        def __init__(self):
            self.adapter = SimpleNamespace(family="qwen3_5")
            self.model = SimpleNamespace(language_model=SimpleNamespace(model=FakeTextModel()))

        def lm_head_argmax(self, hidden_states):
            token = int(hidden_states[0, 0, 0].item())
            return torch.tensor([[{10: 100, 11: 300, 21: 999}[token]]], dtype=torch.int32)

    child_maps = [{100: 1, 200: 2}, {300: 3}, {}, {}]
    accepted, next_token, verifier_hidden = lazy_follow_tree_exact(
        target=FakeTarget(), target_cache=[], layer_ids=[], tree_tokens=[10, 11, 12, 21], child_maps=child_maps,
        temperature=0.0, verify_mode="parallel-greedy-argmax", profile_times=None)
    assert accepted == [0, 1, 3]
    assert next_token == 999
    assert verifier_hidden.tolist() == [[[1010.0], [1011.0], [1021.0]]]


def test_lazy_follow_rejects_other_families():
    from dtree_mlx_b200.dtree_runtime import lazy_follow_tree_exact

    with pytest.raises(NotImplementedError):
        lazy_follow_tree_exact(SimpleNamespace(adapter=SimpleNamespace(family="qwen3")), [], [], [1], [{}], 0.0,
                               "parallel-greedy-argmax", None)


@pytest.mark.gpu
def test_build_dtree_tree_returns_prefix_closed_visibility(lib):
    from dtree_mlx_b200.dtree_runtime import build_dtree_tree

    draft_logits = torch.tensor([[5.0, 4.0, 1.0], [6.0, 2.0, 1.0], [7.0, 3.0, 1.0]], device="cuda")
    node_token_ids, node_depths, parents, child_maps, visibility, _ = build_dtree_tree(draft_logits=draft_logits,
                                                                                      budget=4)
    assert node_token_ids
    assert len(node_token_ids) == len(node_depths)
    assert parents[0] == -1
    assert visibility.shape[0] == 1 + len(node_token_ids)
    assert bool(visibility[0, 0].item()) is True
    for node_index in range(1, len(parents)):
        parent_index = parents[node_index]
        assert parent_index < node_index
        assert child_maps[parent_index][node_token_ids[node_index - 1]] == node_index
        assert bool(visibility[node_index, parent_index].item()) is True
        assert bool(visibility[node_index, node_index].item()) is True


@pytest.mark.gpu
def test_follow_verified_tree_walks_matching_children(lib):
    from dtree_mlx_b200.dtree_runtime import follow_verified_tree

    child_maps = [{11: 1, 12: 2}, {21: 3}, {}, {}]
    accepted, next_token = follow_verified_tree(child_maps, [11, 21, 99, 0])
    assert accepted == [0, 1, 3]
    assert next_token == 0
