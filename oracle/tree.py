"""Oracle: DTree tree construction, compilation, acceptance walk, lineages.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates, in NumPy + ``heapq``, the reference functions

* ``build_dtree_tree``      dtree_mlx/dtree_runtime.py:82-163
* ``compile_dtree_tree``    dtree_mlx/dtree_runtime.py:166-192
* ``follow_verified_tree``  dtree_mlx/dtree_runtime.py:195-208
* ``build_node_lineages``   dtree_mlx/qwen35_tree.py:41-55
* ``_tree_depth_groups``    dtree_mlx/qwen35_tree.py:104-123
* ``longest_prefix_match``  dtree_mlx/runtime.py:33-39
* ``stop_position``         dtree_mlx/runtime.py:42-46

The heap key, the sibling-score formula ``logw - lp[r] + lp[r+1]`` and the
float64 accumulation order are kept exactly as in the reference
(dtree_runtime.py:111-147) because the tree topology must be bit-exact.

Top-k tie rule: the reference takes ``mx.argpartition`` then a descending
``mx.argsort`` of the selected logits (dtree_runtime.py:97-103); the order of
exactly-equal logits is not specified there.  This oracle (and the CUDA
kernel) orders equal logits by ascending token id.
"""
from __future__ import annotations

import heapq

import numpy as np


def topk_log_probs(draft_logits: np.ndarray, topk: int) -> tuple[np.ndarray, np.ndarray]:
    """Per-row top-k token ids (descending logit) and fp32 log-probs.

    dtree_runtime.py:92-107: logits cast to fp32, top-k by argpartition +
    argsort, ``top_logits - logsumexp(logits)`` in fp32.  The logsumexp here is
    evaluated in float64 and rounded once to fp32 (the exact fp32 value up to
    that rounding); a GPU fp32 reduction agrees to within a few ulp.
    """
    logits = np.asarray(draft_logits, dtype=np.float32)
    rows, vocab = logits.shape
    topk = min(int(topk), vocab)
    ids = np.empty((rows, topk), dtype=np.int64)
    lps = np.empty((rows, topk), dtype=np.float32)
    for r in range(rows):
        row = logits[r]
        # descending by value, ascending token id on equal values
        order = np.lexsort((np.arange(vocab), -row.astype(np.float64)))[:topk]
        m = float(np.max(row.astype(np.float64)))
        lse = m + np.log(np.sum(np.exp(row.astype(np.float64) - m)))
        lse32 = np.float32(lse)
        ids[r] = order
        lps[r] = (row[order] - lse32).astype(np.float32)
    return ids, lps


def heap_build(
    top_token_ids: np.ndarray,
    top_log_probs: np.ndarray,
    budget: int,
) -> tuple[list[int], list[int], list[int], list[dict[int, int]]]:
    """Best-first expansion; dtree_runtime.py:110-148, same key and order.

    Returns ``(node_token_ids, node_depths, parents, child_maps)`` where
    ``parents``/``child_maps`` include the root at index 0.
    """
    top_token_ids = np.asarray(top_token_ids)
    top_log_probs = np.asarray(top_log_probs, dtype=np.float32)
    if budget <= 0 or top_token_ids.shape[0] == 0:
        return [], [], [-1], [dict()]
    topk = int(top_token_ids.shape[1])
    depth_limit = int(top_token_ids.shape[0])

    first_logw = float(top_log_probs[0, 0])
    heap: list[tuple[float, tuple[int, ...], int, int, int, float]] = [
        (-first_logw, (0,), 0, 1, 0, first_logw)
    ]
    node_token_ids: list[int] = []
    node_depths: list[int] = []
    parents = [-1]
    child_maps: list[dict[int, int]] = [dict()]
    while heap and len(node_token_ids) < budget:
        _, ranks, parent_index, depth, rank, logw = heapq.heappop(heap)
        token_id = int(top_token_ids[depth - 1, rank])
        current_index = len(node_token_ids) + 1
        node_token_ids.append(token_id)
        node_depths.append(depth)
        parents.append(parent_index)
        child_maps.append(dict())
        child_maps[parent_index][token_id] = current_index
        if rank + 1 < topk:
            sibling_ranks = ranks[:-1] + (rank + 1,)
            sibling_logw = logw - float(top_log_probs[depth - 1, rank]) + float(
                top_log_probs[depth - 1, rank + 1]
            )
            heapq.heappush(
                heap, (-sibling_logw, sibling_ranks, parent_index, depth, rank + 1, sibling_logw)
            )
        if depth < depth_limit:
            child_ranks = ranks + (0,)
            child_logw = logw + float(top_log_probs[depth, 0])
            heapq.heappush(
                heap, (-child_logw, child_ranks, current_index, depth + 1, 0, child_logw)
            )
    return node_token_ids, node_depths, parents, child_maps


def visibility_matrix(parents: list[int]) -> np.ndarray:
    """Prefix-closed visibility; dtree_runtime.py:152-160."""
    n = len(parents)
    vis = np.zeros((n, n), dtype=np.bool_)
    vis[0, 0] = True
    for index in range(1, n):
        p = parents[index]
        vis[index, :index] = vis[p, :index]
        vis[index, index] = True
    return vis


def build_dtree_tree(draft_logits: np.ndarray, budget: int):
    """Full restatement of dtree_runtime.py:82-163 (minus the profile timers).

    Returns ``(node_token_ids, node_depths, parents, child_maps, visibility)``.
    """
    draft_logits = np.asarray(draft_logits)
    if budget <= 0 or draft_logits.shape[0] == 0:
        return [], [], [-1], [dict()], np.ones((1, 1), dtype=np.bool_)
    topk = min(budget, int(draft_logits.shape[-1]))
    ids, lps = topk_log_probs(draft_logits, topk)
    tokens, depths, parents, child_maps = heap_build(ids, lps, budget)
    return tokens, depths, parents, child_maps, visibility_matrix(parents)


def ancestor_masks(parents: list[int], words: int = 2) -> np.ndarray:
    """Bit j of row i is set iff node j is visible to node i (row of the
    visibility matrix packed little-endian into ``words`` uint64)."""
    vis = visibility_matrix(parents)
    n = len(parents)
    out = np.zeros((n, words), dtype=np.uint64)
    for i in range(n):
        for j in range(n):
            if vis[i, j]:
                out[i, j // 64] |= np.uint64(1) << np.uint64(j % 64)
    return out


def compile_dtree_tree(root_token_id: int, start: int, node_token_ids, node_depths):
    """dtree_runtime.py:166-192: verify ids and RoPE positions (uint32)."""
    tree_tokens = [int(root_token_id), *[int(t) for t in node_token_ids]]
    positions = [int(start), *[int(start) + int(d) for d in node_depths]]
    return (
        np.asarray(tree_tokens, dtype=np.uint32),
        np.asarray(positions, dtype=np.uint32),
    )


def tree_attention_mask(visibility: np.ndarray, past_length: int) -> np.ndarray:
    """mask[:, :P] all True, mask[:, P:P+T] = visibility (dtree_runtime.py:190-191)."""
    t = visibility.shape[0]
    mask = np.ones((t, past_length + t), dtype=np.bool_)
    mask[:, past_length:] = visibility
    return mask


def follow_verified_tree(child_maps, posterior_tokens):
    """dtree_runtime.py:195-208."""
    accepted_indices = [0]
    current_index = 0
    next_token = int(posterior_tokens[current_index])
    while next_token in child_maps[current_index]:
        current_index = child_maps[current_index][next_token]
        accepted_indices.append(current_index)
        next_token = int(posterior_tokens[current_index])
    return accepted_indices, next_token


def child_maps_from(parents: list[int], tree_tokens: list[int]) -> list[dict[int, int]]:
    """Rebuild the reference's child maps from parents + tokens (root at 0)."""
    maps: list[dict[int, int]] = [dict() for _ in parents]
    for i in range(1, len(parents)):
        maps[parents[i]][int(tree_tokens[i])] = i
    return maps


def build_node_lineages(parents: list[int]) -> list[list[int]]:
    """qwen35_tree.py:41-55."""
    if not parents:
        return []
    if parents[0] != -1:
        raise ValueError(f"tree root parent must be -1, got {parents[0]}")
    lineages: list[list[int]] = [[]]
    for node_index in range(1, len(parents)):
        parent_index = int(parents[node_index])
        if parent_index < 0 or parent_index >= node_index:
            raise ValueError(
                f"tree parent index must precede child, got parents[{node_index}]={parent_index}"
            )
        lineages.append([*lineages[parent_index], parent_index])
    return lineages


def tree_depth_groups(parents: list[int]) -> list[list[int]]:
    """qwen35_tree.py:104-123."""
    if not parents:
        return []
    if parents[0] != -1:
        raise ValueError(f"tree root parent must be -1, got {parents[0]}")
    depths = [0] * len(parents)
    groups: list[list[int]] = [[0]]
    for node_index in range(1, len(parents)):
        parent_index = int(parents[node_index])
        if parent_index < 0 or parent_index >= node_index:
            raise ValueError(
                f"tree parent index must precede child, got parents[{node_index}]={parent_index}"
            )
        depth = depths[parent_index] + 1
        depths[node_index] = depth
        while len(groups) <= depth:
            groups.append([])
        groups[depth].append(node_index)
    return groups


def longest_prefix_match(draft_tokens, verifier_tokens) -> int:
    """runtime.py:33-39."""
    matched = 0
    for d, v in zip(draft_tokens, verifier_tokens):
        if d != v:
            break
        matched += 1
    return matched


def stop_position(tokens, start_idx: int, stop_token_ids) -> int | None:
    """runtime.py:42-46."""
    for idx in range(start_idx, len(tokens)):
        if tokens[idx] in stop_token_ids:
            return idx
    return None


def compact_kv(keys: np.ndarray, values: np.ndarray, offset: int, past_length: int,
               keep_current_indices: list[int]) -> int:
    """In-place restatement of Qwen3TargetAdapter.compact_kv_caches for one
    layer (adapters.py:635-668).  ``keys``/``values`` are [..., cap, d]
    arrays; returns the new offset."""
    keep_count = len(keep_current_indices)
    current_length = offset - past_length
    if current_length <= 0:
        return offset
    if keep_count == 0:
        return past_length
    if keep_count == current_length:
        return offset
    idx = np.asarray(keep_current_indices, dtype=np.int64)
    kept_k = keys[..., past_length:offset, :][..., idx, :].copy()
    kept_v = values[..., past_length:offset, :][..., idx, :].copy()
    keys[..., past_length:past_length + keep_count, :] = kept_k
    values[..., past_length:past_length + keep_count, :] = kept_v
    return past_length + keep_count
