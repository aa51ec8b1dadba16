"""DTree: best-first tree verification (dtree_mlx/dtree_runtime.py).

``build_dtree_tree``, ``compile_dtree_tree`` and ``follow_verified_tree``
keep the reference's signatures and return values but run on the GPU
(``dtree_tree_build`` / ``dtree_accept_walk``); ``dtree_generate`` is the
device-resident decode loop (see runtime.run_decode), or for a Qwen3.5
target the lazy branch-following loop (``lazy_follow_tree_exact``,
runtime.run_decode_lazy) unless ``DTREE_QWEN35_TREE_MODE=full_tree``, as in
dtree_runtime.py:355-361.
"""
from __future__ import annotations

import os
import time

import numpy as np
import torch

from . import kernels
from .runtime import DTREE_STAGE_ORDER, run_decode  # noqa: F401

DTREE_TREE_BUILD_STAGE_ORDER = (
    "tree_build_copy_time_s",
    "tree_build_heap_time_s",
    "tree_build_visibility_time_s",
)


def _anc_to_visibility(anc: np.ndarray, n: int) -> np.ndarray:
    bits = anc.view(np.uint64)
    vis = np.zeros((n, n), dtype=np.bool_)
    for i in range(n):
        for j in range(n):
            vis[i, j] = bool((int(bits[i, j // 64]) >> (j % 64)) & 1)
    return vis


def build_dtree_tree(draft_logits: torch.Tensor, budget: int):
    """dtree_runtime.py:82-163 on the GPU.  ``draft_logits`` [rows, vocab] is a
    CUDA tensor.  Returns ``(node_token_ids, node_depths, parents, child_maps,
    visibility, subtimes)`` exactly as the reference (visibility as a bool
    CPU tensor)."""
    subtimes = {name: 0.0 for name in DTREE_TREE_BUILD_STAGE_ORDER}
    if budget <= 0 or draft_logits.shape[0] == 0:
        return [], [], [-1], [dict()], torch.ones(1, 1, dtype=torch.bool), subtimes
    logits = draft_logits.float().contiguous()
    rows, vocab = logits.shape
    t0 = time.perf_counter()
    state = kernels.new_state(logits.device)
    out = kernels.TreeBuffers.allocate(logits.device)
    kernels.TreeBuilder(rows, vocab, budget, logits.device).build(logits, state, out, keep_topk=False)
    n = int(state[6].item())
    subtimes["tree_build_heap_time_s"] = time.perf_counter() - t0
    tokens = out.tokens[:n].tolist()
    depths = out.depths[:n].tolist()
    parents = out.parents[:n].tolist()
    child_maps: list[dict[int, int]] = [dict() for _ in range(n)]
    for i in range(1, n):
        child_maps[parents[i]][tokens[i]] = i
    vis = _anc_to_visibility(out.anc[:n].cpu().numpy(), n)
    return tokens[1:], depths[1:], parents, child_maps, torch.from_numpy(vis), subtimes


def compile_dtree_tree(root_token_id: int, start: int, node_token_ids, node_depths, visibility, past_length: int,
                       verify_input_ids_buffer: torch.Tensor, verify_position_ids_buffer: torch.Tensor,
                       attention_mask_buffer: torch.Tensor):
    """dtree_runtime.py:166-192: fills the reusable id / position / mask buffers."""
    tree_tokens = [root_token_id, *node_token_ids]
    positions = [start, *[start + d for d in node_depths]]
    n = len(tree_tokens)
    ids = verify_input_ids_buffer[:, :n]
    pos = verify_position_ids_buffer[:, :n]
    ids[0, :n] = torch.tensor(tree_tokens, dtype=ids.dtype)
    pos[0, :n] = torch.tensor(positions, dtype=pos.dtype)
    mask = attention_mask_buffer[:n, : past_length + n]
    mask[:, past_length : past_length + n] = torch.as_tensor(visibility, dtype=torch.bool).to(mask.device)
    return ids, tree_tokens, pos, mask


def follow_verified_tree(child_maps: list[dict[int, int]], posterior_tokens: list[int]) -> tuple[list[int], int]:
    """dtree_runtime.py:195-208, evaluated by the device walk kernel."""
    n = len(child_maps)
    parents = [-1] * n
    tokens = [0] * n
    for p, cm in enumerate(child_maps):
        for tok, c in cm.items():
            parents[c] = p
            tokens[c] = int(tok)
    dev = torch.device("cuda")
    tree = kernels.TreeBuffers.allocate(dev, cap=max(n, 1))
    tree.tokens[:n] = torch.tensor(tokens, dtype=torch.int32)
    tree.parents[:n] = torch.tensor(parents, dtype=torch.int32)
    state = kernels.new_state(dev)
    state[6] = n
    post = torch.tensor([int(t) for t in posterior_tokens[:n]] + [0] * (n - len(posterior_tokens[:n])),
                        dtype=torch.int32, device=dev)
    acc = torch.zeros(max(n, 1), dtype=torch.int32, device=dev)
    out = torch.zeros(n + 2, dtype=torch.int32, device=dev)
    kernels.accept_walk(tree, post, state, acc, out, None)
    st = kernels.state_dict(state)
    return acc[: st["n_accepted"]].tolist(), st["bonus_token"]


def _text_model(target):
    model = target.model
    if hasattr(model, "language_model") and hasattr(model.language_model, "model"):
        return model.language_model.model
    if hasattr(model, "model"):
        return model.model
    raise AttributeError(f"Unsupported qwen3_5 target model: {type(model)!r}")


def lazy_follow_tree_exact(target, target_cache, layer_ids, tree_tokens: list[int],
                           child_maps: list[dict[int, int]], temperature: float, verify_mode: str,
                           profile_times: dict[str, float] | None):
    """dtree_runtime.py:211-290: verify only the branch the target follows.
    Starting at the root, each step runs ONE token through the target as a
    plain causal decode (its K/V appended, the DeltaNet states advanced), takes
    the posterior token (argmax for parallel-greedy-argmax, else
    sample_tokens at ``temperature``) and moves to the child with that token;
    it stops at the first posterior that is not a child.  The cache then
    holds exactly the accepted path, so nothing is compacted or rolled back.
    Returns (accepted node indices, posterior token, verifier hiddens of the
    accepted nodes concatenated along axis 1)."""
    from .runtime import sample_tokens

    if target.adapter.family != "qwen3_5":
        raise NotImplementedError("lazy_follow_tree_exact is only implemented for qwen3_5.")
    text_model = _text_model(target)
    accepted: list[int] = []
    hidden_chunks = []
    current = 0
    while True:
        t0 = time.perf_counter()
        ids = torch.tensor([[int(tree_tokens[current])]], dtype=torch.int32)
        norm_hidden, verifier_hidden = text_model.forward_dflash(ids, target_cache, layer_ids)
        if profile_times is not None:
            profile_times["verify_tree_forward_time_s"] = profile_times.get("verify_tree_forward_time_s", 0.0) + (
                time.perf_counter() - t0)
        accepted.append(current)
        hidden_chunks.append(verifier_hidden)
        if verify_mode == "parallel-greedy-argmax":
            posterior = target.lm_head_argmax(norm_hidden)
        else:
            posterior = sample_tokens(target.lm_head_logits(norm_hidden), temperature)
        token = int(torch.as_tensor(posterior).reshape(-1)[0].item())
        nxt = child_maps[current].get(token)
        if nxt is None:
            return accepted, token, torch.cat([torch.as_tensor(h) for h in hidden_chunks], dim=1)
        current = nxt


def dtree_generate(target, draft, prompt_tokens, max_new_tokens: int, temperature: float, stop_token_ids,
                   layer_ids, speculative_tokens: int | None, tree_budget: int | None = None,
                   verify_mode: str = "parallel-replay", profile: bool = False):
    """dtree_runtime.py:293-586.  ``parallel-replay`` at temperature >= 1e-5
    samples every node's posterior token (dtree_runtime.py:455-470) on the
    device; the tree itself does not depend on the temperature."""
    del layer_ids
    if not target.supports_tree_verification():
        raise NotImplementedError(f"DTree is not implemented for target adapter family={target.adapter.family!r}.")
    if verify_mode not in {"parallel-replay", "parallel-greedy-argmax"}:
        raise ValueError("DTree only supports verify_mode='parallel-replay' or 'parallel-greedy-argmax'.")
    if verify_mode == "parallel-greedy-argmax" and temperature >= 1e-5:
        raise ValueError("DTree parallel-greedy-argmax only supports temperature=0.")
    if speculative_tokens is None:
        block_size = draft.block_size
    else:
        block_size = max(1, min(speculative_tokens, draft.block_size))
    if block_size <= 1:
        raise ValueError("DTree requires speculative_tokens >= 2.")
    budget = max(tree_budget if tree_budget is not None else block_size - 1, 0)
    if budget > 127:
        raise ValueError("tree_budget must be <= 127 (128 tree rows per verify)")
    if target.adapter.family == "qwen3_5" and os.environ.get("DTREE_QWEN35_TREE_MODE") != "full_tree":
        # the reference's default for the hybrid (dtree_runtime.py:355-361):
        # follow only the taken branch, one token per target forward
        from .runtime import run_decode_lazy

        out, metrics = run_decode_lazy(target, draft, prompt_tokens, max_new_tokens, set(stop_token_ids or ()),
                                       block_size, budget, temperature, verify_mode, profile=profile)
    else:
        out, metrics = run_decode(target, draft, prompt_tokens, max_new_tokens, set(stop_token_ids or ()), "dtree",
                                  block_size, budget, profile=profile, temperature=temperature)
    metrics["verify_mode"] = verify_mode
    return out, metrics
