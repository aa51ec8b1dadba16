"""Oracle: the DTree / DFlash decode loops on the CPU oracle model.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Also the timed CPU
baseline of ``bench.py`` (the reference's own MLX path cannot run here).

* ``dtree_step``   one iteration of dtree_generate's loop
                   (dtree_mlx/dtree_runtime.py:364-552): planted draft logits,
                   build_dtree_tree, compile, tree forward, greedy argmax,
                   follow_verified_tree, compact_kv_caches, output commit
* ``dflash_step``  one iteration of dflash_generate with
                   verify_block_parallel_greedy_argmax (dtree_mlx/runtime.py:
                   474-577, :307-362): drafted chain, longest prefix match,
                   KV rewind
"""
from __future__ import annotations

import time

import numpy as np
import torch

from . import planted
from . import tree as T
from .qwen3 import Qwen3Oracle


class OracleDecoder:
    def __init__(self, model: Qwen3Oracle, seed: int, p_correct: float, continuation, block_size: int = 16):
        self.m = model
        self.seed = int(seed)
        self.p = float(p_correct)
        self.cont = np.asarray(continuation if continuation is not None else [], dtype=np.int64)
        self.block_size = int(block_size)
        self.step_idx = 0

    def prefill(self, prompt: list[int]) -> int:
        norm_h, _ = self.m.prefill(prompt)
        self.prefill_logits = self.m.lm_head_logits(norm_h[-1:])[0]
        first = int(self.m.argmax_bf16(self.prefill_logits[None])[0])
        self.output = list(prompt) + [first]
        self.start = len(prompt)
        self.acceptance: list[int] = []
        return first

    def draft_logits(self) -> np.ndarray:
        rows = self.block_size - 1
        return planted.planted_draft_logits(self.seed, self.step_idx, self.start, rows, self.m.cfg.vocab_size,
                                            self.cont, self.p)

    def dtree_step(self, budget: int, draft_logits=None, posterior_override=None):
        """Returns a dict with the tree, posterior and accepted indices."""
        start = self.start
        root = self.output[start]
        dl = self.draft_logits() if draft_logits is None else draft_logits
        tokens, depths, parents, child_maps, vis = T.build_dtree_tree(dl, budget)
        tree_tokens, positions = T.compile_dtree_tree(root, start, tokens, depths)
        mask = T.tree_attention_mask(vis, start)
        norm_h, _ = self.m.forward_tree(tree_tokens, positions, mask, past=start)
        logits = self.m.lm_head_logits(norm_h)
        post = self.m.argmax_bf16(logits).tolist()
        used = post if posterior_override is None else list(posterior_override)
        accepted, nxt = T.follow_verified_tree(child_maps, used)
        self.m.compact(start, accepted)
        self._commit([int(tree_tokens[i]) for i in accepted], nxt)
        return {"tree_tokens": tree_tokens.tolist(), "parents": parents, "posterior": post, "logits": logits,
                "accepted": accepted, "next": nxt}

    def dflash_step(self, draft_logits=None, posterior_override=None):
        start = self.start
        bs = self.block_size
        dl = self.draft_logits() if draft_logits is None else draft_logits
        drafted = [int(np.argmax(row)) for row in dl[: bs - 1]]  # first index on ties
        block = [self.output[start]] + drafted
        mask = np.ones((bs, start + bs), dtype=bool)
        mask[:, start:] = np.tril(np.ones((bs, bs), dtype=bool))
        norm_h, _ = self.m.forward_tree(block, np.arange(start, start + bs), mask, past=start)
        logits = self.m.lm_head_logits(norm_h)
        post = self.m.argmax_bf16(logits).tolist()
        used = post if posterior_override is None else list(posterior_override)
        matched = T.longest_prefix_match(block[1:], used[:-1])
        acc = matched + 1
        if acc < bs:
            self.m.rewind(bs - acc)
        self._commit(block[:acc], used[matched])
        return {"tree_tokens": block, "posterior": post, "logits": logits, "accepted": list(range(acc)),
                "next": used[matched]}

    def _commit(self, accepted_tokens: list[int], nxt: int) -> None:
        self.output = self.output[: self.start] + accepted_tokens + [int(nxt)]
        self.start += len(accepted_tokens)
        self.acceptance.append(len(accepted_tokens))
        self.step_idx += 1

    def generate(self, prompt, max_new_tokens: int, mode: str = "dtree", budget: int = 24):
        """Full loop with the reference's termination rules; returns (tokens, metrics)."""
        total = len(prompt) + int(max_new_tokens)
        t0 = time.perf_counter()
        self.prefill(prompt)
        t1 = time.perf_counter()
        while self.start < total:
            if mode == "dtree":
                self.dtree_step(budget)
            else:
                self.dflash_step()
            if len(self.output) > total:
                break
        t2 = time.perf_counter()
        out = self.output[:total]
        return out, {"acceptance_lengths": list(self.acceptance), "prefill_time_s": t1 - t0,
                     "decode_time_s": t2 - t1, "num_output_tokens": len(out) - len(prompt)}


def near_tie(logits_row: torch.Tensor, a: int, b: int, tol: float) -> bool:
    """True if tokens a and b are within `tol` of each other and of the max."""
    mx = float(logits_row.max())
    return abs(float(logits_row[a]) - mx) <= tol and abs(float(logits_row[b]) - mx) <= tol
