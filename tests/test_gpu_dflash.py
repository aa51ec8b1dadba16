"""DFlash block drafter forward on the GPU vs the fp32 oracle (tiny target
and drafter): the draft logits after the prompt context and after decode
steps whose accepted rows became context.

Tolerance (bf16 drafter vs fp32 oracle on the same bf16 weights and the same
bf16 target hiddens): draft logits max |d| <= 3e-2, mean <= 5e-3; the top-1
token of every draft row must agree except at near-ties.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.dflash import DFlashOracle
from oracle.runtime import near_tie

pytestmark = pytest.mark.gpu
DEV = "cuda"
MAX_TOL, MEAN_TOL = 3e-2, 5e-3


def _check(g, o, tag):
    err = (g - o).abs()
    print(f"{tag}: draft logits max {err.max():.3e} mean {err.mean():.3e}")
    assert err.max() <= MAX_TOL and err.mean() <= MEAN_TOL, tag
    for r in range(g.shape[0]):
        a, b = int(torch.argmax(g[r])), int(torch.argmax(o[r]))
        if a != b:
            assert near_tie(o[r], a, b, MAX_TOL), (tag, r)


def test_dflash_drafter_matches_oracle(lib):
    from dtree_mlx_b200.adapters import load_target_model
    from dtree_mlx_b200.draft import load_draft_model
    from dtree_mlx_b200.engine import DecodeSession, StepConfig, dtree_nodes
    from dtree_mlx_b200.synthetic import random_prompt

    target = load_target_model("synthetic:qwen3-tiny:seed=0:kv=1024")
    drafter, _ = load_draft_model("dflash:qwen3-tiny:seed=3", target=target)
    cfg = drafter.cfg
    eng = target.adapter.engine(target.model, drafter)
    assert eng.layer_ids == list(cfg.target_layer_ids)
    n_nodes = dtree_nodes(24, 15, cfg.vocab_size)
    sess = DecodeSession(eng, StepConfig("dtree", 15, 24, n_nodes), output_capacity=512, drafter=drafter)
    prompt = random_prompt(40, cfg.vocab_size, seed=5)
    first = sess.prefill(prompt)  # also ingests the prompt context into the draft cache
    orc = DFlashOracle(drafter.weights, target.model.weights.embed)
    orc.context(sess.prompt_hidden.float().cpu())
    for step in range(3):
        st = sess.read_state()
        sess.step()
        torch.cuda.synchronize()
        g = drafter.logits[1:16].float().cpu()
        o = orc.block_logits(st["root_token"])[1:16]
        _check(g, o, f"step {step}")
        new = sess.read_state()
        n = new["n_accepted"]
        orc.context(sess.target_hidden[:n].float().cpu())  # the rows this step accepted
        assert orc.offset == new["start"]
    from dtree_mlx_b200 import _lib

    assert _lib.device_error() == 0
    del first


def test_dtree_generation_with_dflash_drafter(lib):
    """DTree through the public API with the model drafter; random-init
    drafter weights draft poorly, but decoding stays exact: the output equals
    DFlash-mode greedy decoding with the planted drafter (near-ties aside)."""
    from dtree_mlx_b200 import DFlashGenerator
    from dtree_mlx_b200.synthetic import random_prompt

    gen = DFlashGenerator(target_model="synthetic:qwen3-tiny:seed=0:kv=1024", draft_model="dflash:qwen3-tiny:seed=3")
    prompt = random_prompt(64, 32768, seed=1)
    r = gen.generate_from_tokens(prompt, max_new_tokens=32, decode_mode="dtree", speculative_tokens=16,
                                 tree_budget=24)
    ref = DFlashGenerator(target_model="synthetic:qwen3-tiny:seed=0:kv=1024", draft_model="planted:p=0.8:seed=1")
    r2 = ref.generate_from_tokens(prompt, max_new_tokens=32, decode_mode="dflash", speculative_tokens=16,
                                  verify_mode="parallel-greedy-argmax")
    first_diff = next((i for i, (a, b) in enumerate(zip(r.generated_tokens, r2.generated_tokens)) if a != b), 32)
    print(f"dflash-drafter DTree vs planted DFlash: first difference {first_diff}/32, "
          f"accept {r.metrics['avg_acceptance_length']:.2f}")
    assert len(r.generated_tokens) == 32 and first_diff >= 8


def test_context_only_draft_cache_matches_windowed_oracle(lib):
    """ContextOnlyDraftKVCache (draft.py:69-112): with a small sink and window
    the device ring must attend over exactly the reference's sink + last
    window rows (at their real positions) once the context overflows."""
    from dtree_mlx_b200.adapters import load_target_model
    from dtree_mlx_b200.draft import load_draft_model
    from dtree_mlx_b200.engine import DecodeSession, StepConfig, dtree_nodes
    from dtree_mlx_b200.synthetic import random_prompt

    target = load_target_model("synthetic:qwen3-tiny:seed=0:kv=1024")
    drafter, _ = load_draft_model("dflash:qwen3-tiny:seed=3", target=target)
    drafter.cache_mode, drafter.sink_size, drafter.window_size = "context-only", 8, 40
    cfg = drafter.cfg
    eng = target.adapter.engine(target.model, drafter)
    sess = DecodeSession(eng, StepConfig("dtree", 15, 24, dtree_nodes(24, 15, cfg.vocab_size)), output_capacity=512,
                         drafter=drafter)
    sess.prefill(random_prompt(44, cfg.vocab_size, seed=6))  # 44 > 8 + 40 - ... overflows within a few steps
    orc = DFlashOracle(drafter.weights, target.model.weights.embed, sink=8, window=40)
    orc.context(sess.prompt_hidden.float().cpu())
    for step in range(6):
        st = sess.read_state()
        sess.step()
        torch.cuda.synchronize()
        g = drafter.logits[1:16].float().cpu()
        o = orc.block_logits(st["root_token"])[1:16]
        _check(g, o, f"ring step {step}")
        new = sess.read_state()
        orc.context(sess.target_hidden[: new["n_accepted"]].float().cpu())
        # the device appends a step's accepted rows at the start of the next draft
        ring = drafter.ring_state.tolist()
        pending = new["n_accepted"]
        assert ring[7] == orc.appended - pending == new["start"] - pending
        assert ring[0] == min(orc.appended - pending, 48)
    from dtree_mlx_b200 import _lib

    assert _lib.device_error() == 0
