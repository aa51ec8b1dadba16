"""Temperature > 0: sampled posterior and drafted tokens (sample_tokens,
runtime.py:12-19: categorical over logits / T) on the device.

The samplers draw by the Gumbel-max rule with Philox noise keyed by (seed,
step, row, token).  MLX's own random stream cannot be reproduced, so the
checks are distributional: empirical token frequencies over many draws
against softmax(bf16 logits / T) (chi-square, p > 1e-4), temperature -> 0
equal to the argmax, fixed seeds reproducible, and end-to-end sampled
generations that are valid and seed-deterministic.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _chi2_pvalue(counts: np.ndarray, probs: np.ndarray) -> float:
    from scipy.stats import chisquare

    probs = np.asarray(probs, dtype=np.float64)
    probs = probs / probs.sum()
    counts = np.asarray(counts, dtype=np.float64)
    n = counts.sum()
    keep = probs * n >= 5  # pool the rare tokens
    obs = np.append(counts[keep], counts[~keep].sum())
    exp = np.append(probs[keep] * n, probs[~keep].sum() * n)
    if exp[-1] == 0:
        obs, exp = obs[:-1], exp[:-1]
    return float(chisquare(obs, exp).pvalue)


@pytest.mark.parametrize("temperature", [0.7, 1.0, 1.6])
def test_lm_head_sample_matches_softmax(lib, temperature):
    from dtree_mlx_b200 import kernels

    g = torch.Generator().manual_seed(11)
    hidden, vocab, rows = 64, 12, 16
    embed = (torch.randn(vocab, hidden, generator=g) * 0.35).to(torch.bfloat16).to(DEV)
    h = torch.zeros(rows, hidden, dtype=torch.bfloat16, device=DEV)
    h[:] = torch.randn(hidden, generator=g).to(torch.bfloat16).to(DEV)  # every row: the same logits
    logits = (h[0].float() @ embed.float().t()).to(torch.bfloat16).float().cpu().numpy()
    probs = np.exp((logits - logits.max()) / temperature)
    probs /= probs.sum()
    state = kernels.new_state(DEV)
    out = torch.zeros(rows, dtype=torch.int32, device=DEV)
    draws = []
    for step in range(600):
        state[2] = step
        kernels.lm_head_sample(h, embed, rows, temperature, seed=1234, state=state, out=out)
        draws.append(out.clone())
    samples = torch.cat(draws).cpu().numpy()
    counts = np.bincount(samples, minlength=vocab)
    pv = _chi2_pvalue(counts, probs)
    print(f"T={temperature}: {len(samples)} draws, chi-square p = {pv:.3g}")
    assert pv > 1e-4
    # temperature below 1e-5 is the greedy argmax; a fixed (seed, step) repeats
    kernels.lm_head_sample(h, embed, rows, 0.0, seed=1, state=state, out=out)
    assert set(out.tolist()) == {int(np.argmax(logits))}
    state[2] = 3
    a = kernels.lm_head_sample(h, embed, rows, temperature, seed=9, state=state).clone()
    b = kernels.lm_head_sample(h, embed, rows, temperature, seed=9, state=state).clone()
    assert torch.equal(a, b)


def test_chain_sample_matches_softmax(lib):
    from dtree_mlx_b200 import kernels

    g = torch.Generator().manual_seed(3)
    rows, vocab, temperature = 15, 40, 0.9
    base = torch.randn(vocab, generator=g) * 1.5
    logits = base.repeat(rows, 1).contiguous().to(DEV)
    probs = torch.softmax(base / temperature, dim=0).numpy()
    state = kernels.new_state(DEV, start=10, root_token=7)
    tree = kernels.TreeBuffers.allocate(DEV)
    draws = []
    for step in range(400):
        state[2] = step
        kernels.chain_build(logits, state, tree, temperature=temperature, seed=77)
        draws.append(tree.tokens[1:rows + 1].clone())
    samples = torch.cat(draws).cpu().numpy()
    pv = _chi2_pvalue(np.bincount(samples, minlength=vocab), probs)
    print(f"chain sample: {len(samples)} draws, chi-square p = {pv:.3g}")
    assert pv > 1e-4
    assert tree.parents[: rows + 1].tolist() == list(range(-1, rows))
    kernels.chain_build(logits, state, tree, temperature=0.0)
    assert set(tree.tokens[1:rows + 1].tolist()) == {int(torch.argmax(base))}


@pytest.mark.parametrize("mode", ["dtree", "dflash"])
def test_sampled_generation_is_valid_and_seeded(lib, mode):
    from dtree_mlx_b200 import DFlashGenerator
    from dtree_mlx_b200.synthetic import random_prompt

    prompt = random_prompt(64, 32768, seed=2)
    outs = []
    for _ in range(2):
        gen = DFlashGenerator(target_model="synthetic:qwen3-tiny:seed=0:kv=1024",
                              draft_model="planted:p=0.8:seed=1", seed=5)
        kw = dict(max_new_tokens=48, decode_mode=mode, speculative_tokens=16, temperature=0.8)
        if mode == "dtree":
            kw["tree_budget"] = 24
        else:
            kw["verify_mode"] = "parallel-replay"
        r = gen.generate_from_tokens(prompt, **kw)
        assert len(r.output_tokens) == 64 + 48 and r.output_tokens[:64] == prompt
        assert all(0 <= t < 32768 for t in r.generated_tokens)
        assert min(r.metrics["acceptance_lengths"]) >= 1
        outs.append(r.generated_tokens)
    assert outs[0] == outs[1]  # the generator seed fixes the sampling noise
    greedy = DFlashGenerator(target_model="synthetic:qwen3-tiny:seed=0:kv=1024",
                             draft_model="planted:p=0.8:seed=1").generate_from_tokens(
        prompt, max_new_tokens=48, decode_mode=mode, speculative_tokens=16)
    print(f"{mode}: sampled vs greedy agreement "
          f"{sum(a == b for a, b in zip(outs[0], greedy.generated_tokens))}/48")
    with pytest.raises(ValueError):
        gen.generate_from_tokens(prompt, max_new_tokens=8, decode_mode=mode, speculative_tokens=16,
                                 temperature=0.8, verify_mode="parallel-greedy-argmax")
