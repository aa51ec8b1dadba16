"""Tree-verify forward and decode steps on the GPU vs the fp32 CPU oracle.

Tolerances (bf16 engine vs fp32 oracle on the same bf16 weights):
  logits        max |gpu - oracle| <= 3e-2 and mean |gpu - oracle| <= 5e-3
                (tiny config, 4 layers, 25 x 32768 logits)
  hidden states relative Frobenius error <= 2e-2
Tree topology, acceptance indices and compaction indices are compared
bit-exactly given the same draft logits and posterior tokens; posterior
tokens must equal the oracle's bf16 argmax except at near-ties (top-2 logits
within 3e-2), which are counted and reported.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import tree as OT
from oracle.qwen3 import Qwen3Oracle
from oracle.runtime import OracleDecoder, near_tie

pytestmark = pytest.mark.gpu
DEV = "cuda"
LOGIT_TOL = 3e-2
LOGIT_MEAN_TOL = 5e-3
REL_TOL = 2e-2


@pytest.fixture(scope="module", params=["bf16", "q4", "q4_embed"])
def tiny(lib, request):
    """Tiny Qwen3 target, bf16 or with MLX affine 4-bit projections (the
    oracle dequantizes the packed weights itself); q4_embed also quantizes
    the embedding, so the tied LM head runs the 4-bit GEMM."""
    from dtree_mlx_b200.config import PRESETS
    from dtree_mlx_b200.synthetic import quantize_weights, random_qwen3_weights

    cfg = PRESETS["qwen3-tiny"]
    w = random_qwen3_weights(cfg, seed=0, device=DEV, norm_jitter=0.1)
    if request.param != "bf16":
        w = quantize_weights(w, embedding=request.param == "q4_embed")
    return cfg, w


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / max(b.norm(), 1e-12))


def test_prefill_and_tree_forward_match_oracle(tiny):
    from dtree_mlx_b200 import kernels
    from dtree_mlx_b200.engine import Qwen3Engine, chain_anc_masks

    cfg, w = tiny
    layer_ids = [1, 3]
    eng = Qwen3Engine(w, kv_capacity=512, layer_ids=layer_ids)
    orc = Qwen3Oracle(w, kv_capacity=512)
    rng = np.random.default_rng(0)
    prompt = rng.integers(cfg.vocab_size, size=40).tolist()

    state = kernels.new_state(DEV, start=0)
    post = torch.zeros(128, dtype=torch.int32, device=DEV)
    anc = torch.from_numpy(chain_anc_masks(40).view(np.int64)).to(DEV)
    eng.forward_tree(torch.tensor(prompt, dtype=torch.int32, device=DEV),
                     torch.arange(40, dtype=torch.int32, device=DEV), anc, 40, state, post)
    torch.cuda.synchronize()
    o_norm, o_vh = orc.prefill(prompt, layer_ids=layer_ids)
    assert _rel(eng.norm_out[:40], o_norm) < REL_TOL
    assert _rel(eng.capture[:40, : 2 * cfg.hidden_size], o_vh) < REL_TOL
    for l in range(cfg.num_hidden_layers):
        assert _rel(eng.kv_cache[l, 0, :, :40], orc.k[l][:, :40]) < REL_TOL
        assert _rel(eng.kv_cache[l, 1, :, :40], orc.v[l][:, :40]) < REL_TOL
    o_log = orc.lm_head_logits(o_norm)
    mism = 0
    for t, tok in enumerate(post[:40].tolist()):
        ref = int(torch.argmax(o_log[t].to(torch.bfloat16).float()))
        if tok != ref:
            assert near_tie(o_log[t], tok, ref, LOGIT_TOL), (t, tok, ref)
            mism += 1
    print(f"prefill posterior near-tie mismatches: {mism}/40")

    # one tree step on top of the prefix
    budget = 24
    dl = torch.from_numpy((rng.standard_normal((15, cfg.vocab_size)) * 2).astype(np.float32)).to(DEV)
    state = kernels.new_state(DEV, start=40, root_token=int(post[39].item()))
    tree = kernels.TreeBuffers.allocate(DEV)
    kernels.TreeBuilder(15, cfg.vocab_size, budget, DEV).build(dl, state, tree)
    n = int(state[6].item())
    assert n == budget + 1
    eng.forward_tree(tree.tokens, tree.positions, tree.anc, n, state, post)
    torch.cuda.synchronize()
    toks = tree.tokens[:n].tolist()
    parents = tree.parents[:n].tolist()
    pos = tree.positions[:n].tolist()
    ref_tokens, ref_depths, ref_parents, _, vis = OT.build_dtree_tree(dl.cpu().numpy(), budget)
    assert toks[1:] == ref_tokens and parents == ref_parents
    mask = OT.tree_attention_mask(vis, 40)
    o_norm, o_vh = orc.forward_tree(toks, pos, mask, past=40, layer_ids=layer_ids)
    assert _rel(eng.norm_out[:n], o_norm) < REL_TOL
    assert _rel(eng.capture[:n, : 2 * cfg.hidden_size], o_vh) < REL_TOL
    from dtree_mlx_b200.kernels import linear_bf16

    x = torch.zeros(32, cfg.hidden_size, dtype=torch.bfloat16, device=DEV)
    x[:n] = eng.norm_out[:n]
    g_log = linear_bf16(x, w.embed)[:n].float().cpu()
    o_log = orc.lm_head_logits(o_norm)
    err = (g_log - o_log).abs().max().item()
    mean_err = (g_log - o_log).abs().mean().item()
    print(f"tree logits max-abs err {err:.3e} mean-abs err {mean_err:.3e}")
    assert err <= LOGIT_TOL and mean_err <= LOGIT_MEAN_TOL
    for t, tok in enumerate(post[:n].tolist()):
        ref = int(torch.argmax(o_log[t].to(torch.bfloat16).float()))
        if tok != ref:
            assert near_tie(o_log[t], tok, ref, LOGIT_TOL), (t, tok, ref)
    eng.close()


@pytest.mark.parametrize("mode", ["dtree", "dflash"])
def test_decode_steps_lockstep_with_oracle(tiny, mode):
    """Device decode steps vs the oracle loop, step by step (same draft logits)."""
    from dtree_mlx_b200.draft import PlantedDrafter
    from dtree_mlx_b200.engine import DecodeSession, Qwen3Engine, StepConfig, dtree_nodes

    cfg, w = tiny
    eng = Qwen3Engine(w, kv_capacity=1024)
    orc = Qwen3Oracle(w, kv_capacity=1024)
    rng = np.random.default_rng(1)
    prompt = rng.integers(cfg.vocab_size, size=128).tolist()
    budget = 24
    n_nodes = dtree_nodes(budget, 15, cfg.vocab_size) if mode == "dtree" else 16
    sc = StepConfig(mode, 15, budget if mode == "dtree" else 15, n_nodes)
    drafter = PlantedDrafter(seed=3, p_correct=0.8)
    sess = DecodeSession(eng, sc, output_capacity=512, drafter=drafter)
    first = sess.prefill(prompt)
    dec = OracleDecoder(orc, seed=3, p_correct=0.8, continuation=None)
    o_first = dec.prefill(prompt)
    if first != o_first:
        assert near_tie(dec.prefill_logits, first, o_first, LOGIT_TOL)
    dec.output[-1] = first
    near = 0
    for step in range(12):
        start = dec.start
        sess.step()
        torch.cuda.synchronize()
        st = sess.read_state()
        dl = sess.draft_logits.cpu().numpy()
        post = sess.posterior[:n_nodes].tolist()
        if mode == "dtree":
            res = dec.dtree_step(budget, draft_logits=dl, posterior_override=post)
            assert sess.tree.tokens[:n_nodes].tolist() == res["tree_tokens"]
            assert sess.tree.parents[:n_nodes].tolist() == res["parents"]
        else:
            res = dec.dflash_step(draft_logits=dl, posterior_override=post)
            assert sess.tree.tokens[:n_nodes].tolist() == res["tree_tokens"]
        for t in range(n_nodes):
            if post[t] != res["posterior"][t]:
                assert near_tie(res["logits"][t], post[t], res["posterior"][t], LOGIT_TOL)
                near += 1
        assert sess.accepted[: st["n_accepted"]].tolist() == res["accepted"]
        assert st["bonus_token"] == res["next"]
        assert st["start"] == dec.start and st["step"] == step + 1
        assert sess.output[: dec.start + 1].tolist() == dec.output[: dec.start + 1]
        # compacted cache rows match the oracle's (same rows, bf16 vs fp32)
        for l in range(cfg.num_hidden_layers):
            assert _rel(eng.kv_cache[l, 0, :, start : dec.start], orc.k[l][:, start : dec.start]) < REL_TOL
    print(f"{mode}: posterior near-tie mismatches over 12 steps: {near}")
    eng.close()


@pytest.mark.parametrize("quant_bits", [None, 4])
def test_generate_api_tiny(lib, quant_bits):
    from dtree_mlx_b200 import DFlashGenerator
    from dtree_mlx_b200.synthetic import random_prompt

    gen = DFlashGenerator(target_model="synthetic:qwen3-tiny:seed=0:kv=1024", draft_model="planted:p=0.8:seed=1",
                          target_quant_bits=quant_bits)
    assert gen.target_quantization == (None if quant_bits is None else {"group_size": 64, "bits": 4})
    prompt = random_prompt(128, 32768, seed=0)
    r_tree = gen.generate_from_tokens(prompt, max_new_tokens=64, decode_mode="dtree", speculative_tokens=16,
                                      tree_budget=24)
    r_lin = gen.generate_from_tokens(prompt, max_new_tokens=64, decode_mode="dflash", speculative_tokens=16,
                                     verify_mode="parallel-greedy-argmax")
    for r in (r_tree, r_lin):
        assert len(r.output_tokens) == 128 + 64
        assert r.output_tokens[:128] == prompt
        assert r.metrics["num_output_tokens"] == 64
        assert sum(r.metrics["acceptance_lengths"]) >= 64 - len(r.metrics["acceptance_lengths"])
    same = sum(1 for a, b in zip(r_tree.generated_tokens, r_lin.generated_tokens) if a == b)
    print(f"dtree vs dflash agreement {same}/64; accept dtree {r_tree.metrics['avg_acceptance_length']:.2f} "
          f"dflash {r_lin.metrics['avg_acceptance_length']:.2f}")
    # exact decoding: both equal the target's greedy stream (near-ties aside)
    first_diff = next((i for i, (a, b) in enumerate(zip(r_tree.generated_tokens, r_lin.generated_tokens)) if a != b),
                      64)
    assert first_diff >= 16


def test_attention_shape_switch_keeps_the_stream(lib, monkeypatch):
    """A generation whose keys cross the short attention bound (1024) midway
    replays the step graph of the cluster shape, then captures and replays
    the split one; its tokens equal those of a run pinned to the split shape
    (the two give bit-identical attention while the keys fit: same 128-key
    splits, the same merge arithmetic in the same order)."""
    from dtree_mlx_b200 import DFlashGenerator
    from dtree_mlx_b200.engine import Qwen3Engine
    from dtree_mlx_b200.synthetic import random_prompt

    prompt = random_prompt(960, 32768, seed=3)
    kw = dict(max_new_tokens=128, decode_mode="dtree", speculative_tokens=16, tree_budget=24)
    spec = dict(target_model="synthetic:qwen3-tiny:seed=0:kv=1536", draft_model="planted:p=0.8:seed=1")
    r_switch = DFlashGenerator(**spec).generate_from_tokens(prompt, **kw)
    monkeypatch.setattr(Qwen3Engine, "short_attention_keys", 0)
    r_split = DFlashGenerator(**spec).generate_from_tokens(prompt, **kw)
    assert len(r_switch.output_tokens) == 960 + 128
    assert r_switch.output_tokens == r_split.output_tokens
    assert _lib_device_error() == 0


def _lib_device_error() -> int:
    from dtree_mlx_b200 import _lib

    return _lib.device_error()
