"""Pins the fp32 layer oracles to a published implementation of the same models.

``oracle/qwen3.py`` and ``oracle/qwen35.py`` restate the layer arithmetic the
reference gets from mlx-lm (RMSNorm placement, q/k-norm, half-split RoPE,
SwiGLU, tied head; gated DeltaNet, RMSNormGated, gated attention with partial
RoPE).  Here they are checked against Hugging Face ``transformers``' own
``Qwen3ForCausalLM`` and ``Qwen3_5ForCausalLM`` (eager attention, the pure
PyTorch chunked gated-delta rule), built on the oracle's weights, in fp32 on
the CPU:

* a causal prefill: every row's logits;
* a tree step: node t of a best-first tree sees the prompt and its own root
  path, so its logits must equal the last row of the plain causal forward
  over ``prompt + path(t)`` at positions ``past .. past + depth(t)``
  (qwen3_tree.py:69-76 / qwen35_tree.py:180-480 against the sequence model);
  for Qwen3 also once more as one forward with the tree's 4-D additive mask.

Weight conventions mapped explicitly:
* transformers' Qwen3.5 RMSNorm multiplies by ``1 + weight``; the reference's
  checkpoints store ``weight + 1`` after ``sanitize``
  (custom_qwen35_model.py:1251-1275), which is what the oracle multiplies by,
  so the HF module gets ``weight - 1`` (the gated norm is not shifted);
* the HF depthwise conv weight [C, 1, K] is the oracle's [K, C] transposed;
* the reference normalises DeltaNet q/k with ``mx.fast.rms_norm(x, None,
  1e-6)`` scaled by D^-1 / D^-1/2 (qwen35_tree.py:304-306), the HF/FLA
  ``l2norm`` puts its 1e-6 on the sum of squares instead of the mean; the
  test swaps in the reference's placement so that the rest compares exactly.

Tolerance: max |logit difference| <= 1e-5 (fp32 vs fp32; logits are O(1)).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import tree as OT
from oracle.qwen3 import Qwen3Oracle
from oracle.qwen35 import Qwen35Oracle

TOL = 1e-5

transformers = pytest.importorskip("transformers")


def _tree(rng, rows: int, vocab: int, budget: int):
    logits = (rng.standard_normal((rows, vocab)) * 2).astype(np.float32)
    logits[:, rng.integers(vocab, size=4)] += 5.0
    toks, depths, parents, _, vis = OT.build_dtree_tree(logits, budget)
    return toks, depths, parents, vis


def _path(parents, t):
    out = []
    while t >= 0:
        out.append(t)
        t = parents[t]
    return out[::-1]


# ---------------------------------------------------------------- Qwen3
def _hf_qwen3(w):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    c = w.cfg
    hc = Qwen3Config(vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
                     num_hidden_layers=c.num_hidden_layers, num_attention_heads=c.num_attention_heads,
                     num_key_value_heads=c.num_key_value_heads, head_dim=c.head_dim, rms_norm_eps=c.rms_norm_eps,
                     rope_parameters={"rope_type": "default", "rope_theta": c.rope_theta},
                     tie_word_embeddings=True, max_position_embeddings=4096, attention_bias=False)
    hc._attn_implementation = "eager"
    m = Qwen3ForCausalLM(hc).float().eval()
    sd = {"model.embed_tokens.weight": w.embed, "model.norm.weight": w.final_norm, "lm_head.weight": w.embed}
    for i in range(c.num_hidden_layers):
        r = w.reference_weights(i)
        p = f"model.layers.{i}."
        sd.update({p + "input_layernorm.weight": r["input_layernorm"],
                   p + "post_attention_layernorm.weight": r["post_attention_layernorm"],
                   p + "self_attn.q_proj.weight": r["q_proj"], p + "self_attn.k_proj.weight": r["k_proj"],
                   p + "self_attn.v_proj.weight": r["v_proj"], p + "self_attn.o_proj.weight": r["o_proj"],
                   p + "self_attn.q_norm.weight": r["q_norm"], p + "self_attn.k_norm.weight": r["k_norm"],
                   p + "mlp.gate_proj.weight": r["gate_proj"], p + "mlp.up_proj.weight": r["up_proj"],
                   p + "mlp.down_proj.weight": r["down_proj"]})
    missing, unexpected = m.load_state_dict({k: v.float() for k, v in sd.items()}, strict=False)
    assert not unexpected and not [k for k in missing if "rotary" not in k], (missing, unexpected)
    return m


@pytest.fixture(scope="module")
def qwen3_pair():
    from dtree_mlx_b200.config import PRESETS
    from dtree_mlx_b200.synthetic import random_qwen3_weights

    cfg = PRESETS["qwen3-tiny"]
    w = random_qwen3_weights(cfg, seed=0, device="cpu", norm_jitter=0.1)
    return w, _hf_qwen3(w)


@torch.no_grad()
def test_qwen3_prefill_matches_transformers(qwen3_pair):
    w, hf = qwen3_pair
    rng = np.random.default_rng(0)
    prompt = rng.integers(w.cfg.vocab_size, size=40).tolist()
    orc = Qwen3Oracle(w, kv_capacity=256)
    norm_h, _ = orc.prefill(prompt)
    ours = orc.lm_head_logits(norm_h)
    ref = hf(torch.tensor([prompt])).logits[0]
    err = (ours - ref).abs().max().item()
    print(f"qwen3 prefill max |oracle - transformers| = {err:.2e}")
    assert err <= TOL


@torch.no_grad()
def test_qwen3_tree_step_matches_transformers_paths(qwen3_pair):
    w, hf = qwen3_pair
    rng = np.random.default_rng(1)
    past = 40
    prompt = rng.integers(w.cfg.vocab_size, size=past).tolist()
    toks, depths, parents, vis = _tree(rng, 15, w.cfg.vocab_size, 24)
    root = int(rng.integers(w.cfg.vocab_size))
    tree_tokens = [root] + toks
    tree_depths = [0] + depths
    orc = Qwen3Oracle(w, kv_capacity=256)
    orc.prefill(prompt)
    mask = OT.tree_attention_mask(vis, past)
    norm_h, _ = orc.forward_tree(tree_tokens, [past + d for d in tree_depths], mask, past=past)
    ours = orc.lm_head_logits(norm_h)
    worst = 0.0
    for t in range(len(tree_tokens)):
        seq = prompt + [tree_tokens[j] for j in _path(parents, t)]
        ref = hf(torch.tensor([seq])).logits[0, -1]
        worst = max(worst, (ours[t] - ref).abs().max().item())
    print(f"qwen3 tree ({len(tree_tokens)} nodes) max |oracle - transformers path| = {worst:.2e}")
    assert worst <= TOL

    # the same step as one forward with the tree's 4-D additive mask
    T = len(tree_tokens)
    L = past + T
    add = torch.zeros(1, 1, L, L)
    full = np.zeros((L, L), dtype=bool)
    full[:past, :past] = np.tril(np.ones((past, past), dtype=bool))
    full[past:, :] = mask
    add[0, 0][~torch.from_numpy(full)] = torch.finfo(torch.float32).min
    pos = list(range(past)) + [past + d for d in tree_depths]
    ref = hf(torch.tensor([prompt + tree_tokens]), attention_mask=add, position_ids=torch.tensor([pos])).logits[0]
    err = (ours - ref[past:]).abs().max().item()
    print(f"qwen3 tree 4-D mask max |oracle - transformers| = {err:.2e}")
    assert err <= TOL


# ---------------------------------------------------------------- Qwen3.5
def _hf_qwen35(w):
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig

    c = w.cfg
    types = ["linear_attention" if c.is_linear(l) else "full_attention" for l in range(c.num_hidden_layers)]
    hc = Qwen3_5TextConfig(vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
                           num_hidden_layers=c.num_hidden_layers, num_attention_heads=c.num_attention_heads,
                           num_key_value_heads=c.num_key_value_heads, head_dim=c.head_dim,
                           linear_conv_kernel_dim=c.linear_conv_kernel_dim,
                           linear_key_head_dim=c.linear_key_head_dim, linear_value_head_dim=c.linear_value_head_dim,
                           linear_num_key_heads=c.linear_num_key_heads,
                           linear_num_value_heads=c.linear_num_value_heads, layer_types=types,
                           rms_norm_eps=c.rms_norm_eps, tie_word_embeddings=True, max_position_embeddings=4096,
                           rope_parameters={"rope_type": "default", "rope_theta": c.rope_theta,
                                            "partial_rotary_factor": c.partial_rotary_factor})
    hc._attn_implementation = "eager"
    m = M.Qwen3_5ForCausalLM(hc).float().eval()
    shift = lambda t: t.float() - 1.0  # noqa: E731  (HF multiplies by 1 + weight)
    sd = {"model.embed_tokens.weight": w.embed.float(), "model.norm.weight": shift(w.final_norm),
          "lm_head.weight": w.embed.float()}
    for l in range(c.num_hidden_layers):
        r = w.reference_layer(l)
        p = f"model.layers.{l}."
        sd.update({p + "input_layernorm.weight": shift(r["input_layernorm"]),
                   p + "post_attention_layernorm.weight": shift(r["post_attention_layernorm"]),
                   p + "mlp.gate_proj.weight": r["gate_proj"].float(), p + "mlp.up_proj.weight": r["up_proj"].float(),
                   p + "mlp.down_proj.weight": r["down_proj"].float()})
        if c.is_linear(l):
            a = p + "linear_attn."
            sd.update({a + "in_proj_qkv.weight": r["in_proj_qkv"].float(), a + "in_proj_z.weight": r["in_proj_z"].float(),
                       a + "in_proj_b.weight": r["in_proj_b"].float(), a + "in_proj_a.weight": r["in_proj_a"].float(),
                       a + "conv1d.weight": r["conv_weight"].float().t().unsqueeze(1).contiguous(),
                       a + "dt_bias": r["dt_bias"].float(), a + "A_log": r["A_log"].float(),
                       a + "norm.weight": r["norm"].float(), a + "out_proj.weight": r["out_proj"].float()})
        else:
            a = p + "self_attn."
            sd.update({a + "q_proj.weight": r["q_proj"].float(), a + "k_proj.weight": r["k_proj"].float(),
                       a + "v_proj.weight": r["v_proj"].float(), a + "o_proj.weight": r["o_proj"].float(),
                       a + "q_norm.weight": shift(r["q_norm"]), a + "k_norm.weight": shift(r["k_norm"])})
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected and not [k for k in missing if "rotary" not in k], (missing, unexpected)
    for layer in m.model.layers:  # the pure PyTorch gated-delta rule
        if hasattr(layer, "linear_attn"):
            layer.linear_attn.chunk_gated_delta_rule = M.torch_chunk_gated_delta_rule
    return m


@pytest.fixture(scope="module")
def qwen35_pair():
    from dtree_mlx_b200.config import QWEN35_PRESETS
    from dtree_mlx_b200.synthetic import random_qwen35_weights

    cfg = QWEN35_PRESETS["qwen35-tiny"]
    w = random_qwen35_weights(cfg, seed=0, device="cpu", norm_jitter=0.1)
    return w, _hf_qwen35(w)


@pytest.fixture()
def reference_qk_norm(monkeypatch):
    """mx.fast.rms_norm(x, None, 1e-6) / sqrt(D) (qwen35_tree.py:304-306) in
    place of the HF/FLA l2norm (eps on the sum of squares)."""
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M

    def l2norm(x, dim=-1, eps=1e-6):
        return x * torch.rsqrt(x.pow(2).mean(dim, keepdim=True) + eps) / math.sqrt(x.shape[dim])

    monkeypatch.setattr(M, "l2norm", l2norm)


def _oracle35(w, **kw):
    return Qwen35Oracle(w, kv_capacity=256, **kw)


@torch.no_grad()
def test_qwen35_prefill_matches_transformers(qwen35_pair, reference_qk_norm):
    w, hf = qwen35_pair
    rng = np.random.default_rng(2)
    prompt = rng.integers(w.cfg.vocab_size, size=48).tolist()
    orc = _oracle35(w)
    norm_h, _ = orc.prefill(prompt)
    ours = orc.lm_head_logits(norm_h)
    ref = hf(torch.tensor([prompt])).logits[0]
    err = (ours - ref).abs().max().item()
    print(f"qwen3.5 prefill max |oracle - transformers| = {err:.2e}")
    assert err <= TOL


@torch.no_grad()
def test_qwen35_tree_step_matches_transformers_paths(qwen35_pair, reference_qk_norm):
    """fp32 node states (the reference's tree kernel keeps node states in the
    input dtype, fp32 for an fp32 model): each node equals its root path run
    as a sequence."""
    w, hf = qwen35_pair
    rng = np.random.default_rng(3)
    past = 32
    prompt = rng.integers(w.cfg.vocab_size, size=past).tolist()
    toks, depths, parents, vis = _tree(rng, 15, w.cfg.vocab_size, 24)
    tree_tokens = [int(rng.integers(w.cfg.vocab_size))] + toks
    tree_depths = [0] + depths
    orc = _oracle35(w, state_dtype="f32")
    orc.prefill(prompt)
    mask = OT.tree_attention_mask(vis, past)
    norm_h, _ = orc.forward(tree_tokens, [past + d for d in tree_depths], parents, mask, past, tree=True)
    ours = orc.lm_head_logits(norm_h)
    worst = 0.0
    for t in range(len(tree_tokens)):
        seq = prompt + [tree_tokens[j] for j in _path(parents, t)]
        ref = hf(torch.tensor([seq])).logits[0, -1]
        worst = max(worst, (ours[t] - ref).abs().max().item())
    print(f"qwen3.5 tree ({len(tree_tokens)} nodes) max |oracle - transformers path| = {worst:.2e}")
    assert worst <= TOL
