"""Checkpoint I/O (dtree_mlx_b200.weights_io) on the CPU.

* the safetensors reader / writer against the ``safetensors`` package (when
  installed) for every dtype the checkpoints use;
* round trips: a Qwen3 target (bf16 and MLX 4-bit), a Qwen3.5 hybrid written
  in the Hugging Face layout (conv1d [C, 1, K], ``1 + weight`` norms) and read
  back through the reference's sanitize rules (custom_qwen35_model.py:
  1251-1275), and a DFlash drafter -- each must reproduce the engine layout
  bit for bit;
* the sanitize rules themselves on hand-made tensors;
* ``load_target_model`` / ``load_draft_model`` on a checkpoint directory.
"""
from __future__ import annotations

import json

import pytest
import torch

from dtree_mlx_b200 import weights_io as W
from dtree_mlx_b200.config import DRAFT_PRESETS, PRESETS, QWEN35_PRESETS
from dtree_mlx_b200.synthetic import (Q4Tensor, quantize_weights, random_qwen3_weights,
                                      random_qwen35_weights)


def _same(a, b) -> bool:
    if isinstance(a, Q4Tensor):
        return all(torch.equal(getattr(a, f), getattr(b, f)) for f in ("packed", "scales", "biases"))
    return a.dtype == b.dtype and torch.equal(a, b)


def test_safetensors_roundtrip_and_reference_reader(tmp_path):
    g = torch.Generator().manual_seed(0)
    tensors = {
        "a.bf16": torch.randn(7, 5, generator=g).to(torch.bfloat16),
        "b.f32": torch.randn(3, generator=g),
        "c.f16": torch.randn(2, 2, generator=g).to(torch.float16),
        "d.i32": torch.randint(-2**31, 2**31 - 1, (4, 3), generator=g, dtype=torch.int64).to(torch.int32),
        "e.u8": torch.randint(0, 255, (9,), generator=g).to(torch.uint8),
        "f.words": torch.tensor([[-1, 0x7FFFFFFF, -2**31, 5]], dtype=torch.int32),
    }
    f = tmp_path / "x.safetensors"
    W.write_safetensors(f, tensors, metadata={"format": "mlx"}, u32={"f.words"})
    back = W.read_safetensors(f)
    assert set(back) == set(tensors)
    for k in tensors:
        assert back[k].dtype == tensors[k].dtype and torch.equal(back[k], tensors[k]), k
    st = pytest.importorskip("safetensors.torch")
    ref = st.load_file(str(f))
    assert ref["f.words"].dtype == torch.uint32
    assert torch.equal(ref["f.words"].view(torch.int32), tensors["f.words"])
    for k in ("a.bf16", "b.f32", "c.f16", "d.i32", "e.u8"):
        assert ref[k].dtype == tensors[k].dtype and torch.equal(ref[k], tensors[k]), k
    # and the reader on a file the reference writer produced
    g2 = tmp_path / "y.safetensors"
    st.save_file({"w": tensors["a.bf16"], "u": ref["f.words"]}, str(g2))
    back2 = W.read_safetensors(g2)
    assert torch.equal(back2["w"], tensors["a.bf16"]) and torch.equal(back2["u"], tensors["f.words"])


@pytest.mark.parametrize("quant", [False, True])
def test_qwen3_checkpoint_roundtrip(tmp_path, quant):
    w = random_qwen3_weights(PRESETS["qwen3-tiny"], seed=1, device="cpu", norm_jitter=0.1)
    if quant:
        w = quantize_weights(w, embedding=True)
    W.save_qwen3_mlx(w, tmp_path)
    cfg = json.loads((tmp_path / "config.json").read_text())
    assert cfg["model_type"] == "qwen3" and (("quantization" in cfg) == quant)
    mt, back = W.load_target_weights(tmp_path, device="cpu")
    assert mt == "qwen3" and back.cfg == w.cfg and back.quant_bits == w.quant_bits
    assert _same(back.embed, w.embed) and _same(back.final_norm, w.final_norm)
    assert (back.embed_q4 is None) == (not quant)
    if quant:  # the 4-bit tied LM head survives the round trip
        assert _same(back.embed_q4, w.embed_q4)
    for name in ("input_norm", "qkv", "q_norm", "k_norm", "o_proj", "post_norm", "gate_up", "down"):
        for a, b in zip(getattr(back, name), getattr(w, name)):
            assert _same(a, b), name


def test_qwen3_quantized_embedding_is_lm_head_and_lookup(tmp_path):
    w = random_qwen3_weights(PRESETS["qwen3-tiny"], seed=2, device="cpu")
    W.save_qwen3_mlx(w, tmp_path)
    raw = W.read_safetensors(tmp_path / "model.safetensors")
    q = __import__("dtree_mlx_b200.synthetic", fromlist=["quantize_affine_q4"]).quantize_affine_q4(w.embed)
    raw["model.embed_tokens.weight"], raw["model.embed_tokens.scales"] = q.packed, q.scales
    raw["model.embed_tokens.biases"] = q.biases
    cfg = json.loads((tmp_path / "config.json").read_text())
    back = W.qwen3_weights_from_tensors(cfg, raw, device="cpu")
    # lookups read the dequantized rows; the 4-bit form is the tied LM head
    assert torch.equal(back.embed, W.dequantize_q4(q))
    assert torch.equal(back.embed_q4.packed, q.packed) and torch.equal(back.embed_q4.scales, q.scales)
    assert torch.equal(back.embed_q4.biases, q.biases)


def test_qwen35_hf_checkpoint_sanitized_roundtrip(tmp_path):
    w = random_qwen35_weights(QWEN35_PRESETS["qwen35-tiny"], seed=3, device="cpu", norm_jitter=0.1)
    W.save_qwen35_hf(w, tmp_path)
    raw = W.read_safetensors(tmp_path / "model.safetensors")
    conv = [k for k in raw if k.endswith("conv1d.weight")]
    assert conv and raw[conv[0]].shape[1] == 1  # Hugging Face [C, 1, K]
    mt, back = W.load_target_weights(tmp_path, device="cpu")
    assert mt == "qwen3_5" and back.cfg == w.cfg
    assert _same(back.embed, w.embed)
    # norms: stored as weight - 1 in bf16, shifted back by sanitize (+1)
    shift = lambda v: ((v.float() - 1.0).to(torch.bfloat16).float() + 1.0).to(torch.bfloat16)  # noqa: E731
    assert torch.equal(back.final_norm, shift(w.final_norm))
    for l, (a, b) in enumerate(zip(back.layers, w.layers)):
        assert set(a) == set(b), l
        for k in a:
            ref = shift(b[k]) if k in ("input_norm", "post_norm", "q_norm", "k_norm") else b[k]
            assert _same(a[k], ref), (l, k)
    assert torch.equal(back.a_log, w.a_log) and torch.equal(back.dt_bias, w.dt_bias)


def test_qwen35_sanitize_rules():
    raw = {
        "model.language_model.layers.0.input_layernorm.weight": torch.zeros(4),
        "model.language_model.layers.0.linear_attn.norm.weight": torch.zeros(4),
        "model.language_model.layers.0.linear_attn.conv1d.weight": torch.arange(24.0).view(6, 1, 4),
        "model.language_model.norm.weight": torch.zeros(4),
        "mtp.layers.0.x": torch.zeros(1),
        "model.visual.blocks.0.w": torch.zeros(1),
        "lm_head.weight": torch.zeros(2, 4),
    }
    out = W.sanitize_qwen35(raw)
    assert set(out) == {"model.layers.0.input_layernorm.weight", "model.layers.0.linear_attn.norm.weight",
                        "model.layers.0.linear_attn.conv1d.weight", "model.norm.weight"}
    assert torch.equal(out["model.layers.0.input_layernorm.weight"], torch.ones(4))  # shifted
    assert torch.equal(out["model.norm.weight"], torch.ones(4))
    assert torch.equal(out["model.layers.0.linear_attn.norm.weight"], torch.zeros(4))  # gated norm: not shifted
    assert out["model.layers.0.linear_attn.conv1d.weight"].shape == (6, 4, 1)
    # an already-sanitized MLX checkpoint is left alone
    mlx = {"model.layers.0.input_layernorm.weight": torch.ones(4),
           "model.layers.0.linear_attn.conv1d.weight": torch.zeros(6, 4, 1)}
    out2 = W.sanitize_qwen35(mlx)
    assert torch.equal(out2["model.layers.0.input_layernorm.weight"], torch.ones(4))


def test_dflash_checkpoint_roundtrip(tmp_path):
    from dtree_mlx_b200.draft import random_dflash_weights

    cfg = DRAFT_PRESETS["qwen3-tiny"]
    embed = torch.randn(cfg.vocab_size, cfg.hidden_size).to(torch.bfloat16)
    w = random_dflash_weights(cfg, embed, seed=4, norm_jitter=0.1)
    W.save_dflash_mlx(w, tmp_path)
    config, tensors = W.read_checkpoint_dir(tmp_path)
    back = W.dflash_weights_from_tensors(config, tensors, embed)
    assert back.cfg == cfg
    assert _same(back.fc, w.fc) and _same(back.hidden_norm, w.hidden_norm)
    assert _same(back.layers.final_norm, w.layers.final_norm) and back.layers.embed is embed
    for name in ("input_norm", "qkv", "q_norm", "k_norm", "o_proj", "post_norm", "gate_up", "down"):
        for a, b in zip(getattr(back.layers, name), getattr(w.layers, name)):
            assert _same(a, b), name


def test_load_target_model_from_directory(tmp_path):
    from dtree_mlx_b200.adapters import Qwen3TargetAdapter, Qwen35TargetAdapter, load_target_model

    w = random_qwen3_weights(PRESETS["qwen3-tiny"], seed=5, device="cpu")
    W.save_qwen3_mlx(w, tmp_path / "q3")
    t = load_target_model(str(tmp_path / "q3"), device="cpu", kv_capacity=256)
    assert isinstance(t.adapter, Qwen3TargetAdapter) and t.model.kv_capacity == 256
    assert torch.equal(t.model.weights.qkv[0], w.qkv[0])
    h = random_qwen35_weights(QWEN35_PRESETS["qwen35-tiny"], seed=6, device="cpu")
    W.save_qwen35_hf(h, tmp_path / "q35")
    t2 = load_target_model(str(tmp_path / "q35"), device="cpu")
    assert isinstance(t2.adapter, Qwen35TargetAdapter)
    with pytest.raises(NotImplementedError):
        load_target_model(str(tmp_path / "missing"))


@pytest.mark.gpu
def test_checkpoint_target_and_drafter_generate_like_synthetic(tmp_path, lib):
    """A target written to an MLX checkpoint and loaded back generates exactly
    the tokens of the same weights built in memory; a DFlash drafter
    checkpoint loads onto it and drives a generation."""
    from dtree_mlx_b200 import DFlashGenerator
    from dtree_mlx_b200.adapters import load_target_model
    from dtree_mlx_b200.draft import DFlashDraftModel, PlantedDrafter, load_draft_model, random_dflash_weights
    from dtree_mlx_b200.synthetic import random_prompt

    # the synthetic spec draws its weights on the GPU: save those same weights
    W.save_qwen3_mlx(random_qwen3_weights(PRESETS["qwen3-tiny"], seed=0, device="cuda"), tmp_path / "t")
    prompt = random_prompt(96, 32768, seed=1)
    kw = dict(max_new_tokens=40, decode_mode="dtree", speculative_tokens=16, tree_budget=24)
    ref = DFlashGenerator(target_model="synthetic:qwen3-tiny:seed=0:kv=1024",
                          draft_model="planted:p=0.8:seed=1").generate_from_tokens(prompt, **kw)
    target = load_target_model(str(tmp_path / "t"), kv_capacity=1024)
    got = DFlashGenerator.from_components(target, PlantedDrafter(seed=1, p_correct=0.8)).generate_from_tokens(
        prompt, **kw)
    assert got.output_tokens == ref.output_tokens
    dw = random_dflash_weights(DRAFT_PRESETS["qwen3-tiny"], target.model.weights.embed, seed=2)
    W.save_dflash_mlx(dw, tmp_path / "d")
    draft, path = load_draft_model(str(tmp_path / "d"), target=target)
    assert isinstance(draft, DFlashDraftModel) and path == tmp_path / "d"
    r = DFlashGenerator.from_components(target, draft).generate_from_tokens(prompt, **kw)
    assert len(r.output_tokens) == 96 + 40 and min(r.metrics["acceptance_lengths"]) >= 1
