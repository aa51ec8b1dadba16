"""MLX affine 4-bit weights: packing layout, quantizer bounds and the oracle's
dequantization (CPU only).

The layout is the one mlx.core.quantize documents and the reference's
quantize_model produces (dtree_mlx/api.py:46-54): a row of K weights becomes
K/8 uint32 words, element 8j+i in bits 4i..4i+3 of word j, with one bf16
scale and bias per group of 64 consecutive elements; w = scale * q + bias.
"""
from __future__ import annotations

import numpy as np
import torch

from dtree_mlx_b200.synthetic import Q4Tensor, quantize_affine_q4, quantize_weights, split_gate_up
from oracle.qwen3 import dequant_affine_q4


def _pack_loop(q: np.ndarray) -> np.ndarray:
    """Reference packing by explicit loops (uint32 words as int32)."""
    n, k = q.shape
    out = np.zeros((n, k // 8), dtype=np.uint64)
    for r in range(n):
        for j in range(k // 8):
            w = 0
            for i in range(8):
                w |= int(q[r, 8 * j + i]) << (4 * i)
            out[r, j] = w
    return out.astype(np.uint32).view(np.int32)


def test_dequant_matches_loop_on_known_codes():
    rng = np.random.default_rng(0)
    n, k = 5, 128
    q = rng.integers(0, 16, size=(n, k))
    s = torch.from_numpy(rng.uniform(0.001, 0.01, size=(n, k // 64)).astype(np.float32)).to(torch.bfloat16)
    b = torch.from_numpy(rng.uniform(-0.05, 0.05, size=(n, k // 64)).astype(np.float32)).to(torch.bfloat16)
    packed = torch.from_numpy(_pack_loop(q))
    w = dequant_affine_q4(packed, s, b)
    for r in range(n):
        for c in range(k):
            exp = float(s[r, c // 64]) * int(q[r, c]) + float(b[r, c // 64])
            assert abs(float(w[r, c]) - exp) <= 1e-7 * max(1.0, abs(exp))


def test_quantizer_layout_and_error_bound():
    g = torch.Generator().manual_seed(1)
    w = (torch.randn(192, 256, generator=g) * 0.02).to(torch.bfloat16)
    qt = quantize_affine_q4(w)
    assert qt.packed.dtype == torch.int32 and qt.packed.shape == (192, 32)
    assert qt.scales.shape == (192, 4) and qt.biases.dtype == torch.bfloat16
    # unpack by the documented rule and re-pack by loops: identical words
    words = qt.packed.numpy().view(np.uint32).astype(np.uint64)
    q = np.stack([(words >> np.uint64(4 * i)) & np.uint64(15) for i in range(8)], axis=-1).reshape(192, 256)
    assert np.array_equal(_pack_loop(q), qt.packed.numpy())
    # |w - dequant| within half a step (+ the bf16 rounding of scale / bias)
    wd = dequant_affine_q4(qt.packed, qt.scales, qt.biases)
    step = qt.scales.float().repeat_interleave(64, dim=1)
    err = (wd - w.float()).abs()
    assert bool((err <= 0.5 * step + 2.0 ** -7 * w.float().abs().max()).all())
    # every group uses the full code range [0, 15]
    assert int(q.min()) == 0 and int(q.max()) == 15


def test_quantized_weights_keep_row_order():
    """Quantizing the packed q|k|v and interleaved gate|up storage equals
    quantizing the individual projections (groups run along the input dim)."""
    from dtree_mlx_b200.config import PRESETS
    from dtree_mlx_b200.synthetic import random_qwen3_weights

    cfg = PRESETS["qwen3-tiny"]
    w = random_qwen3_weights(cfg, seed=0, device="cpu")
    q = quantize_weights(w)
    assert q.quant_bits == 4 and isinstance(q.qkv[0], Q4Tensor)
    ref = w.reference_weights(1)
    got = q.reference_weights(1)
    for name in ("k_proj", "gate_proj", "up_proj", "down_proj"):
        direct = quantize_affine_q4(ref[name])
        assert torch.equal(got[name].packed, direct.packed), name
        assert torch.equal(got[name].scales, direct.scales), name
    gate, up = split_gate_up(q.gate_up[0])
    assert gate.shape == (cfg.intermediate_size, cfg.hidden_size) and up.shape == gate.shape
    # BASELINE config 3 keeps the embedding; quantize_model's form
    # (embedding=True) quantizes it too: the tied LM head is 4-bit and the
    # lookup table holds its dequantized rows
    from dtree_mlx_b200.weights_io import dequantize_q4

    assert q.embed_q4 is None and torch.equal(q.embed, w.embed)
    qe = quantize_weights(w, embedding=True)
    assert qe.embed_q4 is not None and torch.equal(qe.embed_q4.packed, quantize_affine_q4(w.embed).packed)
    assert torch.equal(qe.embed, dequantize_q4(qe.embed_q4))
    # 0.5625 bytes per parameter (+ the bf16 lookup table and norms)
    proj = sum(t.nbytes() for t in (*q.qkv, *q.o_proj, *q.gate_up, *q.down))
    n_param = sum(t.shape[0] * t.shape[1] for t in (*q.qkv, *q.o_proj, *q.gate_up, *q.down))
    assert proj == int(n_param * 0.5625)
