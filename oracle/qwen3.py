"""Oracle: fp32 PyTorch-CPU restatement of the Qwen3 target on the DTree path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows the reference's tree block and adapter:
* ``forward_tree``   Qwen3TargetAdapter.forward_tree_with_hidden_states
                     (dtree_mlx/adapters.py:568-597) with the compiled tree
                     block of dtree_mlx/qwen3_tree.py:39-83
* ``prefill``        Qwen3TargetAdapter._forward_states (adapters.py:494-514),
                     i.e. the same block with a causal mask
* ``apply_rope``     apply_rope_position_ids (qwen3_tree.py:22-27): mlx
                     ``nn.RoPE(traditional=False)`` = half-split rotation,
                     inv_freq_i = theta^(-2i/d), per-token positions
* ``lm_head_*``      tied embedding LM head (adapters.py:489-492) and its
                     argmax (adapters.py:114-118): argmax over bf16 logits,
                     first index on ties
* ``compact``        compact_kv_caches (adapters.py:635-668)

The arithmetic inside mlx-lm's layers (RMSNorm, SDPA, SwiGLU) is restated
from their public definitions and computed in fp32 from the same bf16 weights
the GPU uses (``parity unpinned`` by the reference's own tests; see DESIGN).
"""
from __future__ import annotations

import math

import numpy as np
import torch


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def apply_rope(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """x [..., T, heads, d] or [T, heads, d]; positions [T]."""
    d = x.shape[-1]
    half = d // 2
    inv = theta ** (-(torch.arange(half, dtype=torch.float64) * 2.0 / d))
    ang = positions.double()[:, None] * inv[None, :]  # [T, half]
    cos = torch.cos(ang).float()[:, None, :]
    sin = torch.sin(ang).float()[:, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)


def dequant_affine_q4(packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                      group_size: int = 64) -> torch.Tensor:
    """fp32 weights of an MLX affine 4-bit matrix: w[n, k] = scales[n, k/g] *
    q[n, k] + biases[n, k/g], q = bits 4i..4i+3 of word k/8 (i = k % 8) of row
    n.  This is the weight the reference's QuantizedLinear layers multiply by
    after quantize_model(bits=4, group_size=64) (dtree_mlx/api.py:46-54; the
    chunked argmax of adapters.py:63-71 goes through the same
    quantized_matmul)."""
    words = packed.to(torch.int64) & 0xFFFFFFFF  # [N, K/8]
    n = words.shape[0]
    q = torch.stack([(words >> (4 * i)) & 0xF for i in range(8)], dim=-1).reshape(n, -1).float()
    s = scales.float().repeat_interleave(group_size, dim=1)
    b = biases.float().repeat_interleave(group_size, dim=1)
    return s * q + b


def _dense(t):
    """Oracle view of a projection weight: the tensor itself, or the fp32
    dequantization of a 4-bit one (objects with packed / scales / biases)."""
    if hasattr(t, "packed"):
        return dequant_affine_q4(t.packed, t.scales, t.biases, t.group_size)
    return t


class Qwen3Oracle:
    """fp32 CPU model over a ``Qwen3Weights`` (weights are copied to CPU)."""

    def __init__(self, weights, kv_capacity: int, bf16_acts: bool = False):
        # bf16_acts: round every activation a bf16 model materializes (norm
        # outputs, projections, attention output, SwiGLU, residual stream) to
        # bf16 -- an estimate of the bf16 rounding noise floor, not a bar
        self.bf16_acts = bool(bf16_acts)
        self.w = weights.to("cpu") if weights.device.type != "cpu" else weights
        self.cfg = self.w.cfg
        c = self.cfg
        self.layers = [{k: _dense(v) for k, v in self.w.reference_weights(i).items()}
                       for i in range(c.num_hidden_layers)]
        self.cap = int(kv_capacity)
        self.k = [torch.zeros(c.num_key_value_heads, self.cap, c.head_dim) for _ in self.layers]
        self.v = [torch.zeros(c.num_key_value_heads, self.cap, c.head_dim) for _ in self.layers]
        self.offset = 0

    # ------------------------------------------------------------------ block
    def _block(self, i: int, h: torch.Tensor, positions: torch.Tensor, mask: torch.Tensor, past: int):
        c = self.cfg
        L = self.layers[i]
        T = h.shape[0]
        r = self._r
        x = r(rms_norm(h, L["input_layernorm"], c.rms_norm_eps))
        q = r(x @ L["q_proj"].float().t())
        k = r(x @ L["k_proj"].float().t())
        v = r(x @ L["v_proj"].float().t())
        q = r(rms_norm(q.view(T, c.num_attention_heads, c.head_dim), L["q_norm"], c.rms_norm_eps))
        k = r(rms_norm(k.view(T, c.num_key_value_heads, c.head_dim), L["k_norm"], c.rms_norm_eps))
        v = v.view(T, c.num_key_value_heads, c.head_dim)
        q = r(apply_rope(q, positions, c.rope_theta))
        k = r(apply_rope(k, positions, c.rope_theta))
        # new K/V appended after the prefix (cache.update_and_fetch, qwen3_tree.py:146)
        self.k[i][:, past : past + T] = k.transpose(0, 1)
        self.v[i][:, past : past + T] = v.transpose(0, 1)
        keys = self.k[i][:, : past + T]  # [Hkv, P+T, d]
        vals = self.v[i][:, : past + T]
        g = c.num_attention_heads // c.num_key_value_heads
        keys = keys.repeat_interleave(g, dim=0)
        vals = vals.repeat_interleave(g, dim=0)
        qh = q.transpose(0, 1)  # [Hq, T, d]
        scores = (qh @ keys.transpose(1, 2)) / math.sqrt(c.head_dim)
        scores = scores.masked_fill(~mask[None, :, :], float("-inf"))
        attn = r(torch.softmax(scores, dim=-1) @ vals)  # [Hq, T, d]
        h = r(h + r(attn.transpose(0, 1).reshape(T, c.q_dim) @ L["o_proj"].float().t()))
        x = r(rms_norm(h, L["post_attention_layernorm"], c.rms_norm_eps))
        gate = r(x @ L["gate_proj"].float().t())
        up = r(x @ L["up_proj"].float().t())
        h = r(h + r(r(torch.nn.functional.silu(gate)) * up) @ L["down_proj"].float().t())
        return h

    def _r(self, x: torch.Tensor) -> torch.Tensor:
        return x.to(torch.bfloat16).float() if self.bf16_acts else x

    def forward_tree(self, tokens, positions, mask, past: int, layer_ids=()):
        """tokens/positions [T] ints, mask bool [T, past+T].  Writes the new K/V at
        [past, past+T).  Returns (norm_hidden [T,H], verifier_hidden [T, H*n])."""
        c = self.cfg
        tokens = torch.as_tensor(np.asarray(tokens), dtype=torch.long)
        positions = torch.as_tensor(np.asarray(positions), dtype=torch.long)
        mask = torch.as_tensor(np.asarray(mask), dtype=torch.bool)
        h = self.w.embed[tokens].float()
        picked = []
        ids = set(layer_ids)
        for i in range(c.num_hidden_layers):
            h = self._block(i, h, positions, mask, past)
            if i in ids:
                picked.append(h.clone())
        norm_h = self._r(rms_norm(h, self.w.final_norm, c.rms_norm_eps))
        vh = torch.cat(picked, dim=-1) if picked else h[:, :0]
        self.offset = past + len(tokens)
        return norm_h, vh

    def prefill(self, tokens, layer_ids=()):
        T = len(tokens)
        past = self.offset
        mask = np.ones((T, past + T), dtype=bool)
        mask[:, past:] = np.tril(np.ones((T, T), dtype=bool))
        return self.forward_tree(tokens, np.arange(past, past + T), mask, past, layer_ids)

    # ------------------------------------------------------------------ head
    def lm_head_logits(self, norm_h: torch.Tensor) -> torch.Tensor:
        return norm_h.float() @ self.w.embed.float().t()

    @staticmethod
    def argmax_bf16(logits: torch.Tensor) -> torch.Tensor:
        """Greedy posterior as the reference computes it: argmax over bf16 logits
        (mlx matmul output dtype), first index on ties."""
        lb = logits.to(torch.bfloat16).float()
        return torch.argmax(lb, dim=-1)

    def lm_head_argmax(self, norm_h):
        return self.argmax_bf16(self.lm_head_logits(norm_h))

    # ------------------------------------------------------------------ cache
    def compact(self, past: int, keep: list[int]):
        keep_t = torch.as_tensor(keep, dtype=torch.long)
        n = len(keep)
        cur = self.offset - past
        if n == 0:
            self.offset = past
            return
        if n == cur:
            return
        for i in range(len(self.layers)):
            self.k[i][:, past : past + n] = self.k[i][:, past : past + cur][:, keep_t].clone()
            self.v[i][:, past : past + n] = self.v[i][:, past : past + cur][:, keep_t].clone()
        self.offset = past + n

    def rewind(self, n: int):
        self.offset -= n
