"""Oracle: the DFlash block drafter forward (fp32, CPU).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates DFlashDraftModel with a KV draft cache and attention mask "none"
(dtree_mlx/draft.py:120-309 DFlashAttention / DFlashDecoderLayer, :318-367
the model) and its use per decode step (dtree_runtime.py:366-376):

  target_hidden' = hidden_norm(fc(target_hidden))                  :329-330
  per layer, context: k = k_norm(k_proj(th')) RoPE'd at the cache
      offset, v = v_proj(th') appended to the layer cache            :172-187
  block h = embed([token, mask x (bs-1)]); per layer:
      q = q_norm(q_proj(n(h))), k / v likewise from the block, RoPE at
      offset = cache length; attention to [cache | block] with no mask
      (scale head_dim^-0.5), o_proj, residual, SwiGLU MLP, residual  :189-309
  logits = norm(h) @ embed^T (the target's tied LM head)            :375
  the block's own K/V are trimmed from the cache afterwards          :377
With a context-only cache (Qwen3.5 targets) the context is windowed
(ContextOnlyDraftKVCache, :69-112).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .qwen3 import apply_rope, rms_norm


class DFlashOracle:
    """``sink`` / ``window``: the context-only draft cache
    (ContextOnlyDraftKVCache, draft.py:69-112): after every append the cache
    keeps its first ``sink`` rows and its last ``window`` rows; positions keep
    counting every appended row (cache.offset)."""

    def __init__(self, weights, target_embed, sink: int | None = None, window: int | None = None):
        self.sink, self.window = sink, window
        self.appended = 0
        w = weights
        self.cfg = c = w.cfg
        L = w.layers.to("cpu") if w.layers.device.type != "cpu" else w.layers
        self.layers = [L.reference_weights(i) for i in range(c.num_hidden_layers)]
        self.final_norm = L.final_norm.float()
        self.fc = w.fc.float().cpu()
        self.hidden_norm = w.hidden_norm.float().cpu()
        self.embed = target_embed.float().cpu()
        self.k = [torch.zeros(c.num_key_value_heads, 0, c.head_dim) for _ in self.layers]
        self.v = [torch.zeros(c.num_key_value_heads, 0, c.head_dim) for _ in self.layers]

    @property
    def offset(self) -> int:
        return self.appended if self.window is not None else self.k[0].shape[1]

    def _kv(self, L, x, pos):
        c = self.cfg
        T = x.shape[0]
        k = rms_norm((x @ L["k_proj"].float().t()).view(T, c.num_key_value_heads, c.head_dim), L["k_norm"],
                     c.rms_norm_eps)
        v = (x @ L["v_proj"].float().t()).view(T, c.num_key_value_heads, c.head_dim)
        return apply_rope(k, pos, c.rope_theta), v

    def context(self, target_hidden) -> None:
        """precompute_context_kv: append the rows at positions offset .. offset+n-1."""
        c = self.cfg
        th = rms_norm(torch.as_tensor(target_hidden).float() @ self.fc.t(), self.hidden_norm, c.rms_norm_eps)
        pos = torch.arange(self.offset, self.offset + th.shape[0])
        for i, L in enumerate(self.layers):
            k, v = self._kv(L, th, pos)
            self.k[i] = torch.cat([self.k[i], k.transpose(0, 1)], dim=1)
            self.v[i] = torch.cat([self.v[i], v.transpose(0, 1)], dim=1)
            if self.window is not None and self.k[i].shape[1] > self.sink + self.window:  # _apply_window, :95-106
                self.k[i] = torch.cat([self.k[i][:, : self.sink], self.k[i][:, -self.window:]], dim=1)
                self.v[i] = torch.cat([self.v[i][:, : self.sink], self.v[i][:, -self.window:]], dim=1)
        self.appended += th.shape[0]

    def block_logits(self, token: int) -> torch.Tensor:
        """Logits [block, vocab] of the block [token, mask x (bs-1)]; the cache
        is left as before the call (trim_draft_cache)."""
        c = self.cfg
        bs = c.block_size
        toks = torch.tensor([int(token)] + [c.mask_token_id] * (bs - 1))
        h = self.embed[toks]
        pos = torch.arange(self.offset, self.offset + bs)
        g = c.num_attention_heads // c.num_key_value_heads
        for i, L in enumerate(self.layers):
            x = rms_norm(h, L["input_layernorm"], c.rms_norm_eps)
            q = rms_norm((x @ L["q_proj"].float().t()).view(bs, c.num_attention_heads, c.head_dim), L["q_norm"],
                         c.rms_norm_eps)
            q = apply_rope(q, pos, c.rope_theta)
            k, v = self._kv(L, x, pos)
            keys = torch.cat([self.k[i], k.transpose(0, 1)], dim=1).repeat_interleave(g, dim=0)
            vals = torch.cat([self.v[i], v.transpose(0, 1)], dim=1).repeat_interleave(g, dim=0)
            s = (q.transpose(0, 1) @ keys.transpose(1, 2)) / math.sqrt(c.head_dim)
            o = (torch.softmax(s, dim=-1) @ vals).transpose(0, 1).reshape(bs, -1)
            h = h + o @ L["o_proj"].float().t()
            x = rms_norm(h, L["post_attention_layernorm"], c.rms_norm_eps)
            h = h + (torch.nn.functional.silu(x @ L["gate_proj"].float().t()) * (x @ L["up_proj"].float().t())) \
                @ L["down_proj"].float().t()
        return rms_norm(h, self.final_norm, c.rms_norm_eps) @ self.embed.t()
