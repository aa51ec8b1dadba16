"""Seeded random-init Qwen3 weights in the engine's packed layouts.

BASELINE configs use random-init weights (normal, std 0.02; RMSNorm weights
1.0) because no checkpoint is available offline.  Weights are generated on
the target device with a seeded ``torch.Generator`` and stored once, packed
for the verify GEMMs:

* ``qkv[l]``      [(Hq + 2 Hkv) * d, H]  rows q | k | v
* ``gate_up[l]``  [2F, H] in 64-row blocks: gate rows 64j..64j+63 followed by
                  the matching up rows (so one 128-row GEMM tile holds both
                  halves of 64 SwiGLU features)

``reference_weights()`` returns mlx-lm-named views (q_proj, gate_proj, ...)
of the same storage for the CPU oracle.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .config import Qwen3Config

STD = 0.02


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    f, h = gate.shape
    assert f % 64 == 0
    out = torch.empty(2 * f, h, dtype=gate.dtype, device=gate.device)
    v = out.view(f // 64, 2, 64, h)
    v[:, 0] = gate.view(f // 64, 64, h)
    v[:, 1] = up.view(f // 64, 64, h)
    return out


def split_gate_up(gate_up: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    two_f, h = gate_up.shape
    f = two_f // 2
    v = gate_up.view(f // 64, 2, 64, h)
    return v[:, 0].reshape(f, h), v[:, 1].reshape(f, h)


@dataclass
class Qwen3Weights:
    cfg: Qwen3Config
    embed: torch.Tensor
    final_norm: torch.Tensor
    input_norm: list[torch.Tensor] = field(default_factory=list)
    qkv: list[torch.Tensor] = field(default_factory=list)
    q_norm: list[torch.Tensor] = field(default_factory=list)
    k_norm: list[torch.Tensor] = field(default_factory=list)
    o_proj: list[torch.Tensor] = field(default_factory=list)
    post_norm: list[torch.Tensor] = field(default_factory=list)
    gate_up: list[torch.Tensor] = field(default_factory=list)
    down: list[torch.Tensor] = field(default_factory=list)

    @property
    def device(self) -> torch.device:
        return self.embed.device

    def nbytes(self) -> int:
        ts = [self.embed, self.final_norm]
        for name in ("input_norm", "qkv", "q_norm", "k_norm", "o_proj", "post_norm", "gate_up", "down"):
            ts += getattr(self, name)
        return sum(t.numel() * t.element_size() for t in ts)

    def reference_weights(self, layer: int) -> dict[str, torch.Tensor]:
        """mlx-lm Qwen3 names for one layer (views / splits of the packed storage)."""
        c = self.cfg
        qkv = self.qkv[layer]
        gate, up = split_gate_up(self.gate_up[layer])
        return {
            "input_layernorm": self.input_norm[layer],
            "q_proj": qkv[: c.q_dim],
            "k_proj": qkv[c.q_dim : c.q_dim + c.kv_dim],
            "v_proj": qkv[c.q_dim + c.kv_dim :],
            "q_norm": self.q_norm[layer],
            "k_norm": self.k_norm[layer],
            "o_proj": self.o_proj[layer],
            "post_attention_layernorm": self.post_norm[layer],
            "gate_proj": gate,
            "up_proj": up,
            "down_proj": self.down[layer],
        }

    def to(self, device) -> "Qwen3Weights":
        mv = lambda t: t.to(device)  # noqa: E731
        w = Qwen3Weights(self.cfg, mv(self.embed), mv(self.final_norm))
        for name in ("input_norm", "qkv", "q_norm", "k_norm", "o_proj", "post_norm", "gate_up", "down"):
            setattr(w, name, [mv(t) for t in getattr(self, name)])
        return w


def random_qwen3_weights(cfg: Qwen3Config, seed: int = 0, device="cuda", dtype=torch.bfloat16,
                         norm_jitter: float = 0.0) -> Qwen3Weights:
    """N(0, 0.02) linear/embedding weights, fixed generation order.  RMSNorm
    weights are 1.0, or 1 + N(0, norm_jitter) when ``norm_jitter`` > 0 (the
    parity tests use that to exercise the norm-weight multiplication)."""
    g = torch.Generator(device=device).manual_seed(int(seed))

    def randn(*shape):
        return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * STD).to(dtype)

    def ones(n):
        if norm_jitter > 0:
            return (1.0 + torch.randn(n, generator=g, device=device) * norm_jitter).to(dtype)
        return torch.ones(n, dtype=dtype, device=device)

    h, f = cfg.hidden_size, cfg.intermediate_size
    w = Qwen3Weights(cfg, embed=randn(cfg.vocab_size, h), final_norm=ones(h))
    for _ in range(cfg.num_hidden_layers):
        q = randn(cfg.q_dim, h)
        k = randn(cfg.kv_dim, h)
        v = randn(cfg.kv_dim, h)
        w.qkv.append(torch.cat([q, k, v], dim=0).contiguous())
        del q, k, v
        w.o_proj.append(randn(h, cfg.q_dim))
        gate = randn(f, h)
        up = randn(f, h)
        w.gate_up.append(interleave_gate_up(gate, up))
        del gate, up
        w.down.append(randn(h, f))
        w.input_norm.append(ones(h))
        w.post_norm.append(ones(h))
        w.q_norm.append(ones(cfg.head_dim))
        w.k_norm.append(ones(cfg.head_dim))
    return w


def random_prompt(n: int, vocab: int, seed: int = 0) -> list[int]:
    """Uniform-random prompt token ids (128 / 256 / 2048)."""
    g = torch.Generator().manual_seed(int(seed) + 7919)
    return torch.randint(0, vocab, (n,), generator=g).tolist()
