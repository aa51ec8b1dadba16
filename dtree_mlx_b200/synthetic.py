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

``quantize_weights(w, bits=4, group_size=64)`` turns the four projections of
every layer into MLX affine 4-bit tensors (``Q4Tensor``: packed uint32
[N, K/8], bf16 scales / biases [N, K/64]), which is what the reference's
``quantize_model`` does to a loaded target (dtree_mlx/api.py:46-54).  The
embedding (the tied LM head) and the norms stay bf16.
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


def split_gate_up(gate_up):
    """Inverse of ``interleave_gate_up`` (also for a ``Q4Tensor``)."""
    if isinstance(gate_up, Q4Tensor):
        parts = [split_gate_up(t) for t in (gate_up.packed, gate_up.scales, gate_up.biases)]
        return tuple(Q4Tensor(*(p[i] for p in parts), gate_up.group_size) for i in range(2))
    two_f = gate_up.shape[0]
    f = two_f // 2
    v = gate_up.view(f // 64, 2, 64, -1)
    return v[:, 0].reshape(f, -1), v[:, 1].reshape(f, -1)


@dataclass
class Q4Tensor:
    """MLX affine 4-bit matrix: w[n, k] ~ scales[n, k//64] * q[n, k] + biases[n, k//64].

    ``packed`` is int32 [N, K/8] holding uint32 words, element 8j+i of a row in
    bits 4i..4i+3 of word j (MLX ``quantize`` layout); ``scales`` and
    ``biases`` are bf16 [N, K/64]."""

    packed: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    group_size: int = 64

    @property
    def shape(self) -> tuple[int, int]:
        return (self.packed.shape[0], self.packed.shape[1] * 8)

    @property
    def device(self) -> torch.device:
        return self.packed.device

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.packed, self.scales, self.biases))

    def rows(self, sl) -> "Q4Tensor":
        return Q4Tensor(self.packed[sl], self.scales[sl], self.biases[sl], self.group_size)

    def to(self, device) -> "Q4Tensor":
        return Q4Tensor(self.packed.to(device), self.scales.to(device), self.biases.to(device), self.group_size)


def tensor_bytes(t) -> int:
    """Bytes of a bf16 tensor or a Q4Tensor (packed + scales + biases)."""
    return t.nbytes() if isinstance(t, Q4Tensor) else t.numel() * t.element_size()


def quantize_affine_q4(w: torch.Tensor, group_size: int = 64) -> Q4Tensor:
    """MLX affine quantization (documented for ``mlx.core.quantize``) with
    bits = 4: per group of ``group_size`` consecutive inputs, beta = min,
    alpha = max, scale = (alpha - beta) / 15, q = round((w - beta) / scale)
    clipped to [0, 15]; scale and bias are stored in bf16."""
    n, k = w.shape
    if k % group_size or group_size != 64:
        raise ValueError("group_size must be 64 and divide the input dimension")
    g = w.float().view(n, k // group_size, group_size)
    lo = g.amin(-1, keepdim=True)
    hi = g.amax(-1, keepdim=True)
    scale = ((hi - lo) / 15.0).clamp_min(1e-8)
    q = torch.round((g - lo) / scale).clamp_(0, 15).to(torch.int64).view(n, k // 8, 8)
    shifts = (torch.arange(8, device=w.device, dtype=torch.int64) * 4)
    words = (q << shifts).sum(-1)  # < 2^32
    packed = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)
    return Q4Tensor(packed.contiguous(), scale.view(n, -1).to(torch.bfloat16).contiguous(),
                    lo.view(n, -1).to(torch.bfloat16).contiguous(), group_size)


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
    # 4-bit tied LM head (quantize_model quantizes the embedding too); `embed`
    # then holds its dequantized rows, the table input tokens are looked up in
    embed_q4: Q4Tensor | None = None

    @property
    def device(self) -> torch.device:
        return self.embed.device

    @property
    def quant_bits(self) -> int:
        return 4 if isinstance(self.qkv[0], Q4Tensor) else 16

    def nbytes(self) -> int:
        ts = [self.embed, self.final_norm] + ([self.embed_q4] if self.embed_q4 is not None else [])
        for name in ("input_norm", "qkv", "q_norm", "k_norm", "o_proj", "post_norm", "gate_up", "down"):
            ts += getattr(self, name)
        return sum(tensor_bytes(t) for t in ts)

    def streamed_bytes(self) -> int:
        """Bytes one verify forward must read: embedding (tied LM head) + the
        four projections of every layer (norm vectors are negligible)."""
        head = self.embed_q4 if self.embed_q4 is not None else self.embed
        ts = [head, *self.qkv, *self.o_proj, *self.gate_up, *self.down]
        return sum(tensor_bytes(t) for t in ts)

    def reference_weights(self, layer: int) -> dict:
        """mlx-lm Qwen3 names for one layer (views / splits of the packed
        storage; ``Q4Tensor`` row slices when quantized)."""
        c = self.cfg
        qkv = self.qkv[layer]
        gate, up = split_gate_up(self.gate_up[layer])
        rows = (lambda t, sl: t.rows(sl)) if isinstance(qkv, Q4Tensor) else (lambda t, sl: t[sl])
        return {
            "input_layernorm": self.input_norm[layer],
            "q_proj": rows(qkv, slice(0, c.q_dim)),
            "k_proj": rows(qkv, slice(c.q_dim, c.q_dim + c.kv_dim)),
            "v_proj": rows(qkv, slice(c.q_dim + c.kv_dim, None)),
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
        if self.embed_q4 is not None:
            w.embed_q4 = mv(self.embed_q4)
        return w


def quantize_weights(w: Qwen3Weights, bits: int = 4, group_size: int = 64, embedding: bool = False) -> Qwen3Weights:
    """4-bit affine (MLX layout) q/k/v, o, gate/up and down projections of
    every layer; norms are kept.  ``embedding=False`` keeps the embedding
    (and with it the tied LM head) bf16: the BASELINE config-3 target ("all
    linear layers except embeddings").  ``embedding=True`` is the target
    after the reference's ``quantize_model(model, bits, group_size)``
    (dtree_mlx/api.py:46-54): mlx-lm quantizes every module with
    ``to_quantized``, ``nn.Embedding`` included, so the tied LM head becomes a
    4-bit matmul (``as_linear``, adapters.py:491) and the lookup table holds
    the dequantized rows."""
    if bits != 4 or group_size != 64:
        raise NotImplementedError("only 4-bit affine weights with group_size 64 are supported")
    if embedding:
        from .weights_io import dequantize_q4

        emb_q = quantize_affine_q4(w.embed, group_size)
        emb = dequantize_q4(emb_q)
    else:
        emb_q, emb = w.embed_q4, w.embed
    q = Qwen3Weights(w.cfg, emb, w.final_norm, list(w.input_norm), [], list(w.q_norm),
                     list(w.k_norm), [], list(w.post_norm), [], [], embed_q4=emb_q)
    for name in ("qkv", "o_proj", "gate_up", "down"):
        setattr(q, name, [quantize_affine_q4(t, group_size) for t in getattr(w, name)])
    return q


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


# ------------------------------------------------------------ Qwen3.5 hybrid
@dataclass
class Qwen35Weights:
    """Seeded random-init Qwen3.5 hybrid in the engine's layouts.

    DeltaNet layer: ``in_proj`` = rows in_proj_qkv | in_proj_z | in_proj_b |
    in_proj_a (one GEMM), ``conv_weight`` [kernel, conv_dim] (the reference's
    conv1d.weight[:, :, 0].T, qwen35_tree.py:389), ``norm`` (RMSNormGated),
    ``out_proj``.  Attention layer: ``qkv`` = q_proj rows (per head [q | gate])
    | k_proj | v_proj.  ``a_log`` f32 [n_linear, Hv], ``dt_bias`` [n_linear, Hv].
    Linear and embedding weights N(0, 0.02); conv weights U(-0.5, 0.5) (MLX
    Conv1d's default scale for a depthwise width-4 kernel); A = U(0, 16),
    A_log = log A and dt_bias = 1 as GatedDeltaNet initializes them
    (custom_qwen35_model.py:812-815); norm weights 1 (or 1 + N(0, jitter))."""

    cfg: "object"
    embed: torch.Tensor
    final_norm: torch.Tensor
    layers: list = field(default_factory=list)
    a_log: torch.Tensor | None = None
    dt_bias: torch.Tensor | None = None

    @property
    def device(self) -> torch.device:
        return self.embed.device

    def streamed_bytes(self) -> int:
        """Weights one verify forward reads (embedding = tied LM head once)."""
        n = tensor_bytes(self.embed)
        for L in self.layers:
            for k in ("in_proj", "out_proj", "qkv", "o_proj", "gate_up", "down", "conv_weight"):
                if k in L:
                    n += tensor_bytes(L[k])
        return n

    def reference_layer(self, l: int) -> dict:
        """mlx-lm names of layer l (views of the packed storage)."""
        c = self.cfg
        L = self.layers[l]
        gate, up = split_gate_up(L["gate_up"])
        out = {"input_layernorm": L["input_norm"], "post_attention_layernorm": L["post_norm"],
               "gate_proj": gate, "up_proj": up, "down_proj": L["down"]}
        if c.is_linear(l):
            li = sum(1 for j in range(l) if c.is_linear(j))
            w = L["in_proj"]
            kd, vd, hv = c.key_dim, c.value_dim, c.linear_num_value_heads
            out.update(in_proj_qkv=w[: c.conv_dim], in_proj_z=w[c.conv_dim : c.conv_dim + vd],
                       in_proj_b=w[c.conv_dim + vd : c.conv_dim + vd + hv],
                       in_proj_a=w[c.conv_dim + vd + hv :], conv_weight=L["conv_weight"], norm=L["norm"],
                       out_proj=L["out_proj"], A_log=self.a_log[li], dt_bias=self.dt_bias[li])
            del kd
        else:
            w = L["qkv"]
            out.update(q_proj=w[: 2 * c.q_dim], k_proj=w[2 * c.q_dim : 2 * c.q_dim + c.kv_dim],
                       v_proj=w[2 * c.q_dim + c.kv_dim :], q_norm=L["q_norm"], k_norm=L["k_norm"],
                       o_proj=L["o_proj"])
        return out

    def to(self, device) -> "Qwen35Weights":
        w = Qwen35Weights(self.cfg, self.embed.to(device), self.final_norm.to(device),
                          a_log=self.a_log.to(device), dt_bias=self.dt_bias.to(device))
        w.layers = [{k: v.to(device) for k, v in L.items()} for L in self.layers]
        return w


def random_qwen35_weights(cfg, seed: int = 0, device="cuda", dtype=torch.bfloat16,
                          norm_jitter: float = 0.0) -> Qwen35Weights:
    g = torch.Generator(device=device).manual_seed(int(seed))

    def randn(*shape):
        return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * STD).to(dtype)

    def uniform(lo, hi, *shape):
        return (torch.rand(*shape, generator=g, device=device, dtype=torch.float32) * (hi - lo) + lo)

    def ones(n):
        if norm_jitter > 0:
            return (1.0 + torch.randn(n, generator=g, device=device) * norm_jitter).to(dtype)
        return torch.ones(n, dtype=dtype, device=device)

    h, f = cfg.hidden_size, cfg.intermediate_size
    w = Qwen35Weights(cfg, embed=randn(cfg.vocab_size, h), final_norm=ones(h))
    a_log, dt_bias = [], []
    for l in range(cfg.num_hidden_layers):
        L = {"input_norm": ones(h), "post_norm": ones(h)}
        if cfg.is_linear(l):
            hv = cfg.linear_num_value_heads
            L["in_proj"] = torch.cat([randn(cfg.conv_dim, h), randn(cfg.value_dim, h), randn(hv, h),
                                      randn(hv, h)], dim=0).contiguous()
            L["conv_weight"] = uniform(-0.5, 0.5, cfg.linear_conv_kernel_dim, cfg.conv_dim).to(dtype)
            L["norm"] = ones(cfg.linear_value_head_dim)
            L["out_proj"] = randn(h, cfg.value_dim)
            a_log.append(torch.log(uniform(0.0, 16.0, hv).clamp_min(1e-3)))
            dt_bias.append(torch.ones(hv, dtype=dtype, device=device))
        else:
            L["qkv"] = torch.cat([randn(2 * cfg.q_dim, h), randn(cfg.kv_dim, h), randn(cfg.kv_dim, h)],
                                 dim=0).contiguous()
            L["q_norm"] = ones(cfg.head_dim)
            L["k_norm"] = ones(cfg.head_dim)
            L["o_proj"] = randn(h, cfg.q_dim)
        L["gate_up"] = interleave_gate_up(randn(f, h), randn(f, h))
        L["down"] = randn(h, f)
        w.layers.append(L)
    w.a_log = torch.stack(a_log).float().contiguous()
    w.dt_bias = torch.stack(dt_bias).contiguous()
    return w
