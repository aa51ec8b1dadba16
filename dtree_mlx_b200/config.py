"""Model shapes of the synthetic workloads.

Names follow mlx-lm's Qwen3 ``ModelArgs`` (hidden_size, num_hidden_layers,
...).  ``rms_norm_eps`` is Qwen3's 1e-6.
"""
from __future__ import annotations

from dataclasses import dataclass, asdict


@dataclass(frozen=True)
class Qwen3Config:
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = True
    model_type: str = "qwen3"

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def n_params(self) -> int:
        h, f = self.hidden_size, self.intermediate_size
        per_layer = (
            h * (self.q_dim + 2 * self.kv_dim)  # q k v
            + self.q_dim * h                     # o
            + 3 * h * f                          # gate up down
            + 2 * h + 2 * self.head_dim          # norms
        )
        return self.num_hidden_layers * per_layer + self.vocab_size * h + h

    def as_dict(self) -> dict:
        return asdict(self)


PRESETS: dict[str, Qwen3Config] = {
    # tiny Qwen3 (CPU plumbing case of the reference)
    "qwen3-tiny": Qwen3Config(
        hidden_size=512,
        num_hidden_layers=4,
        num_attention_heads=8,
        num_key_value_heads=4,
        head_dim=64,
        intermediate_size=1536,
        vocab_size=32768,
    ),
    # Qwen3-4B shape
    "qwen3-4b": Qwen3Config(
        hidden_size=2560,
        num_hidden_layers=36,
        num_attention_heads=32,
        num_key_value_heads=8,
        head_dim=128,
        intermediate_size=9728,
        vocab_size=151936,
    ),
}


def default_layer_ids(cfg: Qwen3Config, n: int = 5) -> list[int]:
    """Target layers whose hidden states feed the drafter (DFlash
    ``target_layer_ids``; the checkpoint's list is not available here, so
    ``n`` evenly spaced layers are used)."""
    L = cfg.num_hidden_layers
    n = min(n, L)
    if n == 1:
        return [L - 1]
    return sorted({round(1 + i * (L - 3) / (n - 1)) for i in range(n)})


@dataclass(frozen=True)
class Qwen35Config:
    """Qwen3.5 text model (dtree_mlx/custom_qwen35_model.py:716-774 TextModelArgs):
    gated DeltaNet layers, every ``full_attention_interval``-th layer a gated
    full-attention layer with partial RoPE."""

    hidden_size: int
    num_hidden_layers: int
    intermediate_size: int
    vocab_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int = 4
    full_attention_interval: int = 4
    rope_theta: float = 100_000.0
    partial_rotary_factor: float = 0.25
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = True
    model_type: str = "qwen3_5"

    def is_linear(self, layer: int) -> bool:
        return (layer + 1) % self.full_attention_interval != 0

    @property
    def key_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def value_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def n_linear(self) -> int:
        return sum(1 for l in range(self.num_hidden_layers) if self.is_linear(l))

    @property
    def n_attn(self) -> int:
        return self.num_hidden_layers - self.n_linear

    def as_dict(self) -> dict:
        return asdict(self)


QWEN35_PRESETS: dict[str, Qwen35Config] = {
    # Qwen3.5-9B-style hybrid (3 DeltaNet : 1 full attention)
    "qwen35-9b": Qwen35Config(
        hidden_size=4096,
        num_hidden_layers=32,
        intermediate_size=12288,
        vocab_size=248320,
        num_attention_heads=16,
        num_key_value_heads=4,
        head_dim=256,
        linear_num_key_heads=16,
        linear_num_value_heads=32,
        linear_key_head_dim=128,
        linear_value_head_dim=128,
    ),
    # small model of the same architecture for parity tests
    "qwen35-tiny": Qwen35Config(
        hidden_size=512,
        num_hidden_layers=4,
        intermediate_size=1024,
        vocab_size=8192,
        num_attention_heads=4,
        num_key_value_heads=2,
        head_dim=256,
        linear_num_key_heads=2,
        linear_num_value_heads=4,
        linear_key_head_dim=128,
        linear_value_head_dim=128,
    ),
}


@dataclass(frozen=True)
class DraftConfig:
    """DFlash block drafter (dtree_mlx/draft.py:26-70 DraftArgs): Qwen3 decoder
    layers over the target's hidden size, ``fc`` from the concatenated target
    hiddens of ``target_layer_ids``.  The trained checkpoints' configs are not
    available offline, so these shapes are chosen to match their targets."""

    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int
    target_layer_ids: tuple
    block_size: int = 16
    mask_token_id: int = 0
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim


DRAFT_PRESETS: dict[str, DraftConfig] = {
    # drafter for the Qwen3-4B-shaped target (5 target layers, 5 drafter layers)
    "qwen3-4b": DraftConfig(hidden_size=2560, num_hidden_layers=5, num_attention_heads=32, num_key_value_heads=8,
                            head_dim=128, intermediate_size=9728, vocab_size=151936,
                            target_layer_ids=(1, 9, 18, 26, 34), mask_token_id=151669),
    # small drafter for the tiny target of the parity tests
    "qwen3-tiny": DraftConfig(hidden_size=512, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=4,
                              head_dim=64, intermediate_size=1536, vocab_size=32768, target_layer_ids=(1, 3),
                              mask_token_id=32767),
}
