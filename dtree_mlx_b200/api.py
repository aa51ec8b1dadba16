"""Public API (dtree_mlx/api.py): ``DFlashGenerator`` with the same
constructor and ``generate`` / ``generate_from_tokens`` keyword arguments."""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch

from .adapters import LoadedTargetModel, load_target_model, quantize_target_model
from .draft import load_draft_model
from .dtree_runtime import dtree_generate
from .runtime import dflash_generate

DEFAULT_TARGET_MODEL = "synthetic:qwen3-4b"
DEFAULT_DRAFT_MODEL = "planted:p=0.85:seed=0"


@dataclass
class DFlashResult:
    text: str
    output_tokens: list[int]
    generated_tokens: list[int]
    metrics: dict[str, Any]


class DFlashGenerator:
    """api.py:29-166.  ``target_quant_bits=4`` (group size 64) quantizes the
    target's projections to MLX affine 4-bit (api.py:46-54) and the verify
    GEMMs dequantize them on the fly; other bit widths and a trained,
    quantized drafter raise NotImplementedError."""

    def __init__(
        self,
        target_model: str = DEFAULT_TARGET_MODEL,
        draft_model: str = DEFAULT_DRAFT_MODEL,
        draft_attention_mask: str = "auto",
        target_quant_bits: int | None = None,
        target_quant_group_size: int = 64,
        draft_quant_bits: int | None = None,
        draft_quant_group_size: int = 64,
        seed: int = 0,
    ):
        torch.manual_seed(seed)
        self.requested_target_model = target_model
        self.requested_draft_model = draft_model
        if target_quant_bits is not None and (target_quant_bits != 4 or target_quant_group_size != 64):
            raise NotImplementedError("target quantization: only bits=4 with group_size=64 is supported")
        if draft_quant_bits is not None:
            raise NotImplementedError("draft_quant_bits: the trained drafter is not available")
        self.target: LoadedTargetModel = load_target_model(target_model)
        self.target_quantization = None
        if target_quant_bits is not None:
            self.target_quantization = quantize_target_model(self.target, target_quant_bits, target_quant_group_size)
        self.draft, self.draft_path = load_draft_model(draft_model, target=self.target)
        self.draft_attention_mask = "none" if draft_attention_mask == "auto" else draft_attention_mask
        if hasattr(self.draft, "cache_mode"):
            # api.py:62-64: the drafter keeps a context-only cache for Qwen3.5 targets
            self.draft.cache_mode = "context-only" if self.target.adapter.family == "qwen3_5" else "kv"
        self.draft_quantization = None
        del target_quant_group_size, draft_quant_group_size

    @classmethod
    def from_components(cls, target: LoadedTargetModel, draft) -> "DFlashGenerator":
        """Wrap an already loaded target and drafter (shares their device state)."""
        self = cls.__new__(cls)
        self.requested_target_model = target.requested_model
        self.requested_draft_model = type(draft).__name__
        self.target = target
        self.target_quantization = None
        self.draft, self.draft_path = draft, None
        self.draft_attention_mask = "none"
        self.draft_quantization = None
        return self

    @property
    def target_model_path(self) -> Path:
        return self.target.resolved_model_path

    def encode_prompt(self, prompt_text: str):
        return self.target.build_prompt(prompt_text)

    def generate_from_tokens(
        self,
        prompt_tokens,
        max_new_tokens: int = 256,
        temperature: float = 0.0,
        speculative_tokens: int | None = None,
        decode_mode: str = "dflash",
        tree_budget: int | None = None,
        verify_mode: str = "parallel-replay",
        verify_chunk_size: int = 4,
        reset_peak_memory: bool = True,
        skip_special_tokens: bool = False,
        profile: bool = False,
    ) -> DFlashResult:
        if reset_peak_memory:
            torch.cuda.reset_peak_memory_stats()
        layer_ids = list(getattr(self.draft, "target_layer_ids", []))
        if decode_mode == "dflash":
            output_tokens, metrics = dflash_generate(
                target=self.target, draft=self.draft, prompt_tokens=prompt_tokens, max_new_tokens=max_new_tokens,
                temperature=temperature, stop_token_ids=self.target.stop_token_ids(), layer_ids=layer_ids,
                speculative_tokens=speculative_tokens, verify_mode=verify_mode,
                verify_chunk_size=verify_chunk_size, profile=profile,
            )
        elif decode_mode == "dtree":
            output_tokens, metrics = dtree_generate(
                target=self.target, draft=self.draft, prompt_tokens=prompt_tokens, max_new_tokens=max_new_tokens,
                temperature=temperature, stop_token_ids=self.target.stop_token_ids(), layer_ids=layer_ids,
                speculative_tokens=speculative_tokens, tree_budget=tree_budget, verify_mode=verify_mode,
                profile=profile,
            )
        else:
            raise ValueError(f"Unknown decode_mode={decode_mode!r}. Expected 'dflash' or 'dtree'.")
        generated_tokens = output_tokens[metrics["num_input_tokens"]:]
        text = self.target.tokenizer.decode(generated_tokens, skip_special_tokens=skip_special_tokens)
        return DFlashResult(text=text, output_tokens=output_tokens, generated_tokens=generated_tokens,
                            metrics=metrics)

    def generate(self, prompt_text: str, max_new_tokens: int = 256, temperature: float = 0.0,
                 speculative_tokens: int | None = None, decode_mode: str = "dflash", tree_budget: int | None = None,
                 verify_mode: str = "parallel-replay", verify_chunk_size: int = 4, reset_peak_memory: bool = True,
                 skip_special_tokens: bool = False, profile: bool = False) -> DFlashResult:
        return self.generate_from_tokens(
            prompt_tokens=self.encode_prompt(prompt_text), max_new_tokens=max_new_tokens, temperature=temperature,
            speculative_tokens=speculative_tokens, decode_mode=decode_mode, tree_budget=tree_budget,
            verify_mode=verify_mode, verify_chunk_size=verify_chunk_size, reset_peak_memory=reset_peak_memory,
            skip_special_tokens=skip_special_tokens, profile=profile,
        )


# Forward-looking alias (api.py:170).
Generator = DFlashGenerator
