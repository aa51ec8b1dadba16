"""Target adapters: the plugin interface the verify path sits behind.

Mirrors dtree_mlx/adapters.py: ``MLXTargetAdapter`` (:88-213) becomes
``TargetAdapter`` with the same method names and argument meaning,
``Qwen3TargetAdapter`` (:451-668) runs on the B200 engine, the registry
(:671-678), ``LoadedTargetModel`` (:681-819) and ``load_target_model``
(:822-846) keep their shapes.  Tensors are torch CUDA tensors instead of
``mx.array``.  Unsupported families raise ``NotImplementedError`` as in the
reference.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import numpy as np
import torch

from . import kernels
from .config import PRESETS, QWEN35_PRESETS, Qwen3Config
from .engine import Qwen3Engine, chain_anc_masks, mask_to_anc, pad_rows
from .synthetic import Qwen3Weights, random_qwen3_weights


@dataclass
class SyntheticQwen3:
    """A random-init Qwen3 target resident on one GPU."""

    cfg: Qwen3Config
    weights: Qwen3Weights
    kv_capacity: int
    seed: int
    engines: dict = field(default_factory=dict)

    @property
    def args(self):
        return self.cfg


class LayerKVCache:
    """Per-layer view of the engine's KV cache (mlx_lm KVCache surface:
    keys/values [1, kv_heads, capacity, head_dim], offset, trim)."""

    def __init__(self, seq: "SequenceCache", layer: int):
        self.seq = seq
        self.layer = layer

    @property
    def keys(self):
        return self.seq.engine.kv_cache[self.layer, 0][None]

    @property
    def values(self):
        return self.seq.engine.kv_cache[self.layer, 1][None]

    @property
    def offset(self) -> int:
        return self.seq.offset

    @offset.setter
    def offset(self, v: int) -> None:
        self.seq.offset = int(v)

    def trim(self, n: int) -> int:
        n = min(self.seq.offset, int(n))
        self.seq.offset -= n
        return n


class SequenceCache(list):
    """List of LayerKVCache sharing one offset (all layers advance together)."""

    def __init__(self, engine: Qwen3Engine):
        self.engine = engine
        self.offset = 0
        super().__init__(LayerKVCache(self, i) for i in range(engine.cfg.num_hidden_layers))


class TargetAdapter:
    """Plugin interface (adapters.py:88-213)."""

    family: str = "unknown"

    def resolve_target_model_path(self, path_or_repo: str) -> Path:
        return Path(path_or_repo)

    def build_prompt(self, tokenizer, prompt_text: str):
        raise NotImplementedError

    def stop_token_ids(self, tokenizer) -> set[int]:
        raise NotImplementedError

    def make_cache(self, model, speculative_linear_cache: bool = False):
        raise NotImplementedError

    def embed_tokens(self, model, tokens):
        raise NotImplementedError

    def lm_head_logits(self, model, hidden_states):
        raise NotImplementedError

    def lm_head_argmax(self, model, hidden_states):
        logits = self.lm_head_logits(model, hidden_states)
        return torch.argmax(logits.float(), dim=-1).to(torch.int32)

    def forward_with_hidden_states(self, model, inputs, cache, layer_ids, return_rollback_records: bool = False):
        raise NotImplementedError

    def forward_verifier_states(self, model, inputs, cache, layer_ids):
        raise NotImplementedError(f"{self.family} does not expose verifier states before the LM head.")

    def supports_tree_verification(self) -> bool:
        return False

    def forward_tree_with_hidden_states(self, model, inputs, cache, layer_ids, parents, position_ids,
                                        attention_mask):
        raise NotImplementedError(f"{self.family} does not expose explicit tree verification.")

    def rewind_kv_caches(self, cache, num_tokens: int) -> None:
        raise NotImplementedError

    def cache_summary(self, cache, offset: int | None = None) -> str:
        raise NotImplementedError

    def compact_kv_caches(self, model, cache, past_length: int, keep_current_indices: list[int]) -> None:
        raise NotImplementedError(f"{self.family} does not implement DTree cache compaction.")

    # linear (recurrent) caches: only hybrid targets have them (adapters.py:174-197)
    def snapshot_linear_caches(self, model, cache):
        return {}

    def restore_linear_caches(self, model, cache, snapshots) -> None:
        return None

    def rollback_linear_caches(self, model, cache, rollback_records, accepted_inputs: int) -> None:
        return None


class Qwen3TargetAdapter(TargetAdapter):
    """Qwen3 on the B200 engine (adapters.py:451-668)."""

    family = "qwen3"

    def __init__(self) -> None:
        self.last_session = None

    # -- engine ------------------------------------------------------------
    def engine(self, model: SyntheticQwen3, draft=None, layer_ids=None) -> Qwen3Engine:
        ids = tuple(sorted(layer_ids if layer_ids is not None else getattr(draft, "target_layer_ids", []) or []))
        eng = model.engines.get(ids)
        if eng is None:
            # one engine (KV cache + scratch) per capture-layer set
            for old in list(model.engines.values()):
                old.close()
            model.engines.clear()
            eng = Qwen3Engine(model.weights, model.kv_capacity, layer_ids=ids)
            model.engines[ids] = eng
        return eng

    # -- prompt / tokens ---------------------------------------------------
    def build_prompt(self, tokenizer, prompt_text: str):
        return torch.tensor(tokenizer.encode(prompt_text), dtype=torch.int32)

    def stop_token_ids(self, tokenizer) -> set[int]:
        return set(getattr(tokenizer, "eos_token_ids", set()))

    def make_cache(self, model, speculative_linear_cache: bool = False):
        del speculative_linear_cache
        return SequenceCache(self.engine(model))

    def embed_tokens(self, model, tokens):
        return model.weights.embed[tokens.to(model.weights.device).long()]

    # -- LM head -------------------------------------------------------------
    def _rows(self, hidden_states):
        h = hidden_states.reshape(-1, hidden_states.shape[-1]).to(torch.bfloat16)
        n = h.shape[0]
        tp = pad_rows(min(n, 128)) if n <= 128 else 128
        return h, n, tp

    def lm_head_logits(self, model, hidden_states):
        """Tied LM head (adapters.py:489-492) with the tcgen05 GEMM, bf16 logits."""
        h, n, _ = self._rows(hidden_states)
        out = []
        for s in range(0, n, 128):
            blk = h[s : s + 128]
            tp = pad_rows(blk.shape[0])
            x = torch.zeros(tp, h.shape[1], dtype=torch.bfloat16, device=h.device)
            x[: blk.shape[0]] = blk
            out.append(kernels.linear_bf16(x, model.weights.embed)[: blk.shape[0]])
        return torch.cat(out, 0).reshape(*hidden_states.shape[:-1], -1)

    def lm_head_argmax(self, model, hidden_states):
        """Fused LM head + argmax (adapters.py:114-118), first index on ties."""
        h, n, _ = self._rows(hidden_states)
        res = []
        for s in range(0, n, 128):
            blk = h[s : s + 128]
            tp = pad_rows(blk.shape[0])
            x = torch.zeros(tp, h.shape[1], dtype=torch.bfloat16, device=h.device)
            x[: blk.shape[0]] = blk
            res.append(kernels.lm_head_argmax(x, model.weights.embed, blk.shape[0]))
        return torch.cat(res).reshape(hidden_states.shape[:-1])

    # -- forwards -------------------------------------------------------------
    def _forward(self, model, tokens: list[int], cache: SequenceCache, layer_ids, anc_rows=None,
                 positions=None):
        eng = self.engine(model, layer_ids=layer_ids)
        if cache.engine is not eng:
            raise ValueError("cache belongs to a different engine (capture layers changed)")
        dev = eng.device
        n = len(tokens)
        state = kernels.new_state(dev, start=cache.offset)
        post = torch.zeros(128, dtype=torch.int32, device=dev)
        norm_rows, cap_rows = [], []
        s = 0
        if anc_rows is None and positions is None and n > eng.t_cap and n >= eng.dense_prefill_min_rows:
            # a causal sequence longer than one verify forward: dense prefill
            width = eng.cfg.hidden_size * max(1, len(eng.layer_ids))
            norm = torch.zeros(n, eng.cfg.hidden_size, dtype=torch.bfloat16, device=dev)
            hid = torch.zeros(n, width, dtype=torch.bfloat16, device=dev)
            nxt = torch.zeros(1, dtype=torch.int32, device=dev)
            toks_all = torch.tensor(tokens, dtype=torch.int32, device=dev)
            while s < n:
                t = min(eng.max_prefill_rows, n - s)
                state[0] = cache.offset + s
                eng.prefill_dense(toks_all[s:s + t], state, hid[s:s + t] if eng.layer_ids else None, nxt,
                                  norm_out=norm[s:s + t])
                s += t
            cache.offset += n
            return norm[None], (hid if eng.layer_ids else hid[..., :0])[None]
        while s < n:
            t = min(eng.t_cap, n - s)
            state[0] = cache.offset + s
            toks = torch.tensor(tokens[s : s + t], dtype=torch.int32, device=dev)
            pos = (torch.tensor(positions[s : s + t], dtype=torch.int32, device=dev) if positions is not None
                   else torch.arange(cache.offset + s, cache.offset + s + t, dtype=torch.int32, device=dev))
            anc = anc_rows if anc_rows is not None else chain_anc_masks(t)
            anc_t = torch.from_numpy(np.ascontiguousarray(anc).view(np.int64)).to(dev)
            eng.forward_tree(toks, pos, anc_t, t, state, post)
            norm_rows.append(eng.norm_out[:t].clone())
            cap_rows.append(eng.capture[:t, : eng.cfg.hidden_size * max(1, len(eng.layer_ids))].clone())
            s += t
        cache.offset += n
        norm = torch.cat(norm_rows)[None]
        hid = torch.cat(cap_rows)[None]
        if not eng.layer_ids:
            hid = hid[..., :0]
        return norm, hid

    def forward_with_hidden_states(self, model, inputs, cache, layer_ids, return_rollback_records: bool = False):
        """adapters.py:516-533: causal forward, full logits."""
        norm, hid = self._forward(model, [int(t) for t in inputs.reshape(-1).tolist()], cache, layer_ids)
        logits = self.lm_head_logits(model, norm)
        return (logits, hid, {}) if return_rollback_records else (logits, hid)

    def forward_verifier_states(self, model, inputs, cache, layer_ids):
        norm, hid = self._forward(model, [int(t) for t in inputs.reshape(-1).tolist()], cache, layer_ids)
        return norm, hid, {}

    def supports_tree_verification(self) -> bool:
        return True

    def forward_tree_with_hidden_states(self, model, inputs, cache, layer_ids, parents, position_ids,
                                        attention_mask):
        """adapters.py:568-597: tree rows with per-node positions and the bool
        mask [T, P+T] (prefix columns must be all True)."""
        del parents
        tokens = [int(t) for t in inputs.reshape(-1).tolist()]
        n = len(tokens)
        if n > 128:
            raise ValueError("at most 128 tree rows per verify")
        mask = torch.as_tensor(attention_mask).bool().cpu().numpy()
        past = cache.offset
        if mask.shape != (n, past + n) or not mask[:, :past].all():
            raise ValueError("attention_mask must be [T, P+T] with an all-visible prefix")
        anc = mask_to_anc(mask[:, past:])
        pos = [int(p) for p in torch.as_tensor(position_ids).reshape(-1).tolist()]
        return self._forward(model, tokens, cache, layer_ids, anc_rows=anc, positions=pos)

    def rewind_kv_caches(self, cache, num_tokens: int) -> None:
        cache.offset = max(0, cache.offset - int(num_tokens))

    def cache_summary(self, cache, offset: int | None = None) -> str:
        off = cache.offset if offset is None and hasattr(cache, "offset") else offset
        return " ".join(f"{i}:kv={off}" for i in range(len(cache)))

    def compact_kv_caches(self, model, cache, past_length: int, keep_current_indices: list[int]) -> None:
        """adapters.py:635-668 via dtree_kv_compact (all layers in one launch)."""
        keep = [int(i) for i in keep_current_indices]
        cur = cache.offset - past_length
        if cur <= 0:
            return
        if not keep:
            cache.offset = past_length
            return
        if len(keep) == cur:
            return
        eng = cache.engine
        dev = eng.device
        state = kernels.new_state(dev, start=past_length)
        state[3] = len(keep)
        acc = torch.zeros(128, dtype=torch.int32, device=dev)
        acc[: len(keep)] = torch.tensor(keep, dtype=torch.int32)
        kernels.kv_compact(eng.kv_cache, acc, state)
        cache.offset = past_length + len(keep)


class Qwen35TargetAdapter(Qwen3TargetAdapter):
    """Qwen3.5 hybrid (gated DeltaNet + gated attention) on the B200 engine
    (adapters.py:216-450).  Tree verification keeps the per-layer DeltaNet
    inputs on the device in place of the reference's pending per-node state
    (``_pending_tree_state``, :430); ``compact_kv_caches`` commits the
    accepted path from them (commit_qwen35_tree_path, qwen35_tree.py:708-732)."""

    family = "qwen3_5"

    def __init__(self) -> None:
        super().__init__()
        self._pending = None

    def engine(self, model, draft=None, layer_ids=None):
        from .engine35 import Qwen35Engine

        ids = tuple(sorted(layer_ids if layer_ids is not None else getattr(draft, "target_layer_ids", []) or []))
        eng = model.engines.get(ids)
        if eng is None:
            for old in list(model.engines.values()):
                old.close()
            model.engines.clear()
            eng = Qwen35Engine(model.weights, model.kv_capacity, layer_ids=ids)
            model.engines[ids] = eng
        return eng

    def make_cache(self, model, speculative_linear_cache: bool = False):
        """A new sequence: zero conv / recurrent states and an empty KV prefix."""
        cache = super().make_cache(model, speculative_linear_cache)
        cache.engine.reset_states()
        return cache

    def _forward(self, model, tokens, cache, layer_ids, anc_rows=None, positions=None, parents=None):
        eng = self.engine(model, layer_ids=layer_ids)
        if cache.engine is not eng:
            raise ValueError("cache belongs to a different engine (capture layers changed)")
        dev = eng.device
        n = len(tokens)
        state = kernels.new_state(dev, start=cache.offset)
        post = torch.zeros(128, dtype=torch.int32, device=dev)
        toks = torch.tensor(tokens, dtype=torch.int32, device=dev)
        if parents is not None:  # tree verify: one forward, states stay committed
            if n > eng.t_cap:
                raise ValueError("at most 128 tree rows per verify")
            pos = torch.tensor(positions, dtype=torch.int32, device=dev)
            par = torch.tensor(parents, dtype=torch.int32, device=dev)
            anc_t = torch.from_numpy(np.ascontiguousarray(anc_rows).view(np.int64)).to(dev)
            eng.forward(toks, pos, par, anc_t, n, state, post, mode=0)
            self._pending = (cache.offset, par)
            cache.offset += n
            norm = eng.norm_out[:n].clone()[None]
            hid = eng.capture[:n].clone()[None]
        elif n > eng.t_cap and n >= eng.dense_prefill_min_rows:  # a long causal sequence: dense prefill
            width = eng.cfg.hidden_size * max(1, len(eng.layer_ids))
            norm = torch.zeros(n, eng.cfg.hidden_size, dtype=torch.bfloat16, device=dev)
            hid = torch.zeros(n, width, dtype=torch.bfloat16, device=dev)
            nxt = torch.zeros(1, dtype=torch.int32, device=dev)
            s = 0
            while s < n:
                t = min(eng.max_prefill_rows, n - s)
                state[0] = cache.offset + s
                eng.prefill_dense(toks[s:s + t], state, hid[s:s + t] if eng.layer_ids else None, nxt,
                                  norm_out=norm[s:s + t])
                s += t
            cache.offset += n
            norm, hid = norm[None], hid[None]
        else:  # causal sequence: states advance chunk by chunk
            norm_rows, cap_rows = [], []
            s = 0
            while s < n:
                t = min(eng.t_cap, n - s)
                state[0] = cache.offset + s
                pos = torch.arange(cache.offset + s, cache.offset + s + t, dtype=torch.int32, device=dev)
                anc_t = torch.from_numpy(chain_anc_masks(t).view(np.int64)).to(dev)
                eng.prefill_chunk(toks[s:s + t].contiguous(), pos, anc_t, t, state, post)
                norm_rows.append(eng.norm_out[:t].clone())
                cap_rows.append(eng.capture[:t].clone())
                s += t
            cache.offset += n
            norm, hid = torch.cat(norm_rows)[None], torch.cat(cap_rows)[None]
        if not eng.layer_ids:
            hid = hid[..., :0]
        return norm, hid

    # -- linear-cache rollback (adapters.py:350-388; RecurrentRollbackCache,
    # qwen35_target.py:23-175; rollback_linear_caches, custom_qwen35_model.py:
    # 1124-1169).  The device decode loop never needs it: its verify keeps the
    # committed DeltaNet state and replays the accepted path on commit.  These
    # methods give host callers of the adapter interface the reference's
    # snapshot / rollback contract on the same engine.
    def forward_with_hidden_states(self, model, inputs, cache, layer_ids, return_rollback_records: bool = False):
        """Causal forward (states advance through every token); with
        ``return_rollback_records`` the pre-forward DeltaNet states and the
        tokens are recorded so rollback_linear_caches can keep a prefix."""
        tokens = [int(t) for t in inputs.reshape(-1).tolist()]
        records = {}
        if return_rollback_records:
            eng = self.engine(model, layer_ids=layer_ids)
            records = {"snapshot": eng.snapshot_states(), "past": cache.offset, "tokens": tokens}
        norm, hid = self._forward(model, tokens, cache, layer_ids)
        logits = self.lm_head_logits(model, norm)
        return (logits, hid, records) if return_rollback_records else (logits, hid)

    def snapshot_linear_caches(self, model, cache):
        return cache.engine.snapshot_states()

    def restore_linear_caches(self, model, cache, snapshots) -> None:
        cache.engine.restore_states(snapshots)

    def rollback_linear_caches(self, model, cache, rollback_records, accepted_inputs: int) -> None:
        """Keep the first ``accepted_inputs`` tokens of the recorded forward:
        restore the recorded DeltaNet states and advance them through those
        tokens again (the K/V rows they rewrite are identical)."""
        if not rollback_records:
            return
        eng = cache.engine
        eng.restore_states(rollback_records["snapshot"])
        keep = int(accepted_inputs)
        if keep > 0:
            offset = cache.offset
            cache.offset = rollback_records["past"]
            self._forward(model, rollback_records["tokens"][:keep], cache, list(eng.layer_ids))
            cache.offset = max(offset, rollback_records["past"] + keep)

    def forward_tree_with_hidden_states(self, model, inputs, cache, layer_ids, parents, position_ids,
                                        attention_mask):
        """adapters.py:410-430 (forward_qwen35_tree_with_hidden_states)."""
        tokens = [int(t) for t in inputs.reshape(-1).tolist()]
        n = len(tokens)
        par = [int(p) for p in parents]
        if len(par) != n or par[0] != -1 or any(not (0 <= p < i) for i, p in enumerate(par) if i > 0):
            raise ValueError("parents must list a tree in topological order with the root first")
        mask = torch.as_tensor(attention_mask).bool().cpu().numpy()
        past = cache.offset
        if mask.shape != (n, past + n) or not mask[:, :past].all():
            raise ValueError("attention_mask must be [T, P+T] with an all-visible prefix")
        pos = [int(p) for p in torch.as_tensor(position_ids).reshape(-1).tolist()]
        return self._forward(model, tokens, cache, layer_ids, anc_rows=mask_to_anc(mask[:, past:]), positions=pos,
                             parents=par)

    def compact_kv_caches(self, model, cache, past_length: int, keep_current_indices: list[int]) -> None:
        """adapters.py:432-448: commit the accepted path of the last tree verify."""
        if self._pending is None:
            raise RuntimeError("Qwen3.5 tree compaction requires pending tree state.")
        keep = [int(i) for i in keep_current_indices]
        past, par = self._pending
        if past != past_length:
            raise ValueError("past_length does not match the pending tree verify")
        eng = cache.engine
        dev = eng.device
        state = kernels.new_state(dev, start=past_length)
        state[3] = len(keep)
        acc = torch.zeros(128, dtype=torch.int32, device=dev)
        acc[: len(keep)] = torch.tensor(keep, dtype=torch.int32)
        eng.commit(par, acc, state)
        cache.offset = past_length + len(keep)
        self._pending = None


ADAPTERS: dict[str, type[TargetAdapter]] = {
    "qwen3": Qwen3TargetAdapter,
    "qwen3_5": Qwen35TargetAdapter,
}


def adapter_for_model_type(model_type: str) -> type[TargetAdapter] | None:
    return ADAPTERS.get(model_type)


class ByteTokenizer:
    """Deterministic stand-in tokenizer for synthetic targets (no vocabulary
    files are available offline): UTF-8 bytes, no stop tokens."""

    eos_token_ids: set[int] = set()

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        return list(text.encode("utf-8"))

    def decode(self, tokens, skip_special_tokens: bool = False) -> str:
        return bytes(int(t) % 256 for t in tokens).decode("utf-8", errors="replace")


class Qwen35TextModel:
    """The text model of a Qwen3.5 target as lazy_follow_tree_exact reaches it
    (``target.model.model``; custom_qwen35_model.py ``forward_dflash``): a
    causal forward of the given tokens that appends their K/V and advances
    the DeltaNet conv / recurrent states, returning (norm_hidden,
    verifier_hidden) [1, n, ...]."""

    def __init__(self, adapter: "Qwen35TargetAdapter", container: SyntheticQwen3):
        self._adapter = adapter
        self._container = container

    def forward_dflash(self, inputs, cache, layer_ids):
        tokens = [int(t) for t in torch.as_tensor(inputs).reshape(-1).tolist()]
        return self._adapter._forward(self._container, tokens, cache, layer_ids)


@dataclass
class LoadedTargetModel:
    """adapters.py:681-819."""

    requested_model: str
    resolved_model_path: Path
    model: Any
    tokenizer: Any
    adapter: TargetAdapter

    def __post_init__(self):
        if isinstance(self.adapter, Qwen35TargetAdapter) and not hasattr(self.model, "model"):
            self.model.model = Qwen35TextModel(self.adapter, self.model)

    def build_prompt(self, prompt_text: str):
        return self.adapter.build_prompt(self.tokenizer, prompt_text)

    def stop_token_ids(self) -> set[int]:
        return self.adapter.stop_token_ids(self.tokenizer)

    def make_cache(self, speculative_linear_cache: bool = False):
        return self.adapter.make_cache(self.model, speculative_linear_cache=speculative_linear_cache)

    def embed_tokens(self, tokens):
        return self.adapter.embed_tokens(self.model, tokens)

    def lm_head_logits(self, hidden_states):
        return self.adapter.lm_head_logits(self.model, hidden_states)

    def lm_head_argmax(self, hidden_states):
        return self.adapter.lm_head_argmax(self.model, hidden_states)

    def forward_with_hidden_states(self, inputs, cache, layer_ids, return_rollback_records: bool = False):
        return self.adapter.forward_with_hidden_states(self.model, inputs, cache, layer_ids,
                                                       return_rollback_records=return_rollback_records)

    def forward_verifier_states(self, inputs, cache, layer_ids):
        return self.adapter.forward_verifier_states(self.model, inputs, cache, layer_ids)

    def supports_tree_verification(self) -> bool:
        return self.adapter.supports_tree_verification()

    def forward_tree_with_hidden_states(self, inputs, cache, layer_ids, parents, position_ids, attention_mask):
        return self.adapter.forward_tree_with_hidden_states(self.model, inputs, cache, layer_ids, parents,
                                                            position_ids, attention_mask)

    def rewind_kv_caches(self, cache, num_tokens: int) -> None:
        self.adapter.rewind_kv_caches(cache, num_tokens)

    def cache_summary(self, cache, offset: int | None = None) -> str:
        return self.adapter.cache_summary(cache, offset=offset)

    def compact_kv_caches(self, cache, past_length: int, keep_current_indices: list[int]) -> None:
        self.adapter.compact_kv_caches(self.model, cache, past_length, keep_current_indices)

    def snapshot_linear_caches(self, cache):
        return self.adapter.snapshot_linear_caches(self.model, cache)

    def restore_linear_caches(self, cache, snapshots) -> None:
        self.adapter.restore_linear_caches(self.model, cache, snapshots)

    def rollback_linear_caches(self, cache, rollback_records, accepted_inputs: int) -> None:
        self.adapter.rollback_linear_caches(self.model, cache, rollback_records, accepted_inputs)


def parse_synthetic_spec(spec: str) -> dict:
    """``synthetic:<preset>[:seed=N][:kv=N]`` -> settings."""
    parts = spec.split(":")
    if parts[0] != "synthetic" or len(parts) < 2:
        raise ValueError(f"not a synthetic model spec: {spec!r}")
    out = {"preset": parts[1], "seed": 0, "kv": 4096}
    for p in parts[2:]:
        k, v = p.split("=", 1)
        out[k] = int(v)
    return out


def quantize_target_model(target: "LoadedTargetModel", bits: int = 4, group_size: int = 64,
                          embedding: bool = True) -> dict:
    """``quantize_model`` on a loaded target (api.py:46-54): its projections
    and (``embedding``, as mlx-lm does) its embedding / tied LM head become
    MLX affine 4-bit; engines built for the bf16 weights are released.
    Returns the ``quantization`` config entry."""
    from .synthetic import Qwen35Weights, quantize_weights

    model = target.model
    if isinstance(model.weights, Qwen35Weights):
        raise NotImplementedError("4-bit weights are implemented for the Qwen3 target only")
    for eng in list(model.engines.values()):
        eng.close()
    model.engines.clear()
    model.weights = quantize_weights(model.weights, bits, group_size, embedding=embedding)
    torch.cuda.empty_cache()
    return {"group_size": group_size, "bits": bits}


def _tokenizer_for(path: Path):
    """The checkpoint's own tokenizer when its files are present (transformers,
    local files only); else the byte stand-in."""
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(str(path), local_files_only=True)
        eos = tok.eos_token_id
        tok.eos_token_ids = set(eos if isinstance(eos, list) else ([eos] if eos is not None else []))
        return tok
    except Exception:
        return ByteTokenizer()


def load_target_model(path_or_repo: str, device: str = "cuda", kv_capacity: int = 4096) -> LoadedTargetModel:
    """adapters.py:822-846.  ``path_or_repo`` is a checkpoint directory
    (config.json + model*.safetensors, MLX or Hugging Face layout: see
    ``weights_io``) or ``synthetic:<preset>[:seed=N][:kv=N]``, a seeded
    random-init target of a BASELINE shape (``qwen3-tiny``, ``qwen3-4b``,
    ``qwen35-tiny``, ``qwen35-9b``).  There is no hub download offline."""
    if not str(path_or_repo).startswith("synthetic:"):
        path = Path(path_or_repo)
        if not (path / "config.json").exists():
            raise NotImplementedError(
                f"Unsupported target {path_or_repo!r}: expected a local checkpoint directory with config.json "
                f"or 'synthetic:<preset>' with preset in {sorted(PRESETS) + sorted(QWEN35_PRESETS)}."
            )
        from .weights_io import load_target_weights

        model_type, weights = load_target_weights(path, device)
        adapter_cls = adapter_for_model_type(model_type)
        if adapter_cls is None:
            registered = ", ".join(sorted(ADAPTERS))
            raise NotImplementedError(f"Unsupported target model_type={model_type!r}. Current adapters: {registered}.")
        model = SyntheticQwen3(weights.cfg, weights, kv_capacity=int(kv_capacity), seed=0)
        return LoadedTargetModel(str(path_or_repo), path, model, _tokenizer_for(path), adapter_cls())
    spec = parse_synthetic_spec(path_or_repo)
    if spec["preset"] in QWEN35_PRESETS:
        from .synthetic import random_qwen35_weights

        cfg = QWEN35_PRESETS[spec["preset"]]
        weights = random_qwen35_weights(cfg, seed=spec["seed"], device=device)
        model = SyntheticQwen3(cfg, weights, kv_capacity=spec["kv"], seed=spec["seed"])
        return LoadedTargetModel(path_or_repo, Path(path_or_repo), model, ByteTokenizer(), Qwen35TargetAdapter())
    cfg = PRESETS.get(spec["preset"])
    if cfg is None:
        raise NotImplementedError(f"unknown synthetic preset {spec['preset']!r}")
    adapter_cls = adapter_for_model_type(cfg.model_type)
    if adapter_cls is None:
        raise NotImplementedError(f"Unsupported model_type={cfg.model_type!r}")
    weights = random_qwen3_weights(cfg, seed=spec["seed"], device=device)
    model = SyntheticQwen3(cfg, weights, kv_capacity=spec["kv"], seed=spec["seed"])
    return LoadedTargetModel(path_or_repo, Path(path_or_repo), model, ByteTokenizer(), adapter_cls())
