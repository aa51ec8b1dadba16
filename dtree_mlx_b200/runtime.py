"""Shared decode runtime: the generation loop of both decode modes.

Mirrors dtree_mlx/runtime.py (dflash_generate, :430-610) and
dtree_mlx/dtree_runtime.py (dtree_generate, :293-586): same arguments, same
validation errors, same output-token commit and stop/truncation rules, same
metrics keys.  The per-step work (draft, tree or chain build, tree-verify
forward with the fused LM-head argmax, acceptance walk, KV compaction, commit)
runs on the GPU as one CUDA graph per step; the host reads back the 32-byte
decode state once per step to drive the loop.
"""
from __future__ import annotations

import time
from typing import Any

import torch

from . import kernels
from .engine import DecodeSession, StepConfig, dtree_nodes

DTREE_STAGE_ORDER = (
    "draft_time_s",
    "tree_build_time_s",
    "tree_compile_time_s",
    "verify_time_s",
    "bookkeeping_time_s",
)


def sample_tokens(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    """runtime.py:12-19: argmax (first index on ties) below 1e-5, else categorical."""
    flat = logits.reshape(-1, logits.shape[-1]).float()
    if temperature < 1e-5:
        out = torch.argmax(flat, dim=-1)
    else:
        out = torch.multinomial(torch.softmax(flat / temperature, dim=-1), 1).squeeze(-1)
    return out.reshape(logits.shape[:-1]).to(torch.int32)


def longest_prefix_match(draft_tokens: list[int], verifier_tokens: list[int]) -> int:
    """runtime.py:33-39."""
    matched = 0
    for d, v in zip(draft_tokens, verifier_tokens):
        if d != v:
            break
        matched += 1
    return matched


def stop_position(tokens: list[int], start_idx: int, stop_token_ids: set[int]) -> int | None:
    """runtime.py:42-46."""
    for idx in range(start_idx, len(tokens)):
        if tokens[idx] in stop_token_ids:
            return idx
    return None


def generated_token_count(output_tokens: list[int], prompt_len: int) -> int:
    return max(len(output_tokens) - prompt_len, 0)


def trim_draft_cache(cache: list[Any], num_tokens: int) -> None:
    """runtime.py:22-26."""
    for layer_cache in cache:
        trim = getattr(layer_cache, "trim", None)
        if trim is not None:
            trim(num_tokens)


def _as_list(prompt_tokens) -> list[int]:
    if isinstance(prompt_tokens, torch.Tensor):
        return [int(t) for t in prompt_tokens.reshape(-1).tolist()]
    return [int(t) for t in prompt_tokens]


class _StateReader:
    """Pinned host mirror of the device decode state (one 32-byte copy a step)."""

    def __init__(self, state: torch.Tensor):
        self.dev = state
        self.host = torch.empty_like(state, device="cpu").pin_memory()

    def read(self) -> list[int]:
        self.host.copy_(self.dev, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return self.host.tolist()


def _sampling_seed(temperature: float) -> int:
    """Philox key of one sampled generation, drawn from torch's generator (so
    DFlashGenerator(seed=...) fixes the sequence of generations)."""
    if temperature < 1e-5:
        return 0
    return int(torch.randint(0, 2**31 - 1, (1,)).item())


def run_decode(target, draft, prompt_tokens, max_new_tokens: int, stop_token_ids: set[int], mode: str,
               block_size: int, budget: int, profile: bool = False, use_graph: bool = True,
               session: DecodeSession | None = None, temperature: float = 0.0,
               seed: int | None = None) -> tuple[list[int], dict[str, Any]]:
    """Device decode loop shared by dtree_generate and dflash_generate.
    temperature >= 1e-5 samples the first token, the posterior of every
    tree / chain node and (DFlash) the drafted tokens (runtime.py:12-19)."""
    engine = target.adapter.engine(target.model, draft)
    temperature = float(temperature)
    seed = _sampling_seed(temperature) if seed is None else int(seed)
    engine.set_sampling(temperature, seed)
    prompt = _as_list(prompt_tokens)
    prompt_len = len(prompt)
    total_max_tokens = prompt_len + int(max_new_tokens)
    vocab = engine.cfg.vocab_size
    rows = block_size - 1
    n_nodes = dtree_nodes(budget, rows, vocab) if mode == "dtree" else block_size
    if total_max_tokens + n_nodes + 1 > engine.kv_capacity:
        raise ValueError(
            f"prompt + max_new_tokens + tree ({total_max_tokens + n_nodes + 1}) exceeds the KV capacity "
            f"{engine.kv_capacity}"
        )
    cfg = StepConfig(mode=mode, rows=rows, budget=budget if mode == "dtree" else rows, n_nodes=n_nodes,
                     temperature=temperature if temperature >= 1e-5 else 0.0, seed=seed)
    if hasattr(draft, "_buffer"):
        draft._buffer(engine.device)  # fix the drafter's device buffers before any capture
    if session is None:
        session = getattr(target.adapter, "last_session", None)
    key = draft.graph_key() if hasattr(draft, "graph_key") else ("drafter", id(draft))
    reusable = (
        session is not None
        and session.engine is engine
        and session.cfg == cfg
        and session.output.numel() >= total_max_tokens + n_nodes + 2
    )
    if not reusable:
        session = DecodeSession(engine, cfg, total_max_tokens + n_nodes + 2, draft)
    elif session.drafter is not draft or getattr(session, "graph_key", None) != key:
        session.drafter = draft
        session.graph = None  # the captured step baked in the old drafter's parameters
    session.graph_key = key
    target.adapter.last_session = session

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    first_token = session.prefill(prompt)
    torch.cuda.synchronize()
    prefill_time = time.perf_counter() - t0

    reader = _StateReader(session.state)
    start = prompt_len
    acceptance_lengths: list[int] = []
    verified_nodes: list[int] = []
    checked = prompt_len
    stop_hit = None
    stages = {k: 0.0 for k in DTREE_STAGE_ORDER} if profile else None
    decode_start = time.perf_counter()
    steps = 0
    while start < total_max_tokens:
        session.host_start = start
        if profile:
            _profiled_step(session, stages)
        elif use_graph and session.graph is None and (steps >= 1 or getattr(session, "warm", False)):
            session.capture_step()
            session.replay()
        elif use_graph and session.graph is not None:
            session.replay()
        else:
            session.step()
            session.warm = True
        st = reader.read()
        steps += 1
        n_acc = st[3]
        new_start = st[0]
        acceptance_lengths.append(n_acc)
        verified_nodes.append(n_nodes)
        if stop_token_ids:
            seg = session.output[checked : new_start + 1].tolist()
            for i, tok in enumerate(seg):
                if tok in stop_token_ids:
                    stop_hit = checked + i
                    break
            checked = new_start + 1
        start = new_start
        if stop_hit is not None:
            break
        if start + 1 > total_max_tokens:
            break
    torch.cuda.synchronize()
    decode_time = time.perf_counter() - decode_start

    end = min(start + 1, total_max_tokens)
    if stop_hit is not None:
        end = min(end, stop_hit + 1)
    output_tokens = session.output[:end].tolist()
    assert end <= prompt_len or output_tokens[prompt_len] == first_token
    generated = generated_token_count(output_tokens, prompt_len)
    total_time = prefill_time + decode_time
    metrics: dict[str, Any] = {
        "decode_mode": mode,
        "num_input_tokens": prompt_len,
        "num_output_tokens": generated,
        "prefill_time_s": prefill_time,
        "decode_time_s": decode_time,
        "total_time_s": total_time,
        "prompt_tps": prompt_len / max(prefill_time, 1e-9),
        "generation_tps": generated / max(decode_time, 1e-9),
        "end_to_end_tps": generated / max(total_time, 1e-9),
        "avg_acceptance_length": sum(acceptance_lengths) / max(len(acceptance_lengths), 1),
        "acceptance_lengths": acceptance_lengths,
        "peak_memory_gb": torch.cuda.max_memory_allocated() / 1e9,
        "target_cache_summary": target.cache_summary([None] * engine.cfg.num_hidden_layers, offset=start),
        "speculative_tokens": block_size,
    }
    if mode == "dtree":
        metrics["avg_verified_tree_nodes"] = sum(verified_nodes) / max(len(verified_nodes), 1)
        metrics["verified_tree_nodes"] = verified_nodes
        metrics["tree_budget"] = budget
    if stages is not None:
        metrics["profile"] = {**stages, "unattributed_decode_time_s": decode_time - sum(stages.values()),
                              "steps": len(acceptance_lengths)}
    return output_tokens, metrics


def run_decode_lazy(target, draft, prompt_tokens, max_new_tokens: int, stop_token_ids: set[int], block_size: int,
                    budget: int, temperature: float, verify_mode: str, profile: bool = False
                    ) -> tuple[list[int], dict[str, Any]]:
    """dtree_generate's loop (dtree_runtime.py:364-552) with the lazy
    Qwen3.5 verify (``lazy_follow_tree_exact``): per step the draft and the
    best-first tree run on the device; the host then walks the tree one
    target token at a time (each a causal 1-token forward through the
    engine, whose cache ends up holding exactly the accepted path) and
    commits the accepted tokens and the posterior token."""
    from .adapters import SequenceCache
    from .dtree_runtime import lazy_follow_tree_exact

    engine = target.adapter.engine(target.model, draft)
    prompt = _as_list(prompt_tokens)
    prompt_len = len(prompt)
    total = prompt_len + int(max_new_tokens)
    vocab = engine.cfg.vocab_size
    rows = block_size - 1
    n_nodes = dtree_nodes(budget, rows, vocab)
    if total + n_nodes + 1 > engine.kv_capacity:
        raise ValueError(f"prompt + max_new_tokens + tree ({total + n_nodes + 1}) exceeds the KV capacity "
                         f"{engine.kv_capacity}")
    temperature = float(temperature)
    seed = _sampling_seed(temperature)
    engine.set_sampling(temperature, seed)
    cfg = StepConfig(mode="dtree", rows=rows, budget=budget, n_nodes=n_nodes,
                     temperature=temperature if temperature >= 1e-5 else 0.0, seed=seed)
    if hasattr(draft, "_buffer"):
        draft._buffer(engine.device)
    session = DecodeSession(engine, cfg, total + n_nodes + 2, draft)
    target.adapter.last_session = session
    layer_ids = list(engine.layer_ids)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    first = session.prefill(prompt)
    torch.cuda.synchronize()
    prefill_time = time.perf_counter() - t0
    cache = SequenceCache(engine)
    cache.offset = prompt_len
    output = prompt + [int(first)]
    start = prompt_len
    acceptance: list[int] = []
    stages = {"draft_time_s": 0.0, "tree_build_time_s": 0.0, "verify_time_s": 0.0} if profile else None
    decode_start = time.perf_counter()
    steps = 0
    while start < total:
        ta = time.perf_counter()
        session.drafter.draft(session)
        session.builder.build(session.draft_logits, session.state, session.tree, keep_topk=False)
        n = int(session.state[6].item())
        tb = time.perf_counter()
        tokens = session.tree.tokens[:n].tolist()
        parents = session.tree.parents[:n].tolist()
        child_maps: list[dict[int, int]] = [dict() for _ in range(n)]
        for i in range(1, n):
            child_maps[parents[i]][tokens[i]] = i
        accepted, posterior, hidden = lazy_follow_tree_exact(target, cache, layer_ids, tokens, child_maps,
                                                             temperature, verify_mode, None)
        tc = time.perf_counter()
        keep = len(accepted)
        output = output[:start] + [tokens[i] for i in accepted] + [int(posterior)]
        start += keep
        acceptance.append(keep)
        steps += 1
        # device decode state for the next draft: start, root, step, accepted
        new_state = torch.tensor([start, int(posterior), steps, keep, int(posterior), 0, n, 0], dtype=torch.int32)
        session.state.copy_(new_state.to(session.state.device))
        if getattr(session.drafter, "needs_hidden", False) and keep > 0:
            session.target_hidden[:keep] = hidden.reshape(keep, -1)[:, : session.target_hidden.shape[1]]
        if stages is not None:
            torch.cuda.synchronize()
            stages["draft_time_s"] += tb - ta
            stages["verify_time_s"] += tc - tb
        if stop_token_ids and any(t in stop_token_ids for t in output[prompt_len:]):
            break
    torch.cuda.synchronize()
    decode_time = time.perf_counter() - decode_start
    end = min(start + 1, total)
    if stop_token_ids:
        hit = stop_position(output, prompt_len, stop_token_ids)
        if hit is not None:
            end = min(end, hit + 1)
    output = output[:end]
    generated = generated_token_count(output, prompt_len)
    total_time = prefill_time + decode_time
    metrics: dict[str, Any] = {
        "decode_mode": "dtree",
        "qwen35_tree_mode": "lazy",
        "num_input_tokens": prompt_len,
        "num_output_tokens": generated,
        "prefill_time_s": prefill_time,
        "decode_time_s": decode_time,
        "total_time_s": total_time,
        "prompt_tps": prompt_len / max(prefill_time, 1e-9),
        "generation_tps": generated / max(decode_time, 1e-9),
        "end_to_end_tps": generated / max(total_time, 1e-9),
        "avg_acceptance_length": sum(acceptance) / max(len(acceptance), 1),
        "acceptance_lengths": acceptance,
        "peak_memory_gb": torch.cuda.max_memory_allocated() / 1e9,
        "target_cache_summary": target.cache_summary([None] * engine.cfg.num_hidden_layers, offset=start),
        "speculative_tokens": block_size,
        "tree_budget": budget,
    }
    if stages is not None:
        metrics["profile"] = {**stages, "steps": steps}
    return output, metrics


def _profiled_step(session: DecodeSession, stages: dict[str, float]) -> None:
    """Eager step with CUDA-event stage timers (dtree_runtime.py:24-56 keys)."""
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    c = session.cfg
    eng = session.engine
    ev[0].record()
    session.drafter.draft(session)
    ev[1].record()
    if c.mode == "dtree":
        session.builder.build(session.draft_logits, session.state, session.tree, keep_topk=False)
    else:
        kernels.chain_build(session.draft_logits[: c.rows], session.state, session.tree, c.temperature, c.seed)
    ev[2].record()
    eng.verify(session)
    ev[3].record()
    kernels.accept_walk(session.tree, session.posterior, session.state, session.accepted, session.output,
                        session.history)
    eng.commit_step(session)
    if getattr(session.drafter, "needs_hidden", False):
        kernels.gather_rows(eng.capture, session.accepted, session.state, session.target_hidden)
    kernels.step_commit(session.state)
    ev[4].record()
    ev[4].synchronize()
    stages["draft_time_s"] += ev[0].elapsed_time(ev[1]) / 1e3
    stages["tree_build_time_s"] += ev[1].elapsed_time(ev[2]) / 1e3
    stages["verify_time_s"] += ev[2].elapsed_time(ev[3]) / 1e3
    stages["bookkeeping_time_s"] += ev[3].elapsed_time(ev[4]) / 1e3


def dflash_generate(target, draft, prompt_tokens, max_new_tokens: int, temperature: float, stop_token_ids,
                    layer_ids, speculative_tokens: int | None, verify_mode: str, verify_chunk_size: int = 4,
                    profile: bool = False):
    """runtime.py:430-610: verify the drafted block as a chain tree.  Every
    verify mode reduces to the same device step: the block's posterior tokens
    (greedy, or sampled at ``temperature`` like sample_tokens in the
    parallel-replay / lazy-logits / stream / chunked verifiers) and the
    longest prefix match of the drafted tokens (drafted by argmax, or sampled
    at ``temperature``, runtime.py:486)."""
    del layer_ids, verify_chunk_size
    if verify_mode not in {"parallel-replay", "parallel-greedy-argmax", "parallel-lazy-logits", "stream", "chunked"}:
        raise ValueError(f"Unknown verify_mode={verify_mode!r}")
    if verify_mode == "parallel-greedy-argmax" and temperature >= 1e-5:
        raise ValueError("parallel-greedy-argmax only supports temperature=0.")
    block_size = draft.block_size if speculative_tokens is None else max(1, min(speculative_tokens, draft.block_size))
    if block_size < 2:
        raise ValueError("DFlash requires speculative_tokens >= 2 on the B200 path.")
    return run_decode(target, draft, prompt_tokens, max_new_tokens, set(stop_token_ids or ()), "dflash",
                      block_size, block_size - 1, profile=profile, temperature=temperature)
