"""Independent-sequence replicas across GPUs (one process per GPU).

The DTree step is a dependent chain per sequence (draft -> tree -> verify ->
accept -> next), so it shards only over independent sequences: every rank
decodes its own prompt with a full copy of the weights, and the only
collectives are the end-of-run statistics below (device-timed, max over
ranks for time; sums for work).  No collective runs in the data path.
"""
from __future__ import annotations

import torch


def max_over_ranks(dist, value: float, device) -> float:
    """Largest per-rank value (the job's device time)."""
    if dist is None:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(dist, value: float, device) -> float:
    if dist is None:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t)
    return float(t.item())


def gather_replica_stats(dist, world: int, tokens: float, ms: float, steps: float, accepted: float,
                         device) -> dict:
    """All ranks' (tokens, ms, decode steps, accepted tokens); rank 0 uses the
    aggregate: whole-job tokens / max-over-ranks time."""
    stats = torch.tensor([tokens, ms, steps, accepted], dtype=torch.float64, device=device)
    rows = [stats]
    if dist is not None and world > 1:
        rows = [torch.zeros_like(stats) for _ in range(world)]
        dist.all_gather(rows, stats)
    per_rank = [[float(x) for x in r.tolist()] for r in rows]
    total_tokens = sum(r[0] for r in per_rank)
    max_ms = max(r[1] for r in per_rank)
    return {"per_rank": per_rank, "total_tokens": total_tokens, "max_ms": max_ms,
            "tokens_per_s": total_tokens / (max_ms / 1e3) if max_ms > 0 else 0.0,
            "mean_accepted": sum(r[3] for r in per_rank) / max(1.0, sum(r[2] for r in per_rank))}
