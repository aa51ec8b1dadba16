"""Replica statistics over torch.distributed with two gloo ranks on the CPU
(the multi-GPU bench runs one independent sequence per GPU and combines only
these statistics)."""
from __future__ import annotations

import os
import socket

import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out) -> None:
    import datetime

    import torch.distributed as dist

    from dtree_mlx_b200.replicas import gather_replica_stats, max_over_ranks, sum_over_ranks

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ms = 100.0 + 10.0 * rank
        assert max_over_ranks(dist, ms, "cpu") == 110.0
        assert sum_over_ranks(dist, 2.0 + rank, "cpu") == 5.0
        agg = gather_replica_stats(dist, world, tokens=512.0, ms=ms, steps=200.0 + rank, accepted=400.0 + rank,
                                   device="cpu")
        if rank == 0:
            out.put(agg)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_replica_stats():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    agg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert agg["total_tokens"] == 1024.0
    assert agg["max_ms"] == 110.0
    assert abs(agg["tokens_per_s"] - 1024.0 / 0.110) < 1e-6
    assert agg["per_rank"][1] == [512.0, 110.0, 201.0, 401.0]
    assert abs(agg["mean_accepted"] - 801.0 / 401.0) < 1e-12


def test_single_process_without_dist():
    from dtree_mlx_b200.replicas import gather_replica_stats, max_over_ranks

    assert max_over_ranks(None, 3.5, "cpu") == 3.5
    agg = gather_replica_stats(None, 1, 512.0, 1000.0, 250.0, 500.0, "cpu")
    assert agg["tokens_per_s"] == 512.0 and agg["mean_accepted"] == 2.0
