"""The persistent single-launch verify forward (csrc/fused.cu) against the
per-kernel chain (csrc/model.cu) on the same weights and inputs.

Both compute the same bf16 pipeline (qwen3_tree.py:39-83); they differ only
in the order of fp32 split-K / attention-split sums, so their outputs agree
to within bf16 rounding: relative Frobenius error <= 2e-2 on the final norm
output, the captured hiddens and the new K/V rows; posterior tokens equal
except at near-ties (top-2 logits within 5e-2).  The chain (the default
schedule) is checked against the fp32 oracle at full depth in
tests/test_gpu_parity_4b.py.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch


pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.float().double(), b.float().double()
    return float((a - b).norm() / max(float(b.norm()), 1e-30))


@pytest.fixture(scope="module")
def engines(lib):
    from dtree_mlx_b200.config import PRESETS
    from dtree_mlx_b200.engine import Qwen3Engine
    from dtree_mlx_b200.synthetic import random_qwen3_weights

    cfg = dataclasses.replace(PRESETS["qwen3-4b"], num_hidden_layers=4)
    w = random_qwen3_weights(cfg, seed=3, device=DEV, norm_jitter=0.1)
    fused = Qwen3Engine(w, kv_capacity=4096, layer_ids=[1, 3], verify_path="persistent")
    chain = Qwen3Engine(w, kv_capacity=4096, layer_ids=[1, 3])
    yield cfg, w, fused, chain
    fused.close()
    chain.close()


@pytest.mark.parametrize("P,budget", [(700, 8), (2048, 24), (3000, 39), (0, 24), (1500, 63)])
def test_fused_matches_chain(engines, P, budget):
    from dtree_mlx_b200 import _lib, kernels

    cfg, w, fused, chain = engines
    g = torch.Generator(device=DEV).manual_seed(P + budget)
    if P > 0:
        kv = torch.randn(fused.kv_cache[:, :, :, :P].shape, generator=g, device=DEV).to(torch.bfloat16)
        fused.kv_cache[:, :, :, :P] = kv
        chain.kv_cache[:, :, :, :P] = kv
    rng = np.random.default_rng(P + budget)
    rows = 16 if budget > 30 else 15
    dl = torch.from_numpy((rng.standard_normal((rows, cfg.vocab_size)) * 2).astype(np.float32)).to(DEV)
    root = int(rng.integers(cfg.vocab_size))
    state = kernels.new_state(DEV, start=P, root_token=root)
    tree = kernels.TreeBuffers.allocate(DEV)
    kernels.TreeBuilder(rows, cfg.vocab_size, budget, DEV).build(dl, state, tree)
    n = int(state[6].item())
    assert n == budget + 1
    posts = {}
    for name, eng in (("fused", fused), ("chain", chain)):
        post = torch.zeros(128, dtype=torch.int32, device=DEV)
        eng.forward_tree(tree.tokens, tree.positions, tree.anc, n, state, post)
        posts[name] = post
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    r_norm = _rel(fused.norm_out[:n], chain.norm_out[:n])
    r_cap = _rel(fused.capture[:n], chain.capture[:n])
    r_kv = max(_rel(fused.kv_cache[l, :, :, P:P + n], chain.kv_cache[l, :, :, P:P + n]) for l in range(4))
    print(f"P={P} T={n}: fused vs chain norm_out rel {r_norm:.2e}, capture rel {r_cap:.2e}, new K/V rel {r_kv:.2e}")
    assert r_norm <= 2e-2 and r_cap <= 2e-2 and r_kv <= 2e-2
    from dtree_mlx_b200.kernels import linear_bf16

    tp = 16 if n <= 16 else 32 if n <= 32 else 64
    x = torch.zeros(tp, cfg.hidden_size, dtype=torch.bfloat16, device=DEV)
    x[:n] = chain.norm_out[:n]
    logits = linear_bf16(x, w.embed)[:n].float()
    for t in range(n):
        a, b = int(posts["fused"][t]), int(posts["chain"][t])
        if a != b:
            mx = float(logits[t].max())
            assert mx - float(logits[t, a]) <= 5e-2 and mx - float(logits[t, b]) <= 5e-2, (t, a, b)


def test_fused_graph_replay_is_deterministic(engines):
    """A captured fused forward replays to bit-identical outputs (fixed
    split order everywhere, counters reset by the graph itself)."""
    from dtree_mlx_b200 import kernels
    from dtree_mlx_b200.engine import chain_anc_masks

    cfg, w, fused, _ = engines
    n = 25
    tokens = torch.randint(0, cfg.vocab_size, (128,), dtype=torch.int32, device=DEV)
    pos = torch.arange(1000, 1128, dtype=torch.int32, device=DEV)
    anc = torch.from_numpy(chain_anc_masks(n).view(np.int64)).to(DEV)
    state = kernels.new_state(DEV, start=1000)
    post = torch.zeros(128, dtype=torch.int32, device=DEV)
    fused.forward_tree(tokens, pos, anc, n, state, post)
    torch.cuda.synchronize()
    ref = fused.norm_out[:n].clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        fused.forward_tree(tokens, pos, anc, n, state, post)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(fused.norm_out[:n], ref)
    del graph
