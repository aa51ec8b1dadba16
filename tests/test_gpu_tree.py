"""CUDA tree path vs the oracle and the reference's own outputs (bit-exact).

Covers dtree_tree_build / dtree_tree_from_topk (dtree_runtime.py:82-192),
dtree_accept_walk (dtree_runtime.py:195-208, 530-537), dtree_kv_compact
(adapters.py:635-668), dtree_chain_build (runtime.py:476-490),
dtree_plant_draft_logits (the synthetic drafter) and dtree_step_commit.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import planted as OP
from oracle import tree as OT

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def K(lib):
    from dtree_mlx_b200 import kernels

    return kernels


@pytest.fixture(scope="module")
def golden(golden_dir):
    return json.loads((golden_dir / "tree_golden.json").read_text()), np.load(golden_dir / "tree_logits.npz")


def _tree_lists(out, n):
    toks = out.tokens[:n].cpu().tolist()
    return toks, out.parents[:n].cpu().tolist(), out.depths[:n].cpu().tolist(), out.positions[:n].cpu().tolist()


def _anc_bits(out, n):
    a = out.anc[:n].cpu().numpy().view(np.uint64)
    return a


def test_tree_build_matches_reference(K, golden):
    data, logits = golden
    for case in data["trees"]:
        lg = logits[case["name"]]
        rows, vocab = lg.shape
        budget = case["budget"]
        start, root = 37, 4242
        state = K.new_state(DEV, start=start, root_token=root)
        tb = K.TreeBuilder(rows, vocab, budget, DEV)
        out = K.TreeBuffers.allocate(DEV)
        tb.build(torch.from_numpy(lg).to(DEV), state, out)
        n = int(state[6].item())
        assert n == 1 + len(case["node_token_ids"]), case["name"]
        toks, parents, depths, pos = _tree_lists(out, n)
        assert toks == [root] + case["node_token_ids"], case["name"]
        assert parents == case["parents"], case["name"]
        assert depths == [0] + case["node_depths"], case["name"]
        assert pos == [start + d for d in depths]
        anc = _anc_bits(out, n)
        ref = OT.ancestor_masks(parents)
        assert np.array_equal(anc, ref), case["name"]
        if budget > 0:
            k = min(budget, vocab)
            np.testing.assert_allclose(tb.top_lp[:rows, :k].cpu().numpy(), np.asarray(case["top_log_probs"]),
                                       rtol=0, atol=4e-6)


def test_tree_from_reference_topk_bit_exact(K, golden):
    """Given the reference's own heap inputs the device heap is bit-exact."""
    data, _ = golden
    for case in data["trees"]:
        if case["budget"] <= 0:
            continue
        ids = torch.tensor(case["top_ids"], dtype=torch.int32, device=DEV)
        lps = torch.tensor(case["top_log_probs"], dtype=torch.float32, device=DEV)
        state = K.new_state(DEV, start=5, root_token=9)
        out = K.TreeBuffers.allocate(DEV)
        K.tree_from_topk(ids, lps, case["budget"], state, out)
        n = int(state[6].item())
        toks, parents, depths, _ = _tree_lists(out, n)
        assert toks[1:] == case["node_token_ids"], case["name"]
        assert parents == case["parents"], case["name"]


@pytest.mark.parametrize("budget", [8, 24, 64, 127])
def test_tree_build_random_vs_oracle(K, budget):
    rng = np.random.default_rng(budget)
    for rows, vocab in [(15, 151936), (16, 32768), (3, 50)]:
        lg = (rng.standard_normal((rows, vocab)) * 2).astype(np.float32)
        lg[:, rng.integers(vocab, size=4)] += 6.0
        state = K.new_state(DEV, start=100, root_token=1)
        tb = K.TreeBuilder(rows, vocab, budget, DEV)
        out = K.TreeBuffers.allocate(DEV)
        tb.build(torch.from_numpy(lg).to(DEV), state, out)
        k = min(budget, vocab)
        ids = tb.top_ids[:rows, :k].cpu().numpy().astype(np.int64)
        lps = tb.top_lp[:rows, :k].cpu().numpy()
        ref_ids, ref_lps = OT.topk_log_probs(lg, k)
        assert np.array_equal(ids, ref_ids)
        np.testing.assert_allclose(lps, ref_lps, rtol=0, atol=4e-6)
        # the heap on the device's own log-probs is bit-exact
        toks, depths, parents, _ = OT.heap_build(ids, lps, budget)
        n = int(state[6].item())
        assert n == 1 + len(toks)
        g_toks, g_parents, g_depths, _ = _tree_lists(out, n)
        assert g_toks[1:] == toks and g_parents == parents and g_depths[1:] == depths


def test_tree_build_vocab_beyond_the_noalloc_scratch(K, lib):
    """The workspace build has no 1 MiB cap: 64 draft rows over a vocabulary
    larger than the no-allocation scratch covers still match the oracle."""
    rows, vocab, budget = 64, 400_000, 24
    assert vocab > int(lib.dtree_tree_build_noalloc_max_vocab(rows))
    rng = np.random.default_rng(7)
    lg = (rng.standard_normal((rows, vocab)) * 2).astype(np.float32)
    lg[:, rng.integers(vocab, size=4)] += 6.0
    state = K.new_state(DEV, start=3, root_token=1)
    tb = K.TreeBuilder(rows, vocab, budget, DEV)
    out = K.TreeBuffers.allocate(DEV)
    tb.build(torch.from_numpy(lg).to(DEV), state, out)
    ids = tb.top_ids[:rows, :budget].cpu().numpy().astype(np.int64)
    ref_ids, _ = OT.topk_log_probs(lg, budget)
    assert np.array_equal(ids, ref_ids)
    toks, depths, parents, _ = OT.heap_build(ids, tb.top_lp[:rows, :budget].cpu().numpy(), budget)
    n = int(state[6].item())
    g_toks, g_parents, _, _ = _tree_lists(out, n)
    assert g_toks[1:] == toks and g_parents == parents


def test_tree_build_ties_by_token_id(K):
    lg = np.zeros((4, 300), dtype=np.float32)
    lg[:, [7, 250, 3, 99]] = 5.0  # exact ties across chunks
    state = K.new_state(DEV)
    tb = K.TreeBuilder(4, 300, 6, DEV)
    out = K.TreeBuffers.allocate(DEV)
    tb.build(torch.from_numpy(lg).to(DEV), state, out)
    ids = tb.top_ids[:4, :6].cpu().numpy()
    ref_ids, _ = OT.topk_log_probs(lg, 6)
    assert np.array_equal(ids, ref_ids)
    assert ids[0, :4].tolist() == [3, 7, 99, 250]


def test_planted_logits_bit_exact(K):
    rows, vocab = 15, 5000
    cont = np.random.default_rng(0).integers(vocab, size=64).astype(np.int32)
    for step, start, p in [(0, 10, 0.8), (3, 40, 0.85), (7, 60, 1.0)]:
        state = K.new_state(DEV, start=start)
        state[2] = step
        out = torch.empty(rows, vocab, dtype=torch.float32, device=DEV)
        K.plant_draft_logits(out, 1234, state, torch.from_numpy(cont).to(DEV), p)
        ref = OP.planted_draft_logits(1234, step, start, rows, vocab, cont, p)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_accept_walk_matches_reference(K, golden):
    data, _ = golden
    for w in data["walks"]:
        n = len(w["parents"])
        out = K.TreeBuffers.allocate(DEV)
        out.tokens[:n] = torch.tensor(w["tree_tokens"], dtype=torch.int32)
        out.parents[:n] = torch.tensor(w["parents"], dtype=torch.int32)
        state = K.new_state(DEV, start=3, root_token=w["tree_tokens"][0])
        state[6] = n
        post = torch.zeros(128, dtype=torch.int32, device=DEV)
        post[:n] = torch.tensor(w["posterior"], dtype=torch.int32)
        acc = torch.full((128,), -1, dtype=torch.int32, device=DEV)
        outbuf = torch.full((256,), -7, dtype=torch.int32, device=DEV)
        hist = torch.zeros(8, dtype=torch.int32, device=DEV)
        K.accept_walk(out, post, state, acc, outbuf, hist)
        st = K.state_dict(state)
        na = st["n_accepted"]
        assert acc[:na].cpu().tolist() == w["accepted"]
        assert st["bonus_token"] == w["next_token"]
        expect = [w["tree_tokens"][i] for i in w["accepted"]] + [w["next_token"]]
        assert outbuf[3:3 + na + 1].cpu().tolist() == expect
        assert st["n_output"] == 3 + na + 1
        assert int(hist[0].item()) == na
        K.step_commit(state)
        st2 = K.state_dict(state)
        assert st2["start"] == 3 + na and st2["root_token"] == w["next_token"] and st2["step"] == 1


def test_kv_compact_matches_reference(K, golden_dir):
    z = np.load(golden_dir / "compact_golden.npz")
    for c in range(int(z["count"])):
        meta = z[f"c{c}_meta"].tolist()
        past, t, nkeep = meta[:3]
        keep = meta[3:3 + nkeep]
        ks = [torch.from_numpy(z[f"c{c}_k_in_{li}"][0]) for li in range(2)]
        vs = [torch.from_numpy(z[f"c{c}_v_in_{li}"][0]) for li in range(2)]
        cache = torch.stack([torch.stack([ks[li], vs[li]]) for li in range(2)]).to(torch.bfloat16).to(DEV).contiguous()
        state = K.new_state(DEV, start=past)
        state[3] = nkeep
        acc = torch.tensor(keep + [0] * (128 - nkeep), dtype=torch.int32, device=DEV)
        K.kv_compact(cache, acc, state)
        K.step_commit(state)
        got = cache.cpu()
        # the committed length is the reference's new cache offset (past when
        # nothing is kept: the rows stay, the offset is trimmed)
        assert int(state[0].item()) == int(z[f"c{c}_offset_0"])
        for li in range(2):
            ek = torch.from_numpy(z[f"c{c}_k_out_{li}"][0]).to(torch.bfloat16)
            ev = torch.from_numpy(z[f"c{c}_v_out_{li}"][0]).to(torch.bfloat16)
            assert torch.equal(got[li, 0], ek) and torch.equal(got[li, 1], ev)


def test_chain_build_first_index_ties(K):
    lg = torch.zeros(5, 1000, dtype=torch.float32)
    lg[0, 17] = 3.0
    lg[1, [400, 40]] = 2.0
    lg[2, 999] = 1.0
    lg[3, [5, 6, 7]] = 9.0
    state = K.new_state(DEV, start=20, root_token=77)
    out = K.TreeBuffers.allocate(DEV)
    K.chain_build(lg.to(DEV), state, out)
    n = int(state[6].item())
    assert n == 6
    toks, parents, depths, pos = _tree_lists(out, n)
    assert toks == [77, 17, 40, 999, 5, 0]
    assert parents == [-1, 0, 1, 2, 3, 4]
    assert pos == [20 + i for i in range(6)]
    anc = _anc_bits(out, n)
    assert np.array_equal(anc, OT.ancestor_masks(parents))


def test_gather_rows(K):
    src = torch.arange(40 * 64, dtype=torch.float32, device=DEV).view(40, 64).to(torch.bfloat16)
    dst = torch.zeros(16, 64, dtype=torch.bfloat16, device=DEV)
    state = K.new_state(DEV)
    state[3] = 4
    acc = torch.tensor([0, 3, 9, 30] + [0] * 124, dtype=torch.int32, device=DEV)
    K.gather_rows(src, acc, state, dst)
    assert torch.equal(dst[:4], src[[0, 3, 9, 30]])
    assert torch.count_nonzero(dst[4:]) == 0


def test_no_device_error(lib):
    from dtree_mlx_b200 import _lib

    assert _lib.device_error(clear=True) == 0
