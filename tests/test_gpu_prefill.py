"""Dense prompt prefill (dtree_qwen3_prefill: tensor-core GEMMs over all
prompt rows, chunked causal attention) against the fp32 CPU oracle and
against the per-128-row verify forward it replaces (adapters.py:494-533 is
the reference's prompt forward).

Tolerances (bf16 engine vs fp32 oracle on the same bf16 weights):
  tiny preset (4 layers, hidden 512): final norm output, captured hiddens
      and every cached K/V row within relative Frobenius error 2e-2 (the
      verify forward's bar in tests/test_gpu_model.py);
  Qwen3-4B width (4 of its layers, hidden 2560, 2048 prompt rows): 3e-2
      against the oracle; dense vs verify-path prefill on the GPU (two bf16
      pipelines that differ only in fp32 summation order) 2e-2;
  next token: the oracle's bf16 argmax of the last row, or a near-tie
      (both within 3e-2 of the row maximum).
"""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from oracle.qwen3 import Qwen3Oracle
from oracle.runtime import near_tie

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a = a.float().cpu().double() if torch.is_tensor(a) else torch.as_tensor(np.asarray(a)).double()
    b = b.float().cpu().double() if torch.is_tensor(b) else torch.as_tensor(np.asarray(b)).double()
    return float((a - b).norm() / max(float(b.norm()), 1e-30))


def _prefill(eng, tokens, start, layer_ids):
    from dtree_mlx_b200 import kernels

    n = len(tokens)
    state = kernels.new_state(DEV, start=start)
    norm = torch.zeros(n, eng.cfg.hidden_size, dtype=torch.bfloat16, device=DEV)
    hid = torch.zeros(n, eng.cfg.hidden_size * len(layer_ids), dtype=torch.bfloat16, device=DEV)
    nxt = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    eng.prefill_dense(torch.tensor(tokens, dtype=torch.int32, device=DEV), state, hid if layer_ids else None, nxt,
                      norm_out=norm)
    torch.cuda.synchronize()
    return norm, hid, int(nxt.item())


@pytest.mark.parametrize("quant", ["bf16", "q4"])
def test_dense_prefill_matches_oracle_tiny(lib, quant):
    """Two prompt pieces (300 rows from slot 0, then 200 rows after them):
    ragged 256-row GEMM tiles and 128-row attention chunks, a nonzero start."""
    from dtree_mlx_b200 import _lib
    from dtree_mlx_b200.config import PRESETS
    from dtree_mlx_b200.engine import Qwen3Engine
    from dtree_mlx_b200.synthetic import quantize_weights, random_qwen3_weights

    cfg = PRESETS["qwen3-tiny"]
    w = random_qwen3_weights(cfg, seed=0, device=DEV, norm_jitter=0.1)
    if quant == "q4":
        w = quantize_weights(w)
    ids = [1, 3]
    eng = Qwen3Engine(w, kv_capacity=1024, layer_ids=ids)
    orc = Qwen3Oracle(w, kv_capacity=1024)
    rng = np.random.default_rng(1)
    p1 = rng.integers(cfg.vocab_size, size=300).tolist()
    p2 = rng.integers(cfg.vocab_size, size=200).tolist()
    for start, toks in ((0, p1), (300, p2)):
        norm, hid, nxt = _prefill(eng, toks, start, ids)
        assert _lib.device_error() == 0
        o_norm, o_vh = orc.prefill(toks, layer_ids=ids)
        r_norm, r_hid = _rel(norm, o_norm), _rel(hid, o_vh)
        print(f"{quant} start={start} n={len(toks)}: norm rel {r_norm:.2e}, hidden rel {r_hid:.2e}")
        assert r_norm < 2e-2 and r_hid < 2e-2
        o_log = orc.lm_head_logits(o_norm[-1:])[0]
        ref = int(torch.argmax(o_log.to(torch.bfloat16).float()))
        assert nxt == ref or near_tie(o_log, nxt, ref, 3e-2), (nxt, ref)
    end = 500
    for l in range(cfg.num_hidden_layers):
        assert _rel(eng.kv_cache[l, 0, :, :end], orc.k[l][:, :end]) < 2e-2
        assert _rel(eng.kv_cache[l, 1, :, :end], orc.v[l][:, :end]) < 2e-2
    eng.close()


@pytest.fixture(scope="module")
def wide(lib):
    from dtree_mlx_b200.config import PRESETS
    from dtree_mlx_b200.synthetic import random_qwen3_weights

    torch.set_num_threads(max(1, min(64, torch.get_num_threads())))
    cfg = dataclasses.replace(PRESETS["qwen3-4b"], num_hidden_layers=4)
    return cfg, random_qwen3_weights(cfg, seed=2, device=DEV, norm_jitter=0.1)


def test_dense_prefill_4b_width_2048_rows(wide):
    """2048 prompt rows at the 4B width: oracle parity, and the dense prefill
    against the 16 verify-path forwards it replaces."""
    from dtree_mlx_b200 import _lib
    from dtree_mlx_b200.engine import Qwen3Engine

    cfg, w = wide
    ids = [1, 3]
    n = 2048
    prompt = np.random.default_rng(3).integers(cfg.vocab_size, size=n).tolist()
    dense = Qwen3Engine(w, kv_capacity=n + 64, layer_ids=ids)
    norm, hid, nxt = _prefill(dense, prompt, 0, ids)
    assert _lib.device_error() == 0
    chain = Qwen3Engine(w, kv_capacity=n + 64, layer_ids=ids)
    c_norm, c_nxt = _verify_path_prefill(chain, prompt)
    r_dc = _rel(norm, c_norm)
    r_kv = max(_rel(dense.kv_cache[l, :, :, :n], chain.kv_cache[l, :, :, :n]) for l in range(cfg.num_hidden_layers))
    print(f"dense vs verify-path prefill: norm rel {r_dc:.2e}, K/V rel {r_kv:.2e}, next {nxt} / {c_nxt}")
    assert r_dc < 2e-2 and r_kv < 2e-2
    chain.close()
    orc = Qwen3Oracle(w, kv_capacity=n + 64)
    o_norm, o_vh = orc.prefill(prompt, layer_ids=ids)
    r_norm, r_hid = _rel(norm, o_norm), _rel(hid, o_vh)
    r_k = max(_rel(dense.kv_cache[l, 0, :, :n], orc.k[l][:, :n]) for l in range(cfg.num_hidden_layers))
    r_v = max(_rel(dense.kv_cache[l, 1, :, :n], orc.v[l][:, :n]) for l in range(cfg.num_hidden_layers))
    print(f"dense prefill vs oracle: norm rel {r_norm:.2e}, hidden rel {r_hid:.2e}, K rel {r_k:.2e}, V rel {r_v:.2e}")
    assert max(r_norm, r_hid, r_k, r_v) < 3e-2
    o_log = orc.lm_head_logits(o_norm[-1:])[0]
    ref = int(torch.argmax(o_log.to(torch.bfloat16).float()))
    assert nxt == ref or near_tie(o_log, nxt, ref, 3e-2), (nxt, ref)
    dense.close()


def test_session_prefill_uses_dense_path(lib):
    """DecodeSession.prefill on a 300-token prompt (longer than one verify
    forward): the first token and the drafter's prompt hiddens match the
    oracle."""
    from dtree_mlx_b200.config import PRESETS
    from dtree_mlx_b200.engine import DecodeSession, Qwen3Engine, StepConfig
    from dtree_mlx_b200.synthetic import random_qwen3_weights

    cfg = PRESETS["qwen3-tiny"]
    w = random_qwen3_weights(cfg, seed=4, device=DEV, norm_jitter=0.1)
    ids = [0, 2]
    eng = Qwen3Engine(w, kv_capacity=1024, layer_ids=ids)
    eng.dense_prefill_min_rows = 129  # (the default routes prompts this short to 128-row verify forwards)
    sess = DecodeSession(eng, StepConfig(mode="dtree", rows=15, budget=24, n_nodes=25), 1024, drafter=None)
    prompt = np.random.default_rng(5).integers(cfg.vocab_size, size=300).tolist()
    first = sess.prefill(prompt)
    orc = Qwen3Oracle(w, kv_capacity=1024)
    o_norm, o_vh = orc.prefill(prompt, layer_ids=ids)
    assert _rel(sess.prompt_hidden, o_vh) < 2e-2
    o_log = orc.lm_head_logits(o_norm[-1:])[0]
    ref = int(torch.argmax(o_log.to(torch.bfloat16).float()))
    assert first == ref or near_tie(o_log, first, ref, 3e-2), (first, ref)
    assert int(sess.state[0].item()) == 300 and int(sess.state[1].item()) == first
    eng.close()


def _verify_path_prefill(eng, tokens):
    from dtree_mlx_b200 import kernels
    from dtree_mlx_b200.engine import chain_anc_masks

    n = len(tokens)
    state = kernels.new_state(DEV, start=0)
    post = torch.zeros(128, dtype=torch.int32, device=DEV)
    toks = torch.tensor(tokens, dtype=torch.int32, device=DEV)
    norms = []
    for s in range(0, n, 128):
        t = min(128, n - s)
        state[0] = s
        anc = torch.from_numpy(chain_anc_masks(t).view(np.int64)).to(DEV)
        eng.prefill_chunk(toks[s:s + t].contiguous(), torch.arange(s, s + t, dtype=torch.int32, device=DEV), anc, t,
                          state, post)
        norms.append(eng.norm_out[:t].clone())
    torch.cuda.synchronize()
    return torch.cat(norms), int(post[t - 1].item())


# ---------------------------------------------------------------- hybrid
# Tolerances as tests/test_gpu_qwen35.py: relative 3e-2 against the oracle
# with bf16 activations, 4e-2 against the fp32 oracle (hidden rows, K/V,
# conv and recurrent states); dense vs verify-path prefill on the GPU 2e-2.
REL35 = {"bf16": 3e-2, "fp32": 4e-2}


def _hybrid_states(eng, cfg):
    return eng.conv_state.clone(), eng.rec_state.clone()


def test_hybrid_dense_prefill_matches_oracle(lib):
    """Two prompt pieces (300 rows, then 200 more): the DeltaNet conv /
    recurrent states carry across pieces, the attention layers see the first
    piece's K/V."""
    from dtree_mlx_b200 import _lib
    from dtree_mlx_b200.config import QWEN35_PRESETS
    from dtree_mlx_b200.engine35 import Qwen35Engine
    from dtree_mlx_b200.synthetic import random_qwen35_weights
    from oracle.qwen35 import Qwen35Oracle

    cfg = QWEN35_PRESETS["qwen35-tiny"]
    w = random_qwen35_weights(cfg, seed=0, device=DEV, norm_jitter=0.1)
    ids = [1, 2]
    eng = Qwen35Engine(w, kv_capacity=1024, layer_ids=ids)
    orcs = {"fp32": Qwen35Oracle(w, kv_capacity=1024), "bf16": Qwen35Oracle(w, kv_capacity=1024, bf16_acts=True)}
    rng = np.random.default_rng(7)
    pieces = [(0, rng.integers(cfg.vocab_size, size=300).tolist()), (300, rng.integers(cfg.vocab_size, size=200).tolist())]
    lin = [l for l in range(cfg.num_hidden_layers) if cfg.is_linear(l)]
    att = [l for l in range(cfg.num_hidden_layers) if not cfg.is_linear(l)]
    for start, toks in pieces:
        norm, hid, nxt = _prefill(eng, toks, start, ids)
        assert _lib.device_error() == 0
        T = len(toks)
        mask = np.ones((T, start + T), dtype=bool)
        mask[:, start:] = np.tril(np.ones((T, T), dtype=bool))
        o_norms = {}
        for name, orc in orcs.items():
            o_norm, o_hid = orc.forward(toks, np.arange(start, start + T), np.arange(-1, T - 1), mask, start,
                                        tree=False, layer_ids=ids)
            o_norms[name] = torch.as_tensor(np.asarray(o_norm.float() if torch.is_tensor(o_norm) else o_norm))
            r_norm, r_hid = _rel(norm, o_norm), _rel(hid, o_hid)
            print(f"hybrid start={start} vs {name}: norm rel {r_norm:.2e}, hidden rel {r_hid:.2e}")
            assert r_norm < REL35[name] and r_hid < REL35[name]
            for li, l in enumerate(lin):
                assert _rel(eng.conv_state[li], orc.conv[l]) < REL35[name], (name, "conv", l)
                assert _rel(eng.rec_state[li], orc.rec[l]) < REL35[name], (name, "rec", l)
            for ai, l in enumerate(att):
                end = start + T
                assert _rel(eng.kv_cache[ai, 0, :, :end], orc.k[l][:, :end]) < REL35[name], (name, "k")
                assert _rel(eng.kv_cache[ai, 1, :, :end], orc.v[l][:, :end]) < REL35[name], (name, "v")
        o_log = torch.as_tensor(np.asarray(orcs["bf16"].lm_head_logits(o_norms["bf16"][-1:].float())))[0].float()
        ref = int(torch.argmax(o_log.to(torch.bfloat16).float()))
        assert nxt == ref or near_tie(o_log, nxt, ref, 0.15), (nxt, ref)
    eng.close()


def test_hybrid_dense_prefill_9b_width(lib):
    """2048 prompt rows through 4 layers of the Qwen3.5-9B shape (3 DeltaNet
    + 1 gated attention): dense prefill against the 16 verify-path
    (sequence-mode) forwards it replaces."""
    from dtree_mlx_b200 import _lib
    from dtree_mlx_b200.config import QWEN35_PRESETS
    from dtree_mlx_b200.engine import chain_anc_masks
    from dtree_mlx_b200.engine35 import Qwen35Engine
    from dtree_mlx_b200.synthetic import random_qwen35_weights

    cfg = dataclasses.replace(QWEN35_PRESETS["qwen35-9b"], num_hidden_layers=4)
    w = random_qwen35_weights(cfg, seed=1, device=DEV, norm_jitter=0.1)
    n = 2048
    prompt = np.random.default_rng(8).integers(cfg.vocab_size, size=n).tolist()
    dense = Qwen35Engine(w, kv_capacity=n + 64, layer_ids=[3])
    norm, hid, nxt = _prefill(dense, prompt, 0, [3])
    assert _lib.device_error() == 0
    chain = Qwen35Engine(w, kv_capacity=n + 64, layer_ids=[3])
    from dtree_mlx_b200 import kernels

    state = kernels.new_state(DEV, start=0)
    post = torch.zeros(128, dtype=torch.int32, device=DEV)
    toks = torch.tensor(prompt, dtype=torch.int32, device=DEV)
    norms = []
    for s in range(0, n, 128):
        state[0] = s
        anc = torch.from_numpy(chain_anc_masks(128).view(np.int64)).to(DEV)
        chain.prefill_chunk(toks[s:s + 128].contiguous(), torch.arange(s, s + 128, dtype=torch.int32, device=DEV), anc,
                            128, state, post)
        norms.append(chain.norm_out[:128].clone())
    torch.cuda.synchronize()
    r_norm = _rel(norm, torch.cat(norms))
    r_conv = _rel(dense.conv_state, chain.conv_state)
    r_rec = _rel(dense.rec_state, chain.rec_state)
    r_kv = _rel(dense.kv_cache[:, :, :, :n], chain.kv_cache[:, :, :, :n])
    print(f"hybrid dense vs verify-path prefill: norm {r_norm:.2e} conv {r_conv:.2e} rec {r_rec:.2e} "
          f"K/V {r_kv:.2e}; next {nxt} / {int(post[127].item())}")
    assert max(r_norm, r_conv, r_rec, r_kv) < 2e-2
    dense.close()
    chain.close()
