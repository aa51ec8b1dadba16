"""Isolated tree-verify step timing (BASELINE config 2 sweep; with
``--quant-bits 4`` the config-3 target with MLX affine 4-bit projections).

Qwen3-4B shape (or another preset), bf16 random-init weights, K/V prefix of
random bf16 values (std 1), trees built on the GPU best-first from 16 rows of
draft log-probs sampled from Dirichlet(alpha=0.1) over a random top-32
support (seeded).  For every (prefix, tree budget) the tree-verify forward
(``dtree_qwen3_forward_tree``: all layers + fused LM-head argmax) is captured
in a CUDA graph and replayed; time per verify from CUDA events, HBM figures
against algorithmic bytes (all weights once + K/V prefix read + new K/V
write).  Mirrors the role of the reference's scripts/micro_verify.py and
scripts/micro_scaling.py.

    python -m dtree_mlx_b200.verify_sweep [--preset qwen3-4b] [--layers N]
        [--prefix 512,2048,8192] [--budget 8,24,64] [--iters 50] [--json]
"""
from __future__ import annotations

import argparse
import json
from dataclasses import replace
from pathlib import Path

import numpy as np
import torch

from . import kernels
from .config import PRESETS, QWEN35_PRESETS
from .engine import Qwen3Engine
from .synthetic import quantize_weights, random_qwen35_weights, random_qwen3_weights


def dirichlet_draft_logits(rows: int, vocab: int, seed: int, support: int = 32, alpha: float = 0.1) -> np.ndarray:
    """Draft log-probs: Dirichlet(alpha) mass over a random top-`support` set,
    every other token at log(1e-30)."""
    rng = np.random.default_rng(seed)
    out = np.full((rows, vocab), np.log(1e-30), dtype=np.float32)
    for r in range(rows):
        ids = rng.choice(vocab, size=support, replace=False)
        p = rng.dirichlet(np.full(support, alpha))
        out[r, ids] = np.log(np.maximum(p, 1e-30)).astype(np.float32)
    return out


def algorithmic_bytes(cfg, weights, prefix: int, t: int) -> float:
    wbytes = weights.streamed_bytes()
    kv_row = 2 * cfg.num_key_value_heads * cfg.head_dim * 2 * cfg.num_hidden_layers
    return float(wbytes + prefix * kv_row + t * kv_row)


def hybrid_algorithmic_bytes(cfg, weights, prefix: int, t: int) -> float:
    """Weights once + attention-layer K/V prefix read + new K/V write +
    DeltaNet conv / recurrent base states read (Qwen3.5 hybrid)."""
    kv_row = 2 * cfg.num_key_value_heads * cfg.head_dim * 2 * cfg.n_attn
    states = cfg.n_linear * (cfg.linear_num_value_heads * cfg.linear_value_head_dim * cfg.linear_key_head_dim * 4
                             + (cfg.linear_conv_kernel_dim - 1) * cfg.conv_dim * 2)
    return float(weights.streamed_bytes() + prefix * kv_row + t * kv_row + states)


def measured_hbm_gbs() -> tuple[float, str]:
    p = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def run(preset: str, layers: int | None, prefixes: list[int], budgets: list[int], iters: int, seed: int = 0,
        eager_only: bool = False, quant_bits: int = 16, q4_embedding: bool = False) -> list[dict]:
    if preset in QWEN35_PRESETS:
        return run_hybrid(preset, layers, prefixes, budgets, iters, seed, eager_only)
    cfg = PRESETS[preset]
    if layers:
        cfg = replace(cfg, num_hidden_layers=layers)
    dev = torch.device("cuda")
    w = random_qwen3_weights(cfg, seed=seed, device=dev)
    if quant_bits == 4:
        w = quantize_weights(w, embedding=q4_embedding)
        torch.cuda.empty_cache()
    eng = Qwen3Engine(w, kv_capacity=max(prefixes) + 160)
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    eng.kv_cache.copy_(torch.randn(eng.kv_cache.shape, generator=g, device=dev).to(torch.bfloat16))
    peak, peak_src = measured_hbm_gbs()
    results = []
    for budget in budgets:
        logits = torch.from_numpy(dirichlet_draft_logits(16, cfg.vocab_size, seed + budget)).to(dev)
        for P in prefixes:
            st = kernels.new_state(dev, start=P, root_token=1)
            tree = kernels.TreeBuffers.allocate(dev)
            kernels.TreeBuilder(16, cfg.vocab_size, budget, dev).build(logits, st, tree, keep_topk=False)
            n = int(st[6].item())
            post = torch.zeros(128, dtype=torch.int32, device=dev)
            eng.use_attention_shape(P, n)  # the shape a decode step at this prefix uses

            def fwd():
                eng.forward_tree(tree.tokens, tree.positions, tree.anc, n, st, post)

            for _ in range(3):
                fwd()
            torch.cuda.synchronize()
            graph = None
            if not eager_only:
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=s):
                    fwd()
                torch.cuda.current_stream().wait_stream(s)
                for _ in range(3):
                    graph.replay()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            a.record()
            for _ in range(iters):
                graph.replay() if graph is not None else fwd()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / iters
            nbytes = algorithmic_bytes(cfg, w, P, n)
            gbs = nbytes / (ms / 1e3) / 1e9
            results.append({"prefix": P, "tree_budget": budget, "tree_rows": n, "verify_ms": round(ms, 4),
                            "algorithmic_gb": round(nbytes / 1e9, 4), "achieved_gbs": round(gbs, 1),
                            "frac_of_hbm": round(gbs / peak, 4), "peak_gbs": peak, "peak_source": peak_src,
                            "layers": cfg.num_hidden_layers, "quant_bits": quant_bits,
                            "q4_embedding": bool(quant_bits == 4 and q4_embedding)})
            del graph
    eng.close()
    return results


def measured_tflops() -> tuple[float, str]:
    """Sustained dense bf16 tensor throughput (a seconds-long GEMM loop)."""
    p = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured sustained"
    return 1400.0, "fallback sustained"


def prefill_flops(cfg, n: int) -> float:
    """Algorithmic FLOPs of a causal prompt forward of n rows from slot 0:
    every projection (2 n K N), causal attention (QK^T and PV over the
    rows' visible keys) and the last row's LM head."""
    H, L = cfg.hidden_size, cfg.num_hidden_layers
    qd, kvd = cfg.num_attention_heads * cfg.head_dim, cfg.num_key_value_heads * cfg.head_dim
    proj = H * (qd + 2 * kvd) + qd * H + 2 * cfg.intermediate_size * H + cfg.intermediate_size * H
    keys = n * (n + 1) / 2
    attn = 4.0 * cfg.num_attention_heads * cfg.head_dim * keys
    return float(L * (2.0 * n * proj + attn) + 2.0 * H * cfg.vocab_size)


def hybrid_prefill_flops(cfg, n: int) -> float:
    """Algorithmic FLOPs of the hybrid's prompt forward of n rows from slot
    0: projections (2 n K N), the gated attention layers' causal attention,
    the DeltaNet recurrence (4 Hv Dv Dk per row) and the last row's LM head."""
    H = cfg.hidden_size
    kd, vd = cfg.linear_num_key_heads * cfg.linear_key_head_dim, cfg.linear_num_value_heads * cfg.linear_value_head_dim
    proj_w = 2 * kd + vd + vd + 2 * cfg.linear_num_value_heads
    qd = cfg.num_attention_heads * cfg.head_dim
    kvd = cfg.num_key_value_heads * cfg.head_dim
    mlp = 3 * H * cfg.intermediate_size
    lin = 2.0 * n * (H * proj_w + vd * H + mlp) + 4.0 * n * cfg.linear_num_value_heads * cfg.linear_value_head_dim * \
        cfg.linear_key_head_dim
    att = 2.0 * n * (H * (2 * qd + 2 * kvd) + qd * H + mlp) + 4.0 * cfg.num_attention_heads * cfg.head_dim * n * (n + 1) / 2
    return float(cfg.n_linear * lin + cfg.n_attn * att + 2.0 * H * cfg.vocab_size)


def run_prefill(preset: str, layers: int | None, n: int, iters: int, quant_bits: int = 16, seed: int = 0) -> dict:
    """Dense prefill of n prompt rows (dtree_qwen3_prefill /
    dtree_qwen35_prefill) against the verify-path prefill it replaces
    (128-row forwards)."""
    from .engine import chain_anc_masks

    hybrid = preset.startswith("qwen35")
    cfg = (QWEN35_PRESETS if hybrid else PRESETS)[preset]
    if layers:
        cfg = replace(cfg, num_hidden_layers=layers)
    if hybrid:
        from .engine35 import Qwen35Engine

        eng = Qwen35Engine(random_qwen35_weights(cfg, seed=seed, device="cuda"), kv_capacity=n + 128, layer_ids=[1])
    else:
        w = random_qwen3_weights(cfg, seed=seed, device="cuda")
        if quant_bits == 4:
            w = quantize_weights(w)
        eng = Qwen3Engine(w, kv_capacity=n + 128, layer_ids=[1])
    toks = torch.randint(0, cfg.vocab_size, (n,), dtype=torch.int32, device="cuda")
    state = kernels.new_state("cuda", start=0)
    hid = torch.zeros(n, cfg.hidden_size, dtype=torch.bfloat16, device="cuda")
    nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
    def dense():
        if hybrid:
            eng.reset_states()
        eng.prefill_dense(toks, state, hid, nxt)

    ms_dense = _time(dense, iters, True)
    post = torch.zeros(128, dtype=torch.int32, device="cuda")
    st2 = kernels.new_state("cuda", start=0)
    chunks = []
    for s in range(0, n, 128):
        t = min(128, n - s)
        chunks.append((s, t, torch.arange(s, s + t, dtype=torch.int32, device="cuda"),
                       torch.from_numpy(chain_anc_masks(t).view(np.int64)).to("cuda")))

    def chained():
        if hybrid:
            eng.reset_states()
        for s, t, pos, anc in chunks:
            st2[0] = s
            eng.prefill_chunk(toks[s:s + t], pos, anc, t, st2, post)

    ms_chain = _time(chained, max(1, iters // 2), True)
    eng.close()
    flops = hybrid_prefill_flops(cfg, n) if hybrid else prefill_flops(cfg, n)
    peak, src = measured_tflops()
    tf = flops / (ms_dense * 1e-3) / 1e12
    return {"prefill_rows": n, "layers": cfg.num_hidden_layers, "quant_bits": quant_bits,
            "dense_ms": round(ms_dense, 3), "verify_path_ms": round(ms_chain, 3),
            "speedup": round(ms_chain / ms_dense, 2), "tflops": round(tf, 1), "peak_tflops": peak,
            "peak_source": src, "frac_of_tensor_peak": round(tf / peak, 4)}


def _time(fn, iters: int, eager_only: bool) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    graph = None
    if not eager_only:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(3):
            graph.replay()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(iters):
        graph.replay() if graph is not None else fn()
    b.record()
    torch.cuda.synchronize()
    del graph
    return a.elapsed_time(b) / iters


def run_hybrid(preset: str, layers: int | None, prefixes: list[int], budgets: list[int], iters: int, seed: int,
               eager_only: bool) -> list[dict]:
    """BASELINE config 4 verify: the Qwen3.5 hybrid tree forward
    (``dtree_qwen35_forward`` mode 0, LM-head argmax included) on random
    committed states and a random bf16 K/V prefix."""
    from .engine35 import Qwen35Engine

    cfg = QWEN35_PRESETS[preset]
    if layers:
        cfg = replace(cfg, num_hidden_layers=layers)
    dev = torch.device("cuda")
    w = random_qwen35_weights(cfg, seed=seed, device=dev)
    eng = Qwen35Engine(w, kv_capacity=max(prefixes) + 160)
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    eng.kv_cache.copy_(torch.randn(eng.kv_cache.shape, generator=g, device=dev).to(torch.bfloat16))
    eng.rec_state.copy_(torch.randn(eng.rec_state.shape, generator=g, device=dev) * 0.05)
    eng.conv_state.copy_((torch.randn(eng.conv_state.shape, generator=g, device=dev) * 0.05).to(torch.bfloat16))
    peak, peak_src = measured_hbm_gbs()
    results = []
    for budget in budgets:
        logits = torch.from_numpy(dirichlet_draft_logits(16, cfg.vocab_size, seed + budget)).to(dev)
        for P in prefixes:
            st = kernels.new_state(dev, start=P, root_token=1)
            tree = kernels.TreeBuffers.allocate(dev)
            kernels.TreeBuilder(16, cfg.vocab_size, budget, dev).build(logits, st, tree, keep_topk=False)
            n = int(st[6].item())
            post = torch.zeros(128, dtype=torch.int32, device=dev)

            def fwd():
                eng.forward(tree.tokens, tree.positions, tree.parents, tree.anc, n, st, post, mode=0)

            ms = _time(fwd, iters, eager_only)
            nbytes = hybrid_algorithmic_bytes(cfg, w, P, n)
            gbs = nbytes / (ms / 1e3) / 1e9
            results.append({"preset": preset, "prefix": P, "tree_budget": budget, "tree_rows": n,
                            "verify_ms": round(ms, 4), "algorithmic_gb": round(nbytes / 1e9, 4),
                            "achieved_gbs": round(gbs, 1), "frac_of_hbm": round(gbs / peak, 4), "peak_gbs": peak,
                            "peak_source": peak_src, "layers": cfg.num_hidden_layers})
    eng.close()
    return results


def run_drafter(preset: str, prefix: int, iters: int, eager_only: bool, seed: int = 0) -> dict:
    """One DFlash draft step at the Qwen3-4B shape: append 16 accepted rows of
    target hiddens to the draft cache, run the 16-token block through the
    drafter layers against a ``prefix``-row context and produce fp32 logits
    through the target's LM head (draft.py:318-367, dtree_runtime.py:366-376)."""
    from types import SimpleNamespace

    from .config import DRAFT_PRESETS
    from .draft import DFlashDrafter, random_dflash_weights
    from .synthetic import STD

    cfg = DRAFT_PRESETS[preset]
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    embed = (torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g, device=dev) * STD).to(torch.bfloat16)
    w = random_dflash_weights(cfg, embed, seed=seed)
    d = DFlashDrafter(w, kv_capacity=prefix + 64)
    d.engine.kv_cache.copy_(torch.randn(d.engine.kv_cache.shape, generator=g, device=dev).to(torch.bfloat16))
    st = kernels.new_state(dev, start=prefix, root_token=1)
    st[3] = 16  # the last step accepted 16 rows
    width = w.fc.shape[1]
    sess = SimpleNamespace(state=st, draft_logits=d.logits[1:16],
                           target_hidden=(torch.randn(128, width, generator=g, device=dev) * 0.5).to(torch.bfloat16))
    ms = _time(lambda: d.draft(sess), iters, eager_only)
    wbytes = sum(x.numel() * x.element_size() for x in [embed, w.fc, *w.layers.qkv, *w.layers.o_proj,
                                                          *w.layers.gate_up, *w.layers.down])
    kv = prefix * 2 * cfg.kv_dim * 2 * cfg.num_hidden_layers
    nbytes = wbytes + kv + cfg.vocab_size * 16 * 4  # + the fp32 logits written
    peak, src = measured_hbm_gbs()
    d.engine.close()
    return {"drafter": preset, "prefix": prefix, "draft_ms": round(ms, 4), "algorithmic_gb": round(nbytes / 1e9, 4),
            "achieved_gbs": round(nbytes / (ms / 1e3) / 1e9, 1), "frac_of_hbm": round(nbytes / (ms / 1e3) / 1e9 / peak, 4),
            "peak_source": src, "layers": cfg.num_hidden_layers}


KERNEL_GROUPS = (
    ("lm_head", lambda k: k.startswith("gemm_streamk_kernel<") and k.split("<")[1].split(",")[1].strip() == "4"),
    ("gemm", lambda k: k.startswith("gemm_streamk_kernel")),
    ("attention", lambda k: k.startswith(("tree_attn_kernel", "tree_attn_tc_kernel", "attn_combine_kernel"))),
    ("norm_rope", lambda k: k.startswith(("residual_rmsnorm_kernel", "rmsnorm_kernel", "qkv_finish_kernel"))),
    ("tree_build", lambda k: k.startswith(("topk_lse_kernel", "heap_tree_kernel"))),
    ("deltanet", lambda k: k.startswith(("tree_conv1d_kernel", "tree_gated_delta_kernel", "rmsnorm_gated_kernel"))),
)


def summarize_launches(csv_path: str, forwards_per_config: int) -> list[dict]:
    """Attention / GEMM split per sweep configuration from an ncu launch list
    (``--metrics gpu__time_duration.sum --csv``) of an ``--eager`` sweep.

    Each configuration starts with its tree build (``topk_lse_kernel``), then
    runs ``forwards_per_config`` verify forwards (3 warm-up + ``--iters``).
    Times are ncu's serialised, cache-flushed per-launch durations: compare
    shares, not absolute milliseconds."""
    import csv
    import re

    rows = list(csv.reader(open(csv_path)))
    hi = next(i for i, r in enumerate(rows) if "Kernel Name" in r)
    hdr = rows[hi]
    ki, vi, ui = hdr.index("Kernel Name"), hdr.index("Metric Value"), hdr.index("Metric Unit")
    scale = {"nsecond": 1e-3, "ns": 1e-3, "usecond": 1.0, "us": 1.0, "msecond": 1e3, "ms": 1e3}
    segments: list[dict[str, float]] = []
    for r in rows[hi + 1:]:
        if len(r) <= vi:
            continue
        name = re.sub(r"\(.*", "", r[ki]).replace("void ", "").replace("dtree::", "").strip()
        us = float(r[vi].replace(",", "")) * scale[r[ui]]
        if name.startswith("topk_lse_kernel"):
            segments.append({})
        if not segments:
            continue
        group = next((g for g, match in KERNEL_GROUPS if match(name)), "other")
        segments[-1][group] = segments[-1].get(group, 0.0) + us
    out = []
    for seg in segments:
        fwd = {g: v / forwards_per_config for g, v in seg.items() if g != "tree_build"}
        total = sum(fwd.values())
        out.append({"per_forward_us": {g: round(v, 1) for g, v in sorted(fwd.items())},
                    "share": {g: round(v / total, 4) for g, v in sorted(fwd.items())},
                    "tree_build_us": round(seg.get("tree_build", 0.0), 1)})
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="qwen3-4b")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (smaller captures)")
    ap.add_argument("--prefix", default="512,2048,8192")
    ap.add_argument("--budget", default="8,24,64")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--eager", action="store_true", help="launch eagerly (no CUDA graph), e.g. under a profiler")
    ap.add_argument("--quant-bits", type=int, default=16, choices=[16, 4],
                    help="4: MLX affine 4-bit projections, group 64 (BASELINE config 3)")
    ap.add_argument("--q4-embedding", action="store_true",
                    help="with --quant-bits 4: quantize the embedding too (the reference's quantize_model), so the "
                         "tied LM head runs the 4-bit GEMM")
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--drafter", default=None, help="time one DFlash draft step of this drafter preset and exit")
    ap.add_argument("--prefill", type=int, default=0,
                    help="time a dense prefill of this many prompt rows (and the verify-path prefill) and exit")
    ap.add_argument("--launches", default=None,
                    help="summarise an ncu launch-list CSV of an --eager sweep (attention/GEMM split) and exit")
    a = ap.parse_args()
    if a.prefill:
        print(json.dumps(run_prefill(a.preset, a.layers, a.prefill, a.iters, a.quant_bits)))
        return
    if a.drafter:
        for P in [int(x) for x in a.prefix.split(",")]:
            print(json.dumps(run_drafter(a.drafter, P, a.iters, a.eager)))
        return
    if a.launches:
        prefixes, budgets = a.prefix.split(","), a.budget.split(",")
        split = summarize_launches(a.launches, 3 + a.iters)
        labels = [(int(b), int(p)) for b in budgets for p in prefixes]
        for (b, p), row in zip(labels, split):
            print(json.dumps({"prefix": p, "tree_budget": b, **row}))
        return
    res = run(a.preset, a.layers, [int(x) for x in a.prefix.split(",")], [int(x) for x in a.budget.split(",")],
              a.iters, eager_only=a.eager, quant_bits=a.quant_bits, q4_embedding=a.q4_embedding)
    if a.json:
        print(json.dumps(res))
    else:
        for r in res:
            print(f"prefix {r['prefix']:5d} budget {r['tree_budget']:3d} rows {r['tree_rows']:3d}: "
                  f"{r['verify_ms']:.3f} ms  {r['achieved_gbs']:7.1f} GB/s  ({100 * r['frac_of_hbm']:.1f}% of "
                  f"{r['peak_source']} HBM)")


if __name__ == "__main__":
    main()
