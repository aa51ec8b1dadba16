"""Device-resident Qwen3 verify engine and per-sequence decode sessions.

``Qwen3Engine`` owns the C model handle (``dtree_qwen3_create``) and the
activation / KV buffers it runs on (allocated once with torch, the device
memory plumbing).  ``DecodeSession`` holds one sequence's device state
(``dtree_step_state``, tree buffers, output tokens) and runs a whole decode
step -- draft logits, tree build, tree-verify forward with the fused LM-head
argmax, acceptance walk, KV compaction, commit -- as device launches with no
host round trip; ``capture_step`` records that step into one CUDA graph.

The step mirrors one iteration of dtree_generate's loop
(dtree_mlx/dtree_runtime.py:364-552) and, with a chain tree, of
dflash_generate's parallel-greedy-argmax verify (dtree_mlx/runtime.py:474-577).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib, kernels
from ._lib import DTREE_MAX_TREE, Qwen3Desc, Qwen3Layer, Qwen3Q4Layer, call, ptr, stream_ptr
from .config import Qwen3Config
from .synthetic import Q4Tensor, Qwen3Weights


def _wptr(t) -> int:
    """Device pointer of a projection weight (packed words for a Q4Tensor)."""
    return ptr(t.packed) if isinstance(t, Q4Tensor) else ptr(t)


def pad_rows(n: int) -> int:
    """Tree rows padded to a legal UMMA N: 16, 32, 64, 80 or 128."""
    for t in (16, 32, 64, 80, 128):
        if n <= t:
            return t
    raise ValueError(f"at most {DTREE_MAX_TREE} tree rows per forward, got {n}")


def chain_anc_masks(n: int) -> np.ndarray:
    """Causal (chain) visibility as packed bits: row i sees nodes 0..i."""
    out = np.zeros((n, 2), dtype=np.uint64)
    for i in range(n):
        lo = min(i, 63)
        out[i, 0] = np.uint64((1 << (lo + 1)) - 1) if lo < 63 else np.uint64(0xFFFFFFFFFFFFFFFF)
        if i >= 64:
            hi = i - 64
            out[i, 1] = np.uint64((1 << (hi + 1)) - 1) if hi < 63 else np.uint64(0xFFFFFFFFFFFFFFFF)
    return out


def mask_to_anc(visibility: np.ndarray) -> np.ndarray:
    """Bool visibility [T, T] -> packed ancestor bits [T, 2] (uint64)."""
    t = visibility.shape[0]
    out = np.zeros((t, 2), dtype=np.uint64)
    for i in range(t):
        for j in np.nonzero(visibility[i])[0]:
            out[i, j // 64] |= np.uint64(1) << np.uint64(j % 64)
    return out


class Qwen3Engine:
    """One Qwen3 target on one GPU (weights + KV cache + scratch buffers)."""

    def __init__(self, weights: Qwen3Weights, kv_capacity: int, layer_ids=(), t_cap: int = DTREE_MAX_TREE,
                 verify_path: str = "chain"):
        """``verify_path``: "chain" runs the verify forward as the per-kernel
        chain; "persistent" as one persistent launch (one CTA per SM) where
        the model supports it (bf16, head_dim 128, <= 64 rows)."""
        if verify_path not in ("chain", "persistent"):
            raise ValueError("verify_path must be 'chain' or 'persistent'")
        cfg: Qwen3Config = weights.cfg
        if weights.device.type != "cuda":
            raise ValueError("engine weights must live on a CUDA device")
        self.cfg = cfg
        self.weights = weights
        self.device = weights.device
        self.layer_ids = sorted(int(i) for i in layer_ids)
        if len(self.layer_ids) > 16:
            raise ValueError("at most 16 hidden-capture layers")
        self.t_cap = int(t_cap)
        self.kv_capacity = int(kv_capacity)
        L = cfg.num_hidden_layers
        self._layers = (Qwen3Layer * L)()
        for i in range(L):
            self._layers[i] = Qwen3Layer(
                ptr(weights.input_norm[i]), _wptr(weights.qkv[i]), ptr(weights.q_norm[i]), ptr(weights.k_norm[i]),
                _wptr(weights.o_proj[i]), ptr(weights.post_norm[i]), _wptr(weights.gate_up[i]),
                _wptr(weights.down[i]),
            )
        self.quant_bits = weights.quant_bits
        self._q4 = None
        if self.quant_bits == 4:
            self._q4 = (Qwen3Q4Layer * L)()
            for i in range(L):
                qs = [weights.qkv[i], weights.o_proj[i], weights.gate_up[i], weights.down[i]]
                self._q4[i] = Qwen3Q4Layer(*[p for t in qs for p in (ptr(t.scales), ptr(t.biases))])
        d = Qwen3Desc()
        d.hidden, d.layers = cfg.hidden_size, L
        d.n_heads, d.n_kv_heads, d.head_dim = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        d.ffn, d.vocab = cfg.intermediate_size, cfg.vocab_size
        d.rope_theta, d.rms_eps = cfg.rope_theta, cfg.rms_norm_eps
        d.t_cap, d.kv_capacity = self.t_cap, self.kv_capacity
        d.verify_path = 1 if verify_path == "persistent" else 0
        d.n_capture = len(self.layer_ids)
        for i, l in enumerate(self.layer_ids):
            d.capture_layers[i] = l
        d.embed, d.final_norm = ptr(weights.embed), ptr(weights.final_norm)
        eq = getattr(weights, "embed_q4", None)
        if eq is not None:  # 4-bit tied LM head
            d.embed_q4_packed, d.embed_q4_scales, d.embed_q4_biases = ptr(eq.packed), ptr(eq.scales), ptr(eq.biases)
        d.layer = C.cast(self._layers, C.POINTER(Qwen3Layer))
        if self._q4 is not None:
            d.quant_bits, d.group_size = 4, 64
            d.q4_layer = C.cast(self._q4, C.POINTER(Qwen3Q4Layer))
        sizes = (C.c_size_t * 9)()
        call("dtree_qwen3_buffer_bytes", C.byref(d), sizes)
        tp = pad_rows(self.t_cap)
        dev = self.device
        bf = torch.bfloat16
        self.kv_cache = torch.zeros(L, 2, cfg.num_key_value_heads, self.kv_capacity, cfg.head_dim, dtype=bf, device=dev)
        self.h = torch.zeros(tp, cfg.hidden_size, dtype=bf, device=dev)
        self.xn = torch.zeros(tp, cfg.hidden_size, dtype=bf, device=dev)
        self.q = torch.zeros(tp, cfg.q_dim, dtype=bf, device=dev)
        self.attn = torch.zeros(tp, cfg.q_dim, dtype=bf, device=dev)
        self.act = torch.zeros(tp, cfg.intermediate_size, dtype=bf, device=dev)
        self.norm_out = torch.zeros(tp, cfg.hidden_size, dtype=bf, device=dev)
        self.capture = torch.zeros(tp, cfg.hidden_size * max(1, len(self.layer_ids)), dtype=bf, device=dev)
        self.workspace = torch.zeros(int(sizes[8]), dtype=torch.uint8, device=dev)
        for t, need in zip([self.kv_cache, self.h, self.xn, self.q, self.attn, self.act, self.norm_out, self.capture],
                           list(sizes)[:8]):
            assert t.numel() * t.element_size() >= need
        d.kv_cache, d.h, d.xn, d.q = ptr(self.kv_cache), ptr(self.h), ptr(self.xn), ptr(self.q)
        d.attn, d.act, d.norm_out, d.capture = ptr(self.attn), ptr(self.act), ptr(self.norm_out), ptr(self.capture)
        d.workspace, d.workspace_bytes = ptr(self.workspace), self.workspace.numel()
        self._desc = d
        handle = C.c_void_p()
        call("dtree_qwen3_create", C.byref(d), C.byref(handle))
        self._handle = handle

    def close(self) -> None:
        if getattr(self, "_handle", None):
            _lib.load().dtree_qwen3_destroy(self._handle)
            self._handle = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    # rows per dense prefill call: its workspace grows ~linearly with the rows
    # (about 65 KB per row at the 4B shape), longer prompts run in pieces
    max_prefill_rows = 4096
    # shorter prompts run as 128-row verify forwards: below ~a thousand rows
    # the weight stream per 128 rows costs less than the dense GEMMs' fixed
    # work (measured at the 4B shape: 256 rows 9.4 ms chained vs 19.2 ms
    # dense, 2048 rows 78 ms vs 36 ms)
    dense_prefill_min_rows = 768

    def prefill_dense(self, tokens: torch.Tensor, state: torch.Tensor, hidden_out: torch.Tensor | None,
                      next_token: torch.Tensor, norm_out: torch.Tensor | None = None) -> None:
        """Dense causal forward of ``tokens`` (int32, device) after the
        state.start cached rows (``dtree_qwen3_prefill``): K/V into the cache,
        the captured layers' hidden rows into ``hidden_out`` [n, width], the
        final-normed rows into ``norm_out`` [n, hidden] (optional) and the last
        row's argmax (or sample) into ``next_token[0]``."""
        n = int(tokens.numel())
        if n <= 0 or n > self.max_prefill_rows:
            raise ValueError(f"prefill rows must be in [1, {self.max_prefill_rows}], got {n}")
        need = int(_lib.load().dtree_qwen3_prefill_workspace_bytes(C.byref(self._desc), n))
        ws = getattr(self, "_prefill_ws", None)
        if ws is None or ws.numel() < need:
            self._prefill_ws = ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        start = int(state[0].item())
        if start + n > self.kv_capacity:
            raise ValueError(f"prompt of {start + n} rows exceeds kv_capacity {self.kv_capacity}")
        pos = torch.arange(start, start + n, dtype=torch.int32, device=self.device)
        ld = 0
        if hidden_out is not None:
            assert hidden_out.is_contiguous() and hidden_out.shape[0] >= n
            ld = int(hidden_out.shape[1])
        call("dtree_qwen3_prefill", self._handle, ptr(tokens), ptr(pos), n, ptr(state),
             ptr(hidden_out) if hidden_out is not None else None, ld,
             ptr(norm_out) if norm_out is not None else None, ptr(next_token), ptr(ws), ws.numel(), stream_ptr())

    def release_prefill_workspace(self) -> None:
        self._prefill_ws = None

    def set_sampling(self, temperature: float, seed: int) -> None:
        """Posterior tokens of later forwards: greedy (temperature < 1e-5) or
        sampled at `temperature` with Philox noise keyed by seed and step."""
        call("dtree_qwen3_set_sampling", self._handle, float(temperature), int(seed) & 0xFFFFFFFF)

    # prefix + tree keys up to which the tree attention can run one cluster
    # of <= 8 CTAs per KV head (8 x 128 keys, one pass each)
    short_attention_keys = 1024

    def set_attention_keys(self, max_keys: int) -> None:
        """Bound on prefix + tree keys of the following forwards (0: the KV
        capacity): a launch-shape hint; forwards within it give the same
        bits in either shape."""
        call("dtree_qwen3_set_attention_keys", self._handle, int(max_keys))

    def use_attention_shape(self, start: int, n_nodes: int) -> None:
        """The attention launch shape for forwards of n_nodes rows at prefix
        lengths up to `start`: one short cluster per KV head while the keys
        fit ``short_attention_keys``, else the split shape."""
        fits = start + n_nodes <= self.short_attention_keys
        self.set_attention_keys(self.short_attention_keys if fits else 0)

    def forward_tree(self, tokens: torch.Tensor, positions: torch.Tensor, anc: torch.Tensor, n_nodes: int,
                     state: torch.Tensor, posterior: torch.Tensor | None) -> None:
        """Tree-verify forward of rows [0, n_nodes) at prefix length state.start."""
        call("dtree_qwen3_forward_tree", self._handle, ptr(tokens), ptr(positions), ptr(anc), int(n_nodes),
             ptr(state), ptr(posterior), stream_ptr())

    @property
    def hidden_width(self) -> int:
        return self.cfg.hidden_size * max(1, len(self.layer_ids))

    # -- decode-session hooks (shared with the Qwen3.5 engine) ---------------
    def prefill_chunk(self, tokens, positions, anc, n: int, state, posterior) -> None:
        self.forward_tree(tokens, positions, anc, n, state, posterior)

    def verify(self, session) -> None:
        self.forward_tree(session.tree.tokens, session.tree.positions, session.tree.anc, session.cfg.n_nodes,
                          session.state, session.posterior)

    def commit_step(self, session) -> None:
        """compact_kv_caches (adapters.py:635-668); a DFlash chain keeps its
        accepted rows where they are."""
        if session.cfg.mode == "dtree":
            kernels.kv_compact(self.kv_cache, session.accepted, session.state)


@dataclass
class StepConfig:
    mode: str            # "dtree" or "dflash"
    rows: int            # draft rows (block_size - 1)
    budget: int          # tree budget (dtree) / rows (dflash)
    n_nodes: int         # tree rows per verify (root included)
    temperature: float = 0.0  # sampled drafts / posteriors above 1e-5 (runtime.py:12-19)
    seed: int = 0             # Philox key of the sampling noise


def dtree_nodes(budget: int, rows: int, vocab: int) -> int:
    """Nodes the best-first builder emits: min(budget, reachable) + root."""
    if budget <= 0 or rows <= 0:
        return 1
    k = min(budget, vocab)
    reach, level = 0, 1
    for _ in range(rows):
        level *= k
        reach += level
        if reach >= budget:
            return 1 + budget
    return 1 + min(budget, reach)


class DecodeSession:
    """Device state of one sequence decoded with DTree or DFlash on an engine."""

    def __init__(self, engine: Qwen3Engine, cfg: StepConfig, output_capacity: int, drafter, history: int = 4096):
        self.engine = engine
        self.cfg = cfg
        dev = engine.device
        self.state = kernels.new_state(dev)
        self.tree = kernels.TreeBuffers.allocate(dev)
        self.posterior = torch.zeros(DTREE_MAX_TREE, dtype=torch.int32, device=dev)
        self.accepted = torch.zeros(DTREE_MAX_TREE, dtype=torch.int32, device=dev)
        self.output = torch.zeros(int(output_capacity), dtype=torch.int32, device=dev)
        self.history = torch.zeros(int(history), dtype=torch.int32, device=dev)
        self.draft_logits = torch.zeros(max(cfg.rows, 1), engine.cfg.vocab_size, dtype=torch.float32, device=dev)
        self.target_hidden = torch.zeros(DTREE_MAX_TREE, engine.hidden_width, dtype=torch.bfloat16, device=dev)
        self.builder = (
            kernels.TreeBuilder(cfg.rows, engine.cfg.vocab_size, cfg.budget, dev) if cfg.mode == "dtree" else None
        )
        self.drafter = drafter
        self.graph: torch.cuda.CUDAGraph | None = None
        # step graphs by attention launch shape (see ``_attention_class``);
        # ``graph`` is the one captured last, None until the first capture
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.host_start = 0  # the last prefix length the host knows of

    # ------------------------------------------------------------ prefill
    def prefill(self, prompt: list[int]) -> int:
        """Causal forward of the prompt in chunks of <= t_cap rows (prefix K/V
        into the cache).  Returns the greedy first token (runtime.py:459-465)."""
        eng = self.engine
        dev = eng.device
        n = len(prompt)
        if n <= 0:
            raise ValueError("empty prompt")
        chunk = eng.t_cap
        toks = torch.tensor(prompt, dtype=torch.int32, device=dev)
        self.output[:n] = toks
        if hasattr(eng, "reset_states"):  # a new sequence starts from zero recurrent state
            eng.reset_states()
        # the prompt's sampling noise (temperature > 0) gets its own stream:
        # step -1, never used by a decode step
        self.state[2] = -1
        start = 0
        hidden_rows = []
        if hasattr(eng, "prefill_dense") and n > chunk and n >= eng.dense_prefill_min_rows:
            # prompts longer than one verify forward: one dense forward per
            # piece of <= max_prefill_rows rows (the weights stream once per
            # piece, not once per 128 rows)
            self.prompt_hidden = torch.zeros(n, eng.hidden_width, dtype=torch.bfloat16, device=dev)
            nxt = torch.zeros(1, dtype=torch.int32, device=dev)
            while start < n:
                t = min(eng.max_prefill_rows, n - start)
                self.state[0] = start
                eng.prefill_dense(toks[start:start + t].contiguous(), self.state,
                                  self.prompt_hidden[start:start + t] if eng.layer_ids else None, nxt)
                start += t
            first = int(nxt.item())
            self._after_prefill(n, first)
            return first
        while start < n:
            t = min(chunk, n - start)
            self.state[0] = start
            pos = torch.arange(start, start + t, dtype=torch.int32, device=dev)
            anc = torch.from_numpy(chain_anc_masks(t).view(np.int64)).to(dev)
            eng.prefill_chunk(toks[start:start + t].contiguous(), pos, anc, t, self.state, self.posterior)
            hidden_rows.append(eng.capture[:t].clone())
            start += t
        first = int(self.posterior[t - 1].item())  # last prompt row of the last chunk
        self.prompt_hidden = torch.cat(hidden_rows, dim=0)
        self._after_prefill(n, first)
        return first

    def _after_prefill(self, n: int, first: int) -> None:
        eng = self.engine
        # recurrent targets: remember the post-prompt states so that ``reset``
        # can restart decoding from the prompt (the KV prefix needs no copy)
        self._snapshot = eng.snapshot_states() if hasattr(eng, "snapshot_states") else None
        self.reset(n, first)
        if hasattr(self.drafter, "begin"):  # a model drafter ingests the prompt context
            self.drafter.begin(self)

    def reset(self, prompt_len: int, first_token: int) -> None:
        """Decode state right after prefill: start = prompt_len, root = first token."""
        self.state.zero_()
        self.state[0] = prompt_len
        self.host_start = prompt_len
        self.state[1] = first_token
        self.output[prompt_len] = first_token
        self.prompt_len = prompt_len
        if getattr(self, "_snapshot", None) is not None:
            self.engine.restore_states(self._snapshot)

    # ------------------------------------------------------------ one step
    def _attention_class(self) -> int:
        """1 while the next verify's keys (prefix + tree rows) fit the short
        attention shape of the engine, else 0.  The host learns the prefix
        length after each step (``host_start``); steps replayed without that
        keep the last known value.  Within the bound the two shapes give
        bit-identical attention (the same 128-key splits merged in the same
        order); a short-shape graph replayed past it stays correct with
        longer splits, rounded differently from the split shape."""
        lim = getattr(self.engine, "short_attention_keys", 0)
        return 1 if lim and self.host_start + self.cfg.n_nodes <= lim else 0

    def _set_attention_shape(self, cls: int) -> None:
        if hasattr(self.engine, "set_attention_keys"):
            self.engine.set_attention_keys(self.engine.short_attention_keys if cls == 1 else 0)

    def step(self) -> None:
        """One decode step, launched on the current stream (no host sync)."""
        eng = self.engine
        c = self.cfg
        self._set_attention_shape(self._attention_class())
        self.drafter.draft(self)
        if c.mode == "dtree":
            self.builder.build(self.draft_logits, self.state, self.tree, keep_topk=False)
        else:
            kernels.chain_build(self.draft_logits[: c.rows], self.state, self.tree, c.temperature, c.seed)
        eng.verify(self)
        kernels.accept_walk(self.tree, self.posterior, self.state, self.accepted, self.output, self.history)
        eng.commit_step(self)
        if getattr(self.drafter, "needs_hidden", False):
            kernels.gather_rows(eng.capture, self.accepted, self.state, self.target_hidden)
        kernels.step_commit(self.state)

    def capture_step(self) -> torch.cuda.CUDAGraph:
        """Record ``step`` into a CUDA graph (after one eager warm-up step has
        built every plan) for the current attention shape, dropping graphs
        captured before; replay it with ``replay``."""
        self.graphs = {}
        return self._capture(self._attention_class())

    def _capture(self, cls: int) -> torch.cuda.CUDAGraph:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.step()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = g
        self.graphs[cls] = g
        return g

    def replay(self) -> None:
        """One step: the captured graph of the current attention shape
        (captured here the first time that shape comes up), or an eager
        step before any capture."""
        if self.graph is None:
            self.graphs = {}
            self.step()
            return
        cls = self._attention_class()
        g = self.graphs.get(cls)
        if g is None:
            g = self._capture(cls)
        g.replay()

    def read_state(self) -> dict[str, int]:
        return kernels.state_dict(self.state)
