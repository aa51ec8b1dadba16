"""Device-resident Qwen3.5 hybrid verify engine (``dtree_qwen35_*``).

Owns the C model handle and the buffers it runs on: the full-attention KV
cache, the DeltaNet conv / recurrent states, activations and the per-layer
DeltaNet projections the commit reads back.  ``forward`` runs a tree verify
(mode 0) or a prefill chunk (mode 1, chain parents); ``commit`` applies
commit_qwen35_tree_path (dtree_mlx/qwen35_tree.py:708-732) for the accepted
path on the device.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import (DTREE_MAX_TREE, QWEN35_BUFFERS, Qwen35AttnLayer, Qwen35Desc, Qwen35LinearLayer, call, ptr,
                   stream_ptr)
from .synthetic import Qwen35Weights


class Qwen35Engine:
    def __init__(self, weights: Qwen35Weights, kv_capacity: int, layer_ids=(), t_cap: int = DTREE_MAX_TREE):
        cfg = weights.cfg
        if weights.device.type != "cuda":
            raise ValueError("engine weights must live on a CUDA device")
        self.cfg, self.weights, self.device = cfg, weights, weights.device
        self.layer_ids = sorted(int(i) for i in layer_ids)
        self.kv_capacity, self.t_cap = int(kv_capacity), int(t_cap)
        lin = [L for l, L in enumerate(weights.layers) if cfg.is_linear(l)]
        att = [L for l, L in enumerate(weights.layers) if not cfg.is_linear(l)]
        self._lin = (Qwen35LinearLayer * max(1, len(lin)))()
        for i, L in enumerate(lin):
            self._lin[i] = Qwen35LinearLayer(*[ptr(L[k]) for k in ("input_norm", "in_proj", "conv_weight", "norm",
                                                                    "out_proj", "post_norm", "gate_up", "down")])
        self._att = (Qwen35AttnLayer * max(1, len(att)))()
        for i, L in enumerate(att):
            self._att[i] = Qwen35AttnLayer(*[ptr(L[k]) for k in ("input_norm", "qkv", "q_norm", "k_norm", "o_proj",
                                                                  "post_norm", "gate_up", "down")])
        d = Qwen35Desc()
        d.hidden, d.layers, d.full_attention_interval = cfg.hidden_size, cfg.num_hidden_layers, \
            cfg.full_attention_interval
        d.ffn, d.vocab = cfg.intermediate_size, cfg.vocab_size
        d.n_heads, d.n_kv_heads, d.head_dim = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        d.rope_theta, d.partial_rotary_factor, d.rms_eps = cfg.rope_theta, cfg.partial_rotary_factor, \
            cfg.rms_norm_eps
        d.lin_k_heads, d.lin_v_heads = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        d.lin_k_dim, d.lin_v_dim = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        d.conv_kernel = cfg.linear_conv_kernel_dim
        d.t_cap, d.kv_capacity = self.t_cap, self.kv_capacity
        d.n_capture = len(self.layer_ids)
        for i, l in enumerate(self.layer_ids):
            d.capture_layers[i] = l
        d.embed, d.final_norm = ptr(weights.embed), ptr(weights.final_norm)
        d.linear_layers = C.cast(self._lin, C.POINTER(Qwen35LinearLayer))
        d.attn_layers = C.cast(self._att, C.POINTER(Qwen35AttnLayer))
        d.a_log, d.dt_bias = ptr(weights.a_log), ptr(weights.dt_bias)
        sizes = (C.c_size_t * 14)()
        call("dtree_qwen35_buffer_bytes", C.byref(d), sizes)
        self.buffers = {}
        for name, n in zip(QWEN35_BUFFERS, sizes):
            dt = torch.float32 if name == "rec_state" else (torch.uint8 if name == "workspace" else torch.bfloat16)
            el = torch.tensor([], dtype=dt).element_size()
            self.buffers[name] = torch.zeros(max(1, (int(n) + el - 1) // el), dtype=dt, device=self.device)
            setattr(d, name, ptr(self.buffers[name]))
        d.workspace_bytes = self.buffers["workspace"].numel()
        n_lin, n_att = cfg.n_linear, cfg.n_attn
        keep = cfg.linear_conv_kernel_dim - 1
        self.kv_cache = self.buffers["kv_cache"][: n_att * 2 * cfg.num_key_value_heads * self.kv_capacity *
                                                 cfg.head_dim].view(n_att, 2, cfg.num_key_value_heads,
                                                                     self.kv_capacity, cfg.head_dim)
        self.conv_state = self.buffers["conv_state"][: n_lin * keep * cfg.conv_dim].view(n_lin, keep, cfg.conv_dim)
        self.rec_state = self.buffers["rec_state"][: n_lin * cfg.linear_num_value_heads *
                                                   cfg.linear_value_head_dim * cfg.linear_key_head_dim].view(
            n_lin, cfg.linear_num_value_heads, cfg.linear_value_head_dim, cfg.linear_key_head_dim)
        tp = 16 if self.t_cap <= 16 else 32 if self.t_cap <= 32 else 64 if self.t_cap <= 64 else 128
        self.norm_out = self.buffers["norm_out"][: tp * cfg.hidden_size].view(tp, cfg.hidden_size)
        cw = cfg.hidden_size * max(1, len(self.layer_ids))
        self.capture = self.buffers["capture"][: tp * cw].view(tp, cw)
        self._desc = d
        handle = C.c_void_p()
        call("dtree_qwen35_create", C.byref(d), C.byref(handle))
        self._handle = handle

    def close(self) -> None:
        if getattr(self, "_handle", None):
            _lib.load().dtree_qwen35_destroy(self._handle)
            self._handle = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def forward(self, tokens, positions, parents, anc, n_nodes: int, state, posterior=None, mode: int = 0) -> None:
        call("dtree_qwen35_forward", self._handle, ptr(tokens), ptr(positions), ptr(parents), ptr(anc),
             int(n_nodes), int(mode), ptr(state), ptr(posterior), stream_ptr())

    max_prefill_rows = 4096  # rows per dense prefill call (workspace ~100 KB per row at the 9B shape)
    # every prompt longer than one verify forward runs dense: the 128-row
    # sequence forwards cost ~21 ms each at the 9B shape (tree kernels on a
    # 128-node chain) against 70 ms for a whole 2048-row dense prefill
    dense_prefill_min_rows = 129

    def prefill_dense(self, tokens: torch.Tensor, state: torch.Tensor, hidden_out: torch.Tensor | None,
                      next_token: torch.Tensor, norm_out: torch.Tensor | None = None) -> None:
        """Dense causal forward of ``tokens`` after the state.start cached rows
        (``dtree_qwen35_prefill``): K/V of the attention layers into the
        cache, every DeltaNet layer's conv / recurrent state advanced to the
        last row, captured hiddens into ``hidden_out``, the final-normed rows
        into ``norm_out`` (optional), the next token into ``next_token[0]``."""
        n = int(tokens.numel())
        if n <= 0 or n > self.max_prefill_rows:
            raise ValueError(f"prefill rows must be in [1, {self.max_prefill_rows}], got {n}")
        need = int(_lib.load().dtree_qwen35_prefill_workspace_bytes(C.byref(self._desc), n))
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
        call("dtree_qwen35_prefill", self._handle, ptr(tokens), ptr(pos), n, ptr(state),
             ptr(hidden_out) if hidden_out is not None else None, ld,
             ptr(norm_out) if norm_out is not None else None, ptr(next_token), ptr(ws), ws.numel(), stream_ptr())

    def release_prefill_workspace(self) -> None:
        self._prefill_ws = None

    def set_sampling(self, temperature: float, seed: int) -> None:
        """As Qwen3Engine.set_sampling."""
        call("dtree_qwen35_set_sampling", self._handle, float(temperature), int(seed) & 0xFFFFFFFF)

    def commit(self, parents, accepted, state) -> None:
        call("dtree_qwen35_commit", self._handle, ptr(parents), ptr(accepted), ptr(state), stream_ptr())

    def reset_states(self) -> None:
        """Fresh sequence: zero conv / recurrent states (make_cache, adapters.py:216-240)."""
        self.conv_state.zero_()
        self.rec_state.zero_()

    def snapshot_states(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Copy of the DeltaNet conv / recurrent states (snapshot_linear_caches,
        custom_qwen35_model.py:1099-1109)."""
        return self.conv_state.clone(), self.rec_state.clone()

    def restore_states(self, snap) -> None:
        """restore_linear_caches (custom_qwen35_model.py:1111-1121)."""
        self.conv_state.copy_(snap[0])
        self.rec_state.copy_(snap[1])

    @property
    def hidden_width(self) -> int:
        return self.cfg.hidden_size * max(1, len(self.layer_ids))

    # -- decode-session hooks (same as the Qwen3 engine's) -------------------
    def prefill_chunk(self, tokens, positions, anc, n: int, state, posterior) -> None:
        """Sequence forward (mode 1): chain parents, states advance."""
        parents = torch.arange(-1, n - 1, dtype=torch.int32, device=self.device)
        self.forward(tokens, positions, parents, anc, n, state, posterior, mode=1)

    def verify(self, session) -> None:
        t = session.tree
        self.forward(t.tokens, t.positions, t.parents, t.anc, session.cfg.n_nodes, session.state,
                     session.posterior, mode=0)

    def commit_step(self, session) -> None:
        """commit_qwen35_tree_path for the accepted path (DTree and DFlash)."""
        self.commit(session.tree.parents, session.accepted, session.state)
