"""Torch-facing wrappers of the C-ABI kernels (device tensors in, device tensors out).

Each wrapper validates shapes/dtypes/devices on the host, then calls the
``libdtree_b200`` entry point on the current CUDA stream.  Nothing here
computes on the CPU: a missing library or a non-CUDA tensor raises.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._lib import DTREE_MASK_WORDS, DTREE_MAX_TREE, STEP_STATE_FIELDS, call, ptr, stream_ptr

STATE_LEN = len(STEP_STATE_FIELDS)


def _cuda(t: torch.Tensor, name: str, dtype=None):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must have dtype {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def new_state(device, start: int = 0, root_token: int = 0) -> torch.Tensor:
    """Device ``dtree_step_state`` as an int32[8] tensor."""
    s = torch.zeros(STATE_LEN, dtype=torch.int32, device=device)
    s[0] = start
    s[1] = root_token
    return s


def state_dict(state: torch.Tensor) -> dict[str, int]:
    vals = state.tolist()
    return dict(zip(STEP_STATE_FIELDS, vals))


@dataclass
class TreeBuffers:
    """Device outputs of tree construction (capacity DTREE_MAX_TREE nodes)."""

    tokens: torch.Tensor     # int32 [cap]
    parents: torch.Tensor    # int32 [cap]
    depths: torch.Tensor     # int32 [cap]
    positions: torch.Tensor  # int32 [cap]
    anc: torch.Tensor        # int64 [cap, 2] (uint64 bit patterns)

    @classmethod
    def allocate(cls, device, cap: int = DTREE_MAX_TREE) -> "TreeBuffers":
        z = lambda *s, dt=torch.int32: torch.zeros(*s, dtype=dt, device=device)  # noqa: E731
        return cls(z(cap), z(cap), z(cap), z(cap), z(cap, DTREE_MASK_WORDS, dt=torch.int64))


class TreeBuilder:
    """Device best-first tree construction (build_dtree_tree, dtree_runtime.py:82-163)."""

    def __init__(self, rows: int, vocab: int, budget: int, device):
        self.rows, self.vocab, self.budget = int(rows), int(vocab), int(budget)
        nbytes = _lib.load().dtree_tree_build_workspace_bytes(self.rows, self.vocab, self.budget)
        self.workspace = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        self.topk = min(self.budget, self.vocab)
        self.top_ids = torch.zeros(max(self.rows, 1), max(self.topk, 1), dtype=torch.int32, device=device)
        self.top_lp = torch.zeros(max(self.rows, 1), max(self.topk, 1), dtype=torch.float32, device=device)

    def build(self, draft_logits: torch.Tensor, state: torch.Tensor, out: TreeBuffers, keep_topk: bool = True):
        _cuda(draft_logits, "draft_logits", torch.float32)
        if tuple(draft_logits.shape) != (self.rows, self.vocab):
            raise ValueError(f"draft_logits must be [{self.rows}, {self.vocab}]")
        _cuda(state, "state", torch.int32)
        call(
            "dtree_tree_build",
            ptr(draft_logits),
            self.rows,
            self.vocab,
            self.budget,
            ptr(state),
            ptr(self.workspace),
            self.workspace.numel(),
            ptr(out.tokens),
            ptr(out.parents),
            ptr(out.depths),
            ptr(out.positions),
            ptr(out.anc),
            ptr(self.top_ids) if (keep_topk and self.topk > 0) else None,
            ptr(self.top_lp) if (keep_topk and self.topk > 0) else None,
            stream_ptr(),
        )


def tree_from_topk(top_ids: torch.Tensor, top_lp: torch.Tensor, budget: int, state: torch.Tensor,
                   out: TreeBuffers) -> None:
    _cuda(top_ids, "top_ids", torch.int32)
    _cuda(top_lp, "top_lp", torch.float32)
    rows, k = top_ids.shape
    call("dtree_tree_from_topk", ptr(top_ids), ptr(top_lp), rows, k, budget, ptr(state), ptr(out.tokens),
         ptr(out.parents), ptr(out.depths), ptr(out.positions), ptr(out.anc), stream_ptr())


def chain_build(draft_logits: torch.Tensor, state: torch.Tensor, out: TreeBuffers, temperature: float = 0.0,
                seed: int = 0) -> None:
    """DFlash chain: drafted token of row i = argmax (temperature < 1e-5) or a
    draw from softmax(row / temperature) (sample_tokens, runtime.py:12-19)."""
    _cuda(draft_logits, "draft_logits", torch.float32)
    rows, vocab = draft_logits.shape
    if temperature < 1e-5:
        call("dtree_chain_build", ptr(draft_logits), rows, vocab, ptr(state), ptr(out.tokens), ptr(out.parents),
             ptr(out.depths), ptr(out.positions), ptr(out.anc), stream_ptr())
    else:
        call("dtree_chain_sample", ptr(draft_logits), rows, vocab, float(temperature), int(seed) & 0xFFFFFFFF,
             ptr(state), ptr(out.tokens), ptr(out.parents), ptr(out.depths), ptr(out.positions), ptr(out.anc),
             stream_ptr())


def plant_draft_logits(out: torch.Tensor, seed: int, state: torch.Tensor, continuation: torch.Tensor | None,
                       p_correct: float) -> None:
    _cuda(out, "out", torch.float32)
    rows, vocab = out.shape
    cont_len = 0 if continuation is None else int(continuation.numel())
    if continuation is not None:
        _cuda(continuation, "continuation", torch.int32)
    call("dtree_plant_draft_logits", ptr(out), rows, vocab, int(seed) & 0xFFFFFFFF, ptr(state), ptr(continuation),
         cont_len, float(p_correct), stream_ptr())


def accept_walk(tree: TreeBuffers, posterior: torch.Tensor, state: torch.Tensor, accepted: torch.Tensor,
                output_tokens: torch.Tensor, history: torch.Tensor | None = None) -> None:
    _cuda(posterior, "posterior", torch.int32)
    _cuda(accepted, "accepted", torch.int32)
    _cuda(output_tokens, "output_tokens", torch.int32)
    call("dtree_accept_walk", ptr(tree.tokens), ptr(tree.parents), ptr(posterior), ptr(state), ptr(accepted),
         ptr(output_tokens), output_tokens.numel(), ptr(history), 0 if history is None else history.numel(),
         stream_ptr())


def kv_compact(kv_cache: torch.Tensor, accepted: torch.Tensor, state: torch.Tensor) -> None:
    """kv_cache: [layers, 2, kv_heads, capacity, head_dim] bf16."""
    _cuda(kv_cache, "kv_cache", torch.bfloat16)
    layers, two, kvh, cap, hd = kv_cache.shape
    assert two == 2
    call("dtree_kv_compact", ptr(kv_cache), layers, kvh, cap, hd, ptr(accepted), ptr(state), stream_ptr())


def gather_rows(src: torch.Tensor, accepted: torch.Tensor, state: torch.Tensor, dst: torch.Tensor) -> None:
    _cuda(src, "src")
    _cuda(dst, "dst")
    row_bytes = src.stride(0) * src.element_size()
    call("dtree_gather_rows", ptr(src), row_bytes, ptr(accepted), ptr(state), ptr(dst), dst.shape[0], stream_ptr())


def step_commit(state: torch.Tensor) -> None:
    call("dtree_step_commit", ptr(state), stream_ptr())


_ws_cache: dict[tuple, torch.Tensor] = {}


def _workspace(key, nbytes: int, device) -> torch.Tensor:
    t = _ws_cache.get(key)
    if t is None or t.numel() < nbytes or t.device != torch.device(device):
        t = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _ws_cache[key] = t
    return t


def linear_bf16(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """x [t_pad, K] bf16 @ w[N, K]^T -> [t_pad, N] bf16 via the tcgen05 GEMM."""
    _cuda(x, "x", torch.bfloat16)
    _cuda(w, "w", torch.bfloat16)
    t_pad, k = x.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty(t_pad, n, dtype=torch.bfloat16, device=x.device)
    nbytes = int(_lib.load().dtree_linear_workspace_bytes(t_pad, n))
    ws = _workspace(("gemm", t_pad), nbytes, x.device)
    call("dtree_linear_bf16", ptr(x), t_pad, k, ptr(w), n, ptr(out), ptr(ws), ws.numel(), 0, stream_ptr())
    return out


def linear_q4(x: torch.Tensor, w, out: torch.Tensor | None = None, split_k: int = 0) -> torch.Tensor:
    """x [t_pad, K] bf16 @ dequant(w)^T -> [t_pad, N] bf16, w a ``Q4Tensor``
    (MLX affine 4-bit, group 64): mx.quantized_matmul(transpose=True)."""
    _cuda(x, "x", torch.bfloat16)
    _cuda(w.packed, "w.packed", torch.int32)
    _cuda(w.scales, "w.scales", torch.bfloat16)
    _cuda(w.biases, "w.biases", torch.bfloat16)
    t_pad, k = x.shape
    n, kw = w.shape
    if kw != k:
        raise ValueError(f"x has K={k} but w has K={kw}")
    if out is None:
        out = torch.empty(t_pad, n, dtype=torch.bfloat16, device=x.device)
    nbytes = int(_lib.load().dtree_linear_q4_workspace_bytes(t_pad, n, k))
    ws = _workspace(("gemm_q4", t_pad, n, k), nbytes, x.device)
    call("dtree_linear_q4", ptr(x), t_pad, k, ptr(w.packed), ptr(w.scales), ptr(w.biases), n, ptr(out), ptr(ws),
         ws.numel(), int(split_k), stream_ptr())
    return out


def lm_head_sample(h: torch.Tensor, embed: torch.Tensor, n_rows: int, temperature: float, seed: int,
                   state: torch.Tensor, out: torch.Tensor | None = None):
    """Token per row t < n_rows drawn from softmax(bf16(h[t] . embed) / T)
    (Gumbel-max, Philox keyed by seed and state.step); T < 1e-5: argmax."""
    _cuda(h, "h", torch.bfloat16)
    _cuda(embed, "embed", torch.bfloat16)
    _cuda(state, "state", torch.int32)
    t_pad, hidden = h.shape
    vocab = embed.shape[0]
    if out is None:
        out = torch.empty(n_rows, dtype=torch.int32, device=h.device)
    nbytes = int(_lib.load().dtree_lm_head_workspace_bytes(t_pad))
    ws = _workspace(("lmhead", t_pad), nbytes, h.device)
    call("dtree_lm_head_sample", ptr(h), t_pad, n_rows, hidden, ptr(embed), vocab, float(temperature),
         int(seed) & 0xFFFFFFFF, ptr(state), ptr(out), ptr(ws), ws.numel(), stream_ptr())
    return out


def lm_head_argmax(h: torch.Tensor, embed: torch.Tensor, n_rows: int, out: torch.Tensor | None = None):
    """argmax_v bf16(h[t] . embed[v]) for t < n_rows (first index on ties)."""
    _cuda(h, "h", torch.bfloat16)
    _cuda(embed, "embed", torch.bfloat16)
    t_pad, hidden = h.shape
    vocab = embed.shape[0]
    if out is None:
        out = torch.empty(n_rows, dtype=torch.int32, device=h.device)
    nbytes = int(_lib.load().dtree_lm_head_workspace_bytes(t_pad))
    ws = _workspace(("lmhead", t_pad), nbytes, h.device)
    call("dtree_lm_head_argmax", ptr(h), t_pad, n_rows, hidden, ptr(embed), vocab, ptr(out), ptr(ws), ws.numel(),
         stream_ptr())
    return out


def tree_attention(q: torch.Tensor, k_plane: torch.Tensor, v_plane: torch.Tensor, state: torch.Tensor,
                   anc: torch.Tensor, n_nodes: int, n_q_heads: int, splits: int = 0,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """Tree-masked attention of n_nodes query rows q [n_nodes, n_q_heads*hd]
    against K/V planes [n_kv_heads, kv_cap, hd] (prefix [0, start) plus the
    tree slots start..start+n_nodes-1), ancestor masks anc [n_nodes, 2]."""
    _cuda(q, "q", torch.bfloat16)
    _cuda(k_plane, "k_plane", torch.bfloat16)
    _cuda(v_plane, "v_plane", torch.bfloat16)
    n_kv_heads, kv_cap, hd = k_plane.shape
    if out is None:
        out = torch.empty(n_nodes, n_q_heads * hd, dtype=torch.bfloat16, device=q.device)
    nbytes = int(_lib.load().dtree_tree_attention_workspace_bytes(n_q_heads, n_nodes, hd, splits))
    ws = _workspace(("attn", n_q_heads, n_nodes, hd, splits), nbytes, q.device)
    call("dtree_tree_attention", ptr(q), q.stride(0), ptr(k_plane), ptr(v_plane), kv_cap, n_q_heads, n_kv_heads, hd,
         n_nodes, ptr(state), ptr(anc), ptr(out), splits, ptr(ws), ws.numel(), stream_ptr())
    return out


# ------------------------------------------------- Qwen3.5 DeltaNet kernels
_DT = {torch.float32: 0, torch.bfloat16: 1}


def _dtype_code(t: torch.Tensor, name: str) -> int:
    if t.dtype not in _DT:
        raise TypeError(f"{name} must be float32 or bfloat16, got {t.dtype}")
    return _DT[t.dtype]


def tree_conv1d(qkv: torch.Tensor, base: torch.Tensor, weight: torch.Tensor, parents: torch.Tensor,
                want_states: bool = False):
    """tree_conv1d_kernel (qwen35_tree_kernels.py:180-206): qkv [T, C],
    base [keep, C], weight [keep+1, C] -> (conv_out [T, C], states or None)."""
    for t, n in ((qkv, "qkv"), (base, "base"), (weight, "weight")):
        _cuda(t, n, qkv.dtype)
    _cuda(parents, "parents", torch.int32)
    T, C = qkv.shape
    keep = base.shape[0]
    out = torch.empty(T, C, dtype=qkv.dtype, device=qkv.device)
    states = torch.empty(T, keep, C, dtype=qkv.dtype, device=qkv.device) if want_states else None
    call("dtree_tree_conv1d", ptr(qkv), qkv.stride(0), ptr(base), ptr(weight), ptr(parents), T, C, keep,
         _dtype_code(qkv, "qkv"), ptr(out), ptr(states), stream_ptr())
    return out, states


def tree_gated_delta(q, k, v, g, beta, state, parents, want_states: bool = False):
    """tree_gated_delta_kernel (qwen35_tree_kernels.py:207-224): q, k
    [T, Hk, Dk]; v [T, Hv, Dv]; g f32 [T, Hv]; beta [T, Hv]; state
    [Hv, Dv, Dk] -> (y [T, Hv, Dv], node states or None)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (beta, "beta")):
        _cuda(t, n, q.dtype)
    _cuda(g, "g", torch.float32)
    _cuda(state, "state")
    _cuda(parents, "parents", torch.int32)
    T, Hk, Dk = k.shape
    Hv, Dv = v.shape[1:]
    y = torch.empty(T, Hv, Dv, dtype=q.dtype, device=q.device)
    ns = torch.empty(T, Hv, Dv, Dk, dtype=state.dtype, device=q.device) if want_states else None
    call("dtree_tree_gated_delta", ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), ptr(state), ptr(parents), T, Hk, Hv,
         Dk, Dv, _dtype_code(q, "q"), _dtype_code(state, "state"), ptr(y), ptr(ns), stream_ptr())
    return y, ns


def gated_delta_commit(q, k, v, g, beta, accepted: torch.Tensor, st: torch.Tensor, state: torch.Tensor) -> None:
    """Advance ``state`` in place along accepted[0:st.n_accepted] (commit_qwen35_tree_path)."""
    _cuda(accepted, "accepted", torch.int32)
    _cuda(st, "state struct", torch.int32)
    T, Hk, Dk = k.shape
    Hv, Dv = v.shape[1:]
    call("dtree_gated_delta_commit", ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), ptr(accepted), ptr(st), T, Hk, Hv,
         Dk, Dv, _dtype_code(q, "q"), _dtype_code(state, "state"), ptr(state), stream_ptr())


def conv_state_commit(qkv: torch.Tensor, parents: torch.Tensor, accepted: torch.Tensor, st: torch.Tensor,
                      base: torch.Tensor) -> None:
    """base <- the conv window of the deepest accepted node (in place)."""
    T, C = qkv.shape
    call("dtree_conv_state_commit", ptr(qkv), qkv.stride(0), ptr(parents), ptr(accepted), ptr(st), T, C,
         base.shape[0], _dtype_code(qkv, "qkv"), ptr(base), stream_ptr())
