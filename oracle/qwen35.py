"""Oracle: Qwen3.5 gated-DeltaNet tree kernels, commit, and the hybrid layers.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates, in NumPy (float32 / float64 accumulation):

* ``tree_conv1d``       tree_conv1d_kernel, dtree_mlx/qwen35_tree_kernels.py:86-134
                        (wrapper :180-206): per node, the parent's conv window
                        (or the base conv state) plus the node's input, weighted
                        sum over the kernel width, SiLU, cast to the input dtype;
                        the node's window = parent window shifted by its input.
* ``tree_gated_delta``  tree_gated_delta_kernel, qwen35_tree_kernels.py:8-82
                        (wrapper :207-224): S = S_parent * g; kv = S k;
                        delta = (v - kv) beta; S += k delta; y = S q; the node's
                        stored state is S rounded to the input dtype.
* ``commit_path``       commit_qwen35_tree_path, dtree_mlx/qwen35_tree.py:708-732
                        (recurrent and conv state of the deepest accepted node).
* ``compute_g``         mlx-lm 0.31.2 ``models.gated_delta.compute_g`` (called at
                        qwen35_tree.py:292): g = exp(-exp(A_log) * softplus(a + dt_bias)).
* ``rms_norm_gated``    mlx-lm ``Qwen3NextRMSNormGated`` (custom_qwen35_model.py:25,
                        817): rms_norm(x, w) * silu(z).

The mlx-lm functions are third-party code absent from the reference tree
(mlx-lm 0.31.2, uv.lock); they are restated from their published
definitions.  The conv and delta restatements are pinned to the reference's
own known-answer tests (tests/test_qwen35_tree_kernels.py) through
``tests/golden/qwen35_tree_kernels.npz`` (``tests/golden/make_qwen35_golden.py``).
"""
from __future__ import annotations

import numpy as np


def _round(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` ("f32" or "bf16", round-to-nearest-even)."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x
    b = x.view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def tree_conv1d(qkv: np.ndarray, base: np.ndarray, weight: np.ndarray, parents, dtype: str = "f32"):
    """qkv [T, C], base [keep, C], weight [keep+1, C] -> (out [T, C], states [T, keep, C])."""
    qkv = np.asarray(qkv, np.float32)
    base = np.asarray(base, np.float32)
    weight = np.asarray(weight, np.float32)
    T, C = qkv.shape
    keep = base.shape[0]
    out = np.zeros((T, C), np.float32)
    states = np.zeros((T, keep, C), np.float32)
    for t in range(T):
        p = int(parents[t])
        window = base if p < 0 else states[p]
        conv_in = np.concatenate([window, qkv[t:t + 1]], axis=0)  # [keep+1, C]
        acc = (conv_in.astype(np.float64) * weight).sum(axis=0)
        out[t] = _round((acc / (1.0 + np.exp(-acc))).astype(np.float32), dtype)
        states[t] = conv_in[1:]
    return out, states


def tree_gated_delta(q, k, v, g, beta, state, parents, dtype: str = "f32"):
    """q, k [T, Hk, Dk]; v [T, Hv, Dv]; g, beta [T, Hv]; state [Hv, Dv, Dk]
    -> (y [T, Hv, Dv], node states [T, Hv, Dv, Dk])."""
    q, k, v = (np.asarray(a, np.float32) for a in (q, k, v))
    g, beta = np.asarray(g, np.float32), np.asarray(beta, np.float32)
    state = np.asarray(state, np.float32)
    T, Hk, Dk = k.shape
    Hv, Dv = v.shape[1:]
    rep = Hv // Hk
    y = np.zeros((T, Hv, Dv), np.float32)
    states = np.zeros((T, Hv, Dv, Dk), np.float32)
    for t in range(T):
        p = int(parents[t])
        s = (state if p < 0 else states[p]).astype(np.float64)
        kk = np.repeat(k[t], rep, axis=0).astype(np.float64)  # [Hv, Dk]
        qq = np.repeat(q[t], rep, axis=0).astype(np.float64)
        s = s * g[t][:, None, None]
        kv = np.einsum("hvd,hd->hv", s, kk)
        delta = (v[t] - kv) * beta[t][:, None]
        s = s + delta[:, :, None] * kk[:, None, :]
        y[t] = _round(np.einsum("hvd,hd->hv", s, qq).astype(np.float32), dtype)
        states[t] = _round(s.astype(np.float32), dtype)
    return y, states


def commit_path(node_states: np.ndarray, conv_node_states: np.ndarray, accepted):
    """Recurrent and conv state after accepting ``accepted`` (root first)."""
    d = int(accepted[-1])
    return node_states[d].copy(), conv_node_states[d].copy()


def compute_g(a_log, a, dt_bias):
    x = np.asarray(a, np.float64) + np.asarray(dt_bias, np.float64)
    sp = np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))
    return np.exp(-np.exp(np.asarray(a_log, np.float64)) * sp).astype(np.float32)


def sigmoid(x):
    return (1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))).astype(np.float32)


def rms_norm(x, w=None, eps: float = 1e-6):
    x = np.asarray(x, np.float64)
    y = x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    if w is not None:
        y = y * np.asarray(w, np.float64)
    return y.astype(np.float32)


def rms_norm_gated(x, z, w, eps: float = 1e-6):
    z = np.asarray(z, np.float64)
    return (rms_norm(x, w, eps).astype(np.float64) * z / (1.0 + np.exp(-z))).astype(np.float32)


# ------------------------------------------------------------ hybrid model
def apply_partial_rope(x, positions, theta: float, rot: int):
    """mlx nn.RoPE(dims=rot, traditional=False) on the first ``rot`` features
    (x [T, heads, D]); the rest pass through (custom_qwen35_model.py:745-774,
    partial_rotary_factor)."""
    import torch

    half = rot // 2
    inv = theta ** (-(torch.arange(half, dtype=torch.float64) * 2.0 / rot))
    ang = torch.as_tensor(np.asarray(positions), dtype=torch.float64)[:, None] * inv[None, :]
    cos = torch.cos(ang).float()[:, None, :]
    sin = torch.sin(ang).float()[:, None, :]
    x1, x2, rest = x[..., :half], x[..., half:rot], x[..., rot:]
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos, rest], dim=-1)


class Qwen35Oracle:
    """fp32 CPU Qwen3.5 hybrid: forward_qwen35_tree_with_hidden_states
    (qwen35_tree.py:629-705; DeltaNet :362-480 through the tree kernels above,
    gated attention :483-626), prefill (the standard sequence forward,
    custom_qwen35_model.py:823-891: no per-step state rounding) and
    commit_qwen35_tree_path (:708-732).  Node states of the tree mode are
    rounded to bf16 per node as the reference's tree kernel does for bf16
    inputs (``state_dtype="f32"``: kept in fp32, as it does for an fp32
    model); everything else is fp32 on the same bf16 weights.

    ``bf16_acts=True`` additionally rounds every activation to bf16 where a
    bf16 MLX model materializes it (projection outputs, norms, conv and
    gated-delta outputs, gates, residual adds), which separates rounding
    noise from real differences when checking a bf16 implementation."""

    def __init__(self, weights, kv_capacity: int, bf16_acts: bool = False, state_dtype: str = "bf16"):
        self.bf16_acts = bool(bf16_acts)
        # tree-mode node states are kept in the model's dtype by the
        # reference's kernel: bf16 for the bf16 engine, fp32 for an fp32 model
        self.state_dtype = state_dtype
        import torch

        self.w = weights.to("cpu") if weights.device.type != "cpu" else weights
        self.cfg = c = self.w.cfg
        self.L = [{k: (v.float() if torch.is_tensor(v) else v) for k, v in self.w.reference_layer(l).items()}
                  for l in range(c.num_hidden_layers)]
        self.cap = int(kv_capacity)
        keep = c.linear_conv_kernel_dim - 1
        self.k = {l: torch.zeros(c.num_key_value_heads, self.cap, c.head_dim)
                  for l in range(c.num_hidden_layers) if not c.is_linear(l)}
        self.v = {l: torch.zeros_like(t) for l, t in self.k.items()}
        self.conv = {l: np.zeros((keep, c.conv_dim), np.float32) for l in range(c.num_hidden_layers) if c.is_linear(l)}
        self.rec = {l: np.zeros((c.linear_num_value_heads, c.linear_value_head_dim, c.linear_key_head_dim),
                                np.float32) for l in self.conv}
        self.embed = self.w.embed.float()
        self.final_norm = self.w.final_norm.float()
        self.pending = None

    # -------------------------------------------------------------- layers
    def _r(self, x):
        """bf16 rounding of an activation (bf16_acts mode only)."""
        import torch

        if not self.bf16_acts:
            return x
        if isinstance(x, np.ndarray):
            return _round(x, "bf16")
        return x.to(torch.bfloat16).float()

    def _rms(self, x, w):
        import torch

        return self._r(x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.rms_norm_eps) * w)

    def _add(self, h, y):
        return self._r(h + self._r(y))

    def _mlp(self, L, h):
        import torch

        x = self._rms(h, L["post_attention_layernorm"])
        g = self._r(x @ L["gate_proj"].t())
        u = self._r(x @ L["up_proj"].t())
        act = self._r(self._r(g * self._r(torch.sigmoid(g))) * u)
        return self._add(h, act @ L["down_proj"].t())

    def _linear(self, l, h, parents, tree: bool):
        import torch

        c, L = self.cfg, self.L[l]
        T = h.shape[0]
        x = self._rms(h, L["input_layernorm"])
        r = self._r
        qkv = r((x @ L["in_proj_qkv"].t()).numpy())
        z = r((x @ L["in_proj_z"].t()).numpy())
        b = r((x @ L["in_proj_b"].t()).numpy())
        a = r((x @ L["in_proj_a"].t()).numpy())
        act_dt = "bf16" if self.bf16_acts else "f32"
        conv_out, conv_states = tree_conv1d(qkv, self.conv[l], L["conv_weight"].numpy(), parents, dtype=act_dt)
        kd, Dk, Dv = c.key_dim, c.linear_key_head_dim, c.linear_value_head_dim
        q = r(r(rms_norm(conv_out[:, :kd].reshape(T, -1, Dk))) / Dk)
        k = r(r(rms_norm(conv_out[:, kd:2 * kd].reshape(T, -1, Dk))) / np.sqrt(Dk))
        v = conv_out[:, 2 * kd:].reshape(T, -1, Dv)
        if self.bf16_acts:
            x_dt = r(a + L["dt_bias"].numpy())
            sp = r(np.where(x_dt > 20.0, x_dt, np.log1p(np.exp(np.minimum(x_dt, 20.0)))).astype(np.float32))
            g = np.exp(-np.exp(L["A_log"].numpy().astype(np.float64)) * sp).astype(np.float32)
        else:
            g = compute_g(L["A_log"].numpy(), a, L["dt_bias"].numpy())
        beta = r(sigmoid(b))
        y, states = tree_gated_delta(q, k, v, g, beta, self.rec[l], parents,
                                     dtype="bf16" if ((tree and self.state_dtype == "bf16") or self.bf16_acts)
                                     else "f32")
        if not tree:  # sequence mode: the state is not rounded per step
            _, states = tree_gated_delta(q, k, v, g, beta, self.rec[l], parents, dtype="f32")
        zz = z.reshape(T, -1, Dv)
        if self.bf16_acts:
            n = r(rms_norm(y, L["norm"].numpy(), c.rms_norm_eps))
            sz = r((zz / (1.0 + np.exp(-zz.astype(np.float64)))).astype(np.float32))
            o = r(n * sz).reshape(T, -1)
        else:
            o = rms_norm_gated(y, zz, L["norm"].numpy(), c.rms_norm_eps).reshape(T, -1)
        h = self._add(h, torch.from_numpy(o) @ L["out_proj"].t())
        return self._mlp(L, h), (conv_states, states)

    def _attn(self, l, h, positions, mask, past: int):
        import math

        import torch

        c, L = self.cfg, self.L[l]
        T, D = h.shape[0], c.head_dim
        x = self._rms(h, L["input_layernorm"])
        r = self._r
        qg = r(x @ L["q_proj"].t()).view(T, c.num_attention_heads, 2 * D)
        q, gate = qg[..., :D], qg[..., D:].reshape(T, -1)
        k = r(x @ L["k_proj"].t()).view(T, c.num_key_value_heads, D)
        v = r(x @ L["v_proj"].t()).view(T, c.num_key_value_heads, D)
        rot = int(round(D * c.partial_rotary_factor))
        q = r(apply_partial_rope(self._rms(q, L["q_norm"]), positions, c.rope_theta, rot))
        k = r(apply_partial_rope(self._rms(k, L["k_norm"]), positions, c.rope_theta, rot))
        self.k[l][:, past:past + T] = k.transpose(0, 1)
        self.v[l][:, past:past + T] = v.transpose(0, 1)
        rep = c.num_attention_heads // c.num_key_value_heads
        keys = self.k[l][:, :past + T].repeat_interleave(rep, dim=0)
        vals = self.v[l][:, :past + T].repeat_interleave(rep, dim=0)
        s = (q.transpose(0, 1) @ keys.transpose(1, 2)) / math.sqrt(D)
        s = s.masked_fill(~torch.as_tensor(np.asarray(mask))[None], float("-inf"))
        o = r((torch.softmax(s, dim=-1) @ vals).transpose(0, 1).reshape(T, -1))
        h = self._add(h, r(o * r(torch.sigmoid(gate))) @ L["o_proj"].t())
        return self._mlp(L, h)

    # ------------------------------------------------------------ forward
    def forward(self, tokens, positions, parents, mask, past: int, tree: bool, layer_ids=()):
        """Returns (norm_hidden [T, H], verifier_hidden [T, H*n]); tree=True keeps
        per-node states pending for ``commit``, tree=False (chain) advances the
        conv / recurrent states to the last token."""
        import torch

        c = self.cfg
        h = self.embed[torch.as_tensor(np.asarray(tokens), dtype=torch.long)]
        picked, pending = [], {}
        for l in range(c.num_hidden_layers):
            if c.is_linear(l):
                h, (cs, rs) = self._linear(l, h, parents, tree)
                pending[l] = (cs, rs)
                if not tree:
                    self.conv[l] = cs[-1].copy()
                    self.rec[l] = rs[-1].copy()
            else:
                h = self._attn(l, h, positions, mask, past)
            if l in set(layer_ids):
                picked.append(h.clone())
        self.pending = (past, pending) if tree else None
        norm_h = self._rms(h, self.final_norm)
        return norm_h, (torch.cat(picked, dim=-1) if picked else h[:, :0])

    def prefill(self, tokens, past: int = 0):
        T = len(tokens)
        mask = np.ones((T, past + T), dtype=bool)
        mask[:, past:] = np.tril(np.ones((T, T), dtype=bool))
        parents = np.arange(-1, T - 1)
        return self.forward(tokens, np.arange(past, past + T), parents, mask, past, tree=False)

    def lm_head_logits(self, norm_h):
        return norm_h @ self.embed.t()

    def commit(self, accepted):
        """commit_qwen35_tree_path: KV of the accepted nodes moves to
        past..past+n-1; DeltaNet layers take the deepest node's states."""
        past, pending = self.pending
        acc = list(int(i) for i in accepted)
        for l in self.k:
            src = [past + i for i in acc]
            self.k[l][:, past:past + len(acc)] = self.k[l][:, src].clone()
            self.v[l][:, past:past + len(acc)] = self.v[l][:, src].clone()
        for l, (cs, rs) in pending.items():
            self.conv[l], self.rec[l] = commit_path(rs, cs, acc)[::-1]
        self.pending = None
