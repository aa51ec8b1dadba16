"""Tree attention (dtree_tree_attention) against a plain PyTorch fp32 reference.

The reference is the masked scaled_dot_product_attention of
dtree_mlx/qwen3_tree.py:67-76 with the ancestor mask of
dtree_mlx/dtree_runtime.py:190-191: every prefix key is visible, tree slot j
is visible to node t iff j is t or one of its ancestors.  Cache rows past the
live keys are filled with NaN: they must not reach the output.
Tolerance: max |out - ref| <= 2e-2 (bf16 probabilities and bf16 output).
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _random_tree(n: int, gen: torch.Generator) -> tuple[list[int], torch.Tensor]:
    """Random parents (node i > 0 under a uniform earlier node): ancestor
    masks as Python ints and as the [n, 2] int64 words the kernels read."""
    parents = [-1] + [int(torch.randint(0, i, (1,), generator=gen)) for i in range(1, n)]
    masks = []
    for i in range(n):
        m = 1 << i
        p = parents[i]
        while p >= 0:
            m |= 1 << p
            p = parents[p]
        masks.append(m)
    words = []
    for m in masks:
        lo, hi = m & ((1 << 64) - 1), m >> 64
        words.append([lo - (1 << 64) if lo >= 1 << 63 else lo, hi - (1 << 64) if hi >= 1 << 63 else hi])
    return masks, torch.tensor(words, dtype=torch.int64)


def _reference(q, k_plane, v_plane, start, n, masks, n_q_heads):
    n_kv, _, hd = k_plane.shape
    group = n_q_heads // n_kv
    L = start + n
    k = k_plane[:, :L].float()
    v = v_plane[:, :L].float()
    vis = torch.ones(n, L, dtype=torch.bool, device=q.device)
    for t in range(n):
        m = masks[t]
        for j in range(n):
            vis[t, start + j] = bool((m >> j) & 1)
    qf = q.float().view(n, n_q_heads, hd)
    out = torch.empty(n, n_q_heads, hd, device=q.device)
    for h in range(n_q_heads):
        s = qf[:, h] @ k[h // group].T / math.sqrt(hd)
        s = s.masked_fill(~vis, float("-inf"))
        out[:, h] = torch.softmax(s, dim=-1) @ v[h // group]
    return out.view(n, n_q_heads * hd)


@pytest.mark.parametrize("heads", [(32, 8, 128), (8, 4, 64), (16, 4, 256)])
@pytest.mark.parametrize("start,n,splits", [(0, 1, 0), (5, 25, 0), (200, 64, 0), (2048, 25, 0), (3000, 25, 0),
                                            (2048, 25, 3), (777, 7, 0), (2048, 65, 0), (8192, 65, 0),
                                            (8192, 25, 0), (513, 100, 0), (8192, 128, 0), (0, 128, 0),
                                            (2048, 25, 16), (2048, 25, 32), (100, 25, 16), (1500, 64, 13)])
def test_tree_attention_matches_fp32(lib, heads, start, n, splits):
    from dtree_mlx_b200 import kernels

    n_q, n_kv, hd = heads
    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(start * 131 + n * 7 + hd + splits)
    cap = start + n + 300
    k_plane = torch.randn(n_kv, cap, hd, generator=gen).to(torch.bfloat16)
    v_plane = torch.randn(n_kv, cap, hd, generator=gen).to(torch.bfloat16)
    k_plane[:, start + n:] = float("nan")
    v_plane[:, start + n:] = float("nan")
    q = torch.randn(n, n_q * hd, generator=gen).to(torch.bfloat16)
    masks, anc = _random_tree(n, gen)
    k_plane, v_plane, q, anc = k_plane.to(dev), v_plane.to(dev), q.to(dev), anc.to(dev)
    state = kernels.new_state(dev, start=start)
    out = kernels.tree_attention(q, k_plane, v_plane, state, anc, n, n_q, splits=splits)
    ref = _reference(q, k_plane, v_plane, start, n, masks, n_q)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2, f"max abs err {err}"


@pytest.mark.parametrize("p_early,p_late", [(3000, 2048), (1024, 2900), (2047, 2048)])
def test_tree_attention_start_changed_upstream(lib, p_early, p_late):
    """The attention kernel reads `start` before its dependency wait to begin
    loading K/V early; when a kernel still running upstream changes `start`,
    the early load must land unused and the result must be the one for the
    new prefix.  Cache rows past the live keys hold NaN, so a zeroed V tail
    overwritten by a late load would show up as a non-finite output."""
    from dtree_mlx_b200 import _lib, kernels

    n_q, n_kv, hd, n = 32, 8, 128, 25
    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(p_early + p_late)
    cap = max(p_early, p_late) + n + 200
    k_plane = torch.randn(n_kv, cap, hd, generator=gen).to(torch.bfloat16)
    v_plane = torch.randn(n_kv, cap, hd, generator=gen).to(torch.bfloat16)
    k_plane[:, p_late + n:] = float("nan")
    v_plane[:, p_late + n:] = float("nan")
    q = torch.randn(n, n_q * hd, generator=gen).to(torch.bfloat16)
    masks, anc = _random_tree(n, gen)
    k_plane, v_plane, q, anc = k_plane.to(dev), v_plane.to(dev), q.to(dev), anc.to(dev)
    state = kernels.new_state(dev, start=p_early)
    out = torch.empty(n, n_q * hd, dtype=torch.bfloat16, device=dev)
    nbytes = int(lib.dtree_tree_attention_workspace_bytes(n_q, n, hd, 0))
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    st = _lib.stream_ptr()
    for _ in range(3):  # the store lands ~30 us after the attention kernel started
        state[0] = p_early
        _lib.call("dtree_test_delayed_store", state.data_ptr(), p_late, 30000, st)
        _lib.call("dtree_tree_attention", q.data_ptr(), q.stride(0), k_plane.data_ptr(), v_plane.data_ptr(), cap,
                  n_q, n_kv, hd, n, state.data_ptr(), anc.data_ptr(), out.data_ptr(), 0, ws.data_ptr(),
                  ws.numel(), st)
        torch.cuda.synchronize()
        assert int(state[0].item()) == p_late
        ref = _reference(q, k_plane, v_plane, p_late, n, masks, n_q)
        assert torch.isfinite(out.float()).all()
        err = (out.float() - ref).abs().max().item()
        assert err <= 2e-2, f"max abs err {err}"
    assert _lib.device_error() == 0


@pytest.mark.parametrize("heads", [(32, 8, 128), (8, 4, 64)])
@pytest.mark.parametrize("start,n", [(0, 1), (300, 25), (700, 9), (999, 25), (900, 64)])
def test_cluster_merge_bit_identical_to_split_shape(lib, heads, start, n):
    """With kv_cap <= 1024 and automatic splits the KV splits of a head run as
    one cluster that merges in shared memory; explicit splits of the same
    count run the split shape with attn_combine_kernel.  Both cut the keys
    into the same 128-key blocks and merge in split order, so the outputs
    agree bit for bit."""
    from dtree_mlx_b200 import kernels

    n_q, n_kv, hd = heads
    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(start * 7 + n + hd)
    cap = 1024
    k_plane = torch.randn(n_kv, cap, hd, generator=gen).to(torch.bfloat16)
    v_plane = torch.randn(n_kv, cap, hd, generator=gen).to(torch.bfloat16)
    k_plane[:, start + n:] = float("nan")
    v_plane[:, start + n:] = float("nan")
    q = torch.randn(n, n_q * hd, generator=gen).to(torch.bfloat16)
    masks, anc = _random_tree(n, gen)
    k_plane, v_plane, q, anc = k_plane.to(dev), v_plane.to(dev), q.to(dev), anc.to(dev)
    state = kernels.new_state(dev, start=start)
    out_cluster = kernels.tree_attention(q, k_plane, v_plane, state, anc, n, n_q, splits=0)
    out_split = kernels.tree_attention(q, k_plane, v_plane, state, anc, n, n_q, splits=cap // 128)
    torch.cuda.synchronize()
    assert torch.isfinite(out_cluster.float()).all()
    assert torch.equal(out_cluster, out_split)
