"""tcgen05 stream-K GEMM and the fused LM-head argmax vs a torch fp32 reference.

Tolerance for bf16 outputs: |y - ref| <= 2^-7 |ref| + 1e-3 max|ref| (one bf16
rounding of an fp32 accumulation of the same bf16 inputs).
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def K(lib):
    from dtree_mlx_b200 import kernels

    return kernels


def _check(y, ref):
    err = (y.float() - ref).abs()
    tol = ref.abs() * 2.0 ** -7 + 1e-3 * ref.abs().max()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{bad} elements out of tolerance, max err {err.max().item()}"


@pytest.mark.parametrize(
    "t_pad,k,n",
    [
        (16, 64, 128),
        (32, 256, 384),
        (32, 2560, 6144),   # fused q|k|v of the 4B shape
        (32, 4096, 2560),   # o_proj: 20 tiles -> stream-K partial tiles
        (32, 9728, 2560),   # down_proj
        (16, 512, 200),     # ragged N (zero-filled TMA rows)
        (64, 1024, 1536),
        (80, 2560, 6144),   # 65 tree rows (budget 64) pad to 80 (a legal UMMA N)
        (80, 9728, 2560),
        (128, 512, 640),
    ],
)
def test_linear_matches_fp32(K, t_pad, k, n):
    g = torch.Generator(device=DEV).manual_seed(t_pad * 7 + k + n)
    x = torch.randn(t_pad, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    y = K.linear_bf16(x, w)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    _check(y, ref)


@pytest.mark.parametrize(
    "t_pad,k,n,split_k",
    [
        (16, 64, 128, 0),
        (32, 2560, 6144, 0),    # q|k|v of the 4B shape, stream-K
        (32, 4096, 2560, 0),    # o_proj
        (32, 9728, 2560, 7),    # down_proj, tile-aligned split-K grid
        (16, 512, 200, 0),      # ragged N
        (64, 1024, 1536, 0),
        (80, 2560, 6144, 0),    # 65 tree rows pad to 80
        (128, 512, 640, 0),
        (32, 320, 1280, 0),     # K/64 = 5: scalar scale loads, one unit per CTA
        (16, 192, 384, 2),      # one or two units per CTA (a lone unit pair)
    ],
)
def test_linear_q4_matches_dequantized_fp32(K, t_pad, k, n, split_k):
    """The fused dequant GEMM equals x @ bf16(scale*q + bias)^T accumulated in
    fp32: the oracle dequantizes the MLX-packed weights independently."""
    from dtree_mlx_b200.synthetic import quantize_affine_q4
    from oracle.qwen3 import dequant_affine_q4

    g = torch.Generator(device=DEV).manual_seed(t_pad * 5 + k + n)
    x = torch.randn(t_pad, k, device=DEV, generator=g).to(torch.bfloat16)
    w = quantize_affine_q4((torch.randn(n, k, device=DEV, generator=g) * 0.02).to(torch.bfloat16))
    y = K.linear_q4(x, w, split_k=split_k)
    torch.cuda.synchronize()
    wd = dequant_affine_q4(w.packed.cpu(), w.scales.cpu(), w.biases.cpu()).to(torch.bfloat16).float()
    ref = x.float().cpu() @ wd.t()
    _check(y.cpu(), ref)


def test_linear_q4_deterministic(K):
    from dtree_mlx_b200.synthetic import quantize_affine_q4

    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(32, 2560, device=DEV, generator=g).to(torch.bfloat16)
    w = quantize_affine_q4((torch.randn(9728, 2560, device=DEV, generator=g) * 0.02).to(torch.bfloat16))
    y1 = K.linear_q4(x, w).clone()
    y2 = K.linear_q4(x, w).clone()
    assert torch.equal(y1, y2)


def test_linear_deterministic(K):
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(32, 9728, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(2560, 9728, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    y1 = K.linear_bf16(x, w).clone()
    y2 = K.linear_bf16(x, w).clone()
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("t_pad,n_rows,hidden,vocab", [(32, 25, 2560, 151936), (16, 9, 512, 32768), (64, 40, 512, 5000),
                                                      (80, 65, 2560, 151936)])
def test_lm_head_argmax(K, t_pad, n_rows, hidden, vocab):
    g = torch.Generator(device=DEV).manual_seed(vocab)
    h = torch.randn(t_pad, hidden, device=DEV, generator=g).to(torch.bfloat16)
    e = (torch.randn(vocab, hidden, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    out = K.lm_head_argmax(h, e, n_rows)
    torch.cuda.synchronize()
    logits = (h[:n_rows].double() @ e.double().t()).to(torch.bfloat16).float()
    ref = torch.argmax(logits, dim=-1)
    got = out.long()
    mism = (got != ref).nonzero().flatten().tolist()
    for t in mism:  # only near-ties may differ (one bf16 ulp at the max)
        mx = logits[t].max()
        assert (mx - logits[t, got[t]]).abs() <= mx.abs() * 2.0 ** -7, (t, got[t].item(), ref[t].item())
    assert len(mism) <= max(1, n_rows // 10)


def test_lm_head_argmax_first_index_on_ties(K):
    """Exact ties (also across vocab tiles / CTAs) keep the smallest id."""
    hidden, vocab = 256, 40000
    e = torch.zeros(vocab, hidden, device=DEV, dtype=torch.bfloat16)
    h = torch.ones(16, hidden, device=DEV, dtype=torch.bfloat16)
    for v in (70, 5, 39000, 20000):
        e[v] = 1.0
    out = K.lm_head_argmax(h, e, 16)
    assert out.tolist() == [5] * 16
    # repeated calls: the device keys/counters reset themselves
    out2 = K.lm_head_argmax(h, e, 16)
    assert out2.tolist() == [5] * 16


def test_shared_workspace_across_grids(K):
    """GEMMs with different stream-K grids and tile widths share one workspace:
    the tile counters must not be overwritten by another plan's partials."""
    g = torch.Generator(device=DEV).manual_seed(11)
    shapes = [(32, 512, 512), (32, 2560, 6144), (32, 1536, 512), (32, 512, 3072), (32, 512, 512)]
    for t_pad, k, n in shapes * 2:
        x = torch.randn(t_pad, k, device=DEV, generator=g).to(torch.bfloat16)
        w = (torch.randn(n, k, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
        y = K.linear_bf16(x, w)
        _check(y, x.float() @ w.float().t())
