"""Oracle: the seeded planted-draft generator used by the synthetic workloads.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The reference drafts with a trained DFlash drafter (dtree_mlx/draft.py:351-367,
logits through the target LM head, dtree_runtime.py:366-376).  Random-init
weights make a real drafter useless, so the benchmark workloads plant the
draft logits instead: for draft row ``r`` (block position ``r+1``, i.e. output
position ``start + r + 1``) the logits are N(0,1)-like noise with +8 on the
target's greedy-continuation token with probability ``p``, otherwise +8 on a
uniformly random token.

Bit-exact CPU/GPU reproducibility: noise comes from Philox4x32-10 (integer
only) and the Irwin-Hall sum of 12 uniforms, each uniform ``(x >> 8) * 2^-24``
(exact in fp32), summed in a fixed order with fp32 round-to-nearest adds, then
``- 6``.  The CUDA kernel ``plant_draft_logits_kernel`` performs the same
operations, so both produce identical fp32 logits.
"""
from __future__ import annotations

import numpy as np

M0 = np.uint64(0xD2511F53)
M1 = np.uint64(0xCD9E8D57)
W0 = np.uint32(0x9E3779B9)
W1 = np.uint32(0xBB67AE85)
MASK32 = np.uint64(0xFFFFFFFF)

NOISE_TAG = 0xD1CE
PLANT_TAG = 0xB1A5
KEY_HI = 0x5EED0001
SPIKE = np.float32(8.0)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Vectorised Philox4x32 with 10 rounds (Salmon et al., SC'11)."""
    c0 = np.asarray(c0, dtype=np.uint32)
    c1 = np.asarray(c1, dtype=np.uint32)
    c2 = np.asarray(c2, dtype=np.uint32)
    c3 = np.asarray(c3, dtype=np.uint32)
    k0 = np.asarray(k0, dtype=np.uint32)
    k1 = np.asarray(k1, dtype=np.uint32)
    c0, c1, c2, c3 = np.broadcast_arrays(c0, c1, c2, c3)
    c0, c1, c2, c3 = c0.copy(), c1.copy(), c2.copy(), c3.copy()
    with np.errstate(over="ignore"):
        for r in range(10):
            if r > 0:
                k0 = (k0 + W0).astype(np.uint32)
                k1 = (k1 + W1).astype(np.uint32)
            p0 = c0.astype(np.uint64) * M0
            p1 = c2.astype(np.uint64) * M1
            hi0 = (p0 >> np.uint64(32)).astype(np.uint32)
            lo0 = (p0 & MASK32).astype(np.uint32)
            hi1 = (p1 >> np.uint64(32)).astype(np.uint32)
            lo1 = (p1 & MASK32).astype(np.uint32)
            c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
    return c0, c1, c2, c3


def _uniform(x: np.ndarray) -> np.ndarray:
    return ((x >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)).astype(np.float32)


def noise_row(seed: int, step: int, row: int, vocab: int) -> np.ndarray:
    """Irwin-Hall(12) - 6 noise for one draft row (fp32)."""
    v = np.arange(vocab, dtype=np.uint32)
    acc = np.zeros(vocab, dtype=np.float32)
    for j in range(3):
        x = philox4x32_10(v, np.uint32(row | (j << 16)), np.uint32(step), np.uint32(NOISE_TAG),
                          np.uint32(seed), np.uint32(KEY_HI))
        for lane in range(4):
            acc = (acc + _uniform(x[lane])).astype(np.float32)
    return (acc - np.float32(6.0)).astype(np.float32)


def plant_choice(seed: int, step: int, row: int, vocab: int, p_correct: float):
    """(take_correct, random_token) for one row."""
    x = philox4x32_10(np.uint32(0xFFFFFFFF), np.uint32(row), np.uint32(step), np.uint32(PLANT_TAG),
                      np.uint32(seed), np.uint32(KEY_HI))
    u = float(_uniform(np.asarray(x[0])))
    thresh = np.float32(p_correct)
    take = np.float32(u) < thresh
    rand_tok = int(np.asarray(x[1])) % vocab
    return bool(take), rand_tok


def planted_draft_logits(seed: int, step: int, start: int, rows: int, vocab: int,
                         continuation: np.ndarray, p_correct: float) -> np.ndarray:
    """Draft logits [rows, vocab] for the decode step that begins at ``start``
    (the number of committed tokens).  ``continuation[i]`` is the target's
    greedy token at absolute output position ``i`` (length may be short,
    entries may be -1: such positions plant on a random token)."""
    out = np.empty((rows, vocab), dtype=np.float32)
    for r in range(rows):
        out[r] = noise_row(seed, step, r, vocab)
        take, rand_tok = plant_choice(seed, step, r, vocab, p_correct)
        pos = start + r + 1
        known = take and pos < len(continuation) and int(continuation[pos]) >= 0
        tok = int(continuation[pos]) if known else rand_tok
        out[r, tok] = np.float32(out[r, tok] + SPIKE)
    return out
