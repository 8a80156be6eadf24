"""Seeded synthetic requests with the shapes of the benchmark configurations.

No public dataset is involved; the real tokenizer and checkpoint are absent, so
token ids are drawn uniformly from the non-special vocabulary [0, 50280) and
laid out the way the reference's sequence builder lays them out
(systemone.rs:156-198): [CLS] at 0, a [SEP] closing the question head, one
[MASK] per option marker, the state, and a closing [SEP]; padding id 0.
"""
from __future__ import annotations

import numpy as np

from . import arch
from .engine import Req

NON_SPECIAL = 50280


def _row(rng, r, n_markers):
    """One sequence of length r with n_markers [MASK] markers after a mid [SEP]."""
    ids = rng.integers(0, NON_SPECIAL, r)
    ids[0] = arch.CLS_ID
    ids[r - 1] = arch.SEP_ID
    head = max(2, min(r // 3, r - n_markers - 3))
    ids[head] = arch.SEP_ID
    pos = np.sort(rng.choice(np.arange(head + 1, r - 1), size=n_markers, replace=False))
    ids[pos] = arch.MASK_ID
    return ids, pos


def padded_batch(rng, lens, l, markers_lo=2, markers_hi=6, qtypes=None) -> Req:
    n = len(lens)
    nms = [int(rng.integers(markers_lo, markers_hi + 1)) for _ in lens]
    k = max(nms)
    ids = np.zeros((n, l), np.int64)
    att = np.zeros((n, l), np.int64)
    mpos = np.zeros((n, k), np.int64)
    mmask = np.zeros((n, k), np.int64)
    for b, (r, nm) in enumerate(zip(lens, nms)):
        row, pos = _row(rng, r, nm)
        ids[b, :r] = row
        att[b, :r] = 1
        mpos[b, :nm] = pos
        mmask[b, :nm] = 1
    qtype = np.asarray(qtypes if qtypes is not None else rng.integers(0, 3, n), np.int64)
    return Req(n, l, k, ids, att, mpos, mmask, qtype)


def forward_16k(seed: int = 0) -> Req:
    """Config 2: the default --max-tokens 16384 budget as 128 sequences x 128
    padded tokens, real lengths uniform in [24, 128]."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(24, 129, 128)
    return padded_batch(rng, lens, 128)


def long_state(seed: int = 3) -> Req:
    """Config 3: 8 sequences at the maximum position length (512): ~32 tokens
    of question head with 3 criteria markers, state filling the rest."""
    rng = np.random.default_rng(seed)
    return padded_batch(rng, [512] * 8, 512, markers_lo=3, markers_hi=3, qtypes=[0] * 8)


def real_tokens(req: Req) -> int:
    return int((req.att != 0).sum())


def padded_tokens(req: Req) -> int:
    return req.n * req.l


def gemm_flops(req: Req) -> float:
    """Algorithmic GEMM FLOPs of one forward on real tokens (scorer included)."""
    R = real_tokens(req)
    p_enc = 28 * (1024 * 3072 + 1024 * 1024 + 1024 * 5248 + 2624 * 1024)
    p_head = 2 * (3072 * 1024 + 1024 * 1024 + 2 * 1024 * 4096)
    return 2.0 * R * (p_enc + p_head) + 2.0 * req.n * req.k * 1024 * 1024


def attention_flops(req: Req) -> float:
    """4*H per visible (query, key) pair: 10 global + 18 windowed encoder
    layers and 2 global head layers, real tokens only."""
    lens = (req.att.reshape(req.n, req.l) != 0).sum(1)
    g = float((lens.astype(np.float64) ** 2).sum())
    band = 0.0
    for r in lens:
        i = np.arange(r)
        band += float((np.minimum(i + 64, r - 1) - np.maximum(i - 64, 0) + 1).sum())
    return 4.0 * 1024 * (10 * g + 18 * band + 2 * g)
