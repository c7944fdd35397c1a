"""Fitting the P3 acceptance table from a drafting log (host numpy, no GPU).

The drafting study fits, per feature code, the probability that draft position j is
accepted given that positions 1..j-1 were (tools/spec_replay.py:474-503): every draft point
contributes a trial at depth j when its first j-1 drafted ids were accepted and j is still
inside the turn, a hit when j was accepted too; sparse codes are smoothed toward the same
(match length, agreement) cell over all depths, that toward the match length alone, and
that toward the global rate, each with `alpha` pseudo-samples. The runtime side -- the
codes of a draft and the length they give -- is k3_suffix_drafter_features /
k3_spec_p3_length / k3_spec_p3_cost_length in the library; this file turns a log of
(codes, accepted prefix, ids left in the turn) into the table those calls take.
"""
from __future__ import annotations

import numpy as np

SPEC_MAX = 8
N_DEPTH, N_ELL, N_AGREE = 3, 13, 6
N_CODES = N_DEPTH * N_ELL * N_AGREE
NO_DRAFT = 255


def fit_p3_table(codes, accepted, remaining, weights=None, alpha: float = 20.0) -> np.ndarray:
    """q[N_CODES] from per-draft-point codes [P][8] (255 where nothing was drafted), the
    accepted prefix length of each point's full draft, and the ids left in its turn."""
    codes = np.asarray(codes)
    if codes.ndim != 2 or codes.shape[1] != SPEC_MAX:
        raise ValueError(f"codes must be [points][{SPEC_MAX}], got {codes.shape}")
    acc = np.asarray(accepted, np.int64)
    rem = np.asarray(remaining, np.int64)
    w = np.ones(len(acc)) if weights is None else np.asarray(weights, np.float64)
    drafted = codes[:, 0] != NO_DRAFT
    hits = np.zeros(N_CODES)
    trials = np.zeros(N_CODES)
    for j in range(1, SPEC_MAX + 1):
        at = drafted & (acc >= j - 1) & (rem >= j)        # position j was reached
        c = codes[at, j - 1].astype(np.int64)
        trials += np.bincount(c, w[at], minlength=N_CODES)
        ok = acc[at] >= j
        hits += np.bincount(c[ok], w[at][ok], minlength=N_CODES)
    h3 = hits.reshape(N_DEPTH, N_ELL, N_AGREE)
    t3 = trials.reshape(N_DEPTH, N_ELL, N_AGREE)
    rate = hits.sum() / max(trials.sum(), 1e-9)
    by_len = (h3.sum(axis=(0, 2)) + alpha * rate) / (t3.sum(axis=(0, 2)) + alpha)
    by_cell = (h3.sum(axis=0) + alpha * by_len[:, None]) / (t3.sum(axis=0) + alpha)
    return ((h3 + alpha * by_cell[None]) / (t3 + alpha)).reshape(-1)
