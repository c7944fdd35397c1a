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

import json
import re

import numpy as np

SPEC_MAX = 8
N_DEPTH, N_ELL, N_AGREE = 3, 13, 6
N_CODES = N_DEPTH * N_ELL * N_AGREE
NO_DRAFT = 255
LENGTH_EDGES = (1, 2, 3, 4, 5, 6, 7, 9, 12, 16, 24, 32, 64)   # lower edges of the 13 length buckets


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


def load_study(path) -> dict:
    """The acceptance table, verify-cost tiers and calibrated P2 settings a drafting study
    recorded (the JSON that tools/spec_replay.py writes, docs/measurements/spec-replay.json:
    its p3_table, cost_model and p2_defaults_from_calibration sections), checked against the
    codes this library computes: a table whose buckets or code formula differ is refused,
    since its entries would be read under the wrong codes.

    Returns {"q": float64[N_CODES], "costs": {tier: {a_T, a_E, a_C, eps, expert_ratio}},
    "p2_defaults": {tier: {"min_len", "N"}}}; the costs map onto K3SpecCost fields."""
    with open(path) as f:
        d = json.load(f)
    t = d["p3_table"]
    if tuple(t["length_bucket_lower_edges"]) != LENGTH_EDGES or len(t["depth_buckets"]) != N_DEPTH \
            or len(t["agreement_buckets"]) != N_AGREE:
        raise ValueError("the table's buckets are not the ones k3_suffix_drafter_features codes with")
    if t["code_index"].replace(" ", "") != f"(depth_bucket*{N_ELL}+length_bucket)*{N_AGREE}+agreement_bucket":
        raise ValueError(f"unknown code formula {t['code_index']!r}")
    q = np.asarray(t["q"], np.float64)
    if q.shape != (N_CODES,) or not np.all(np.isfinite(q)) or q.min() < 0 or q.max() > 1:
        raise ValueError(f"a table of {N_CODES} probabilities is needed, got shape {q.shape}")
    out = {"q": q, "costs": {}, "p2_defaults": {}}
    cm = d.get("cost_model")
    if cm:
        m = re.fullmatch(r"u\(n\) = (\d+)\*\(1 - \((\d+)/(\d+)\)\^n\)", cm["u"].strip())
        if not m or int(m.group(2)) != int(m.group(1)) - 1 or int(m.group(3)) != int(m.group(1)):
            raise ValueError(f"unknown distinct-expert term {cm['u']!r}")
        for tier, c in cm["tiers"].items():
            out["costs"][tier] = {"a_T": float(c["a_T"]), "a_E": float(c["a_E"]), "a_C": float(c["a_C"]),
                                  "eps": float(cm.get("eps", 0.0)), "expert_ratio": float(m.group(1))}
    for tier, name in d.get("p2_defaults_from_calibration", {}).items():
        m = re.fullmatch(r"P2/min(\d+)/N(\d+)", name)
        if not m:
            raise ValueError(f"unknown P2 setting {name!r}")
        out["p2_defaults"][tier] = {"min_len": int(m.group(1)), "N": int(m.group(2))}
    return out
