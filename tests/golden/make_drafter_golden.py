"""Generate tests/golden/ref_drafters.npz from the reference's drafting study
(tools/spec_replay.py), run here where the reference tree exists.

For seeded id sequences with planted repeats (copies of earlier spans, periodic runs), at
every draft point T (the history seq[0..T), after the tool's SuffixAutomaton.extend of id
T-1 and before its commit, exactly as analyze_sequence steps, tools/spec_replay.py:408-469):
  p0[T]      spec_draft(seq, T, 8)  (P0, the engine's drafter, :122-171, the tool's port of
             src/cli/k3_run.c:450-491), -1 padded, with its length p0n[T]
  p1[T]      eager_draft(seq, T, 8)  (P1, :174-184), -1 padded, with its length
  L2[T]      the suffix automaton's match length (0: none)
  g2[T]      its period pos - last_end (0: none)
  p2[T]      periodic_copy(seq, last_end + 1, g, 8)  (P2, :333-336, 442-449), -1 padded
  f3[T]      draft_features of that P2 draft (P3's feature codes, :371-397), 255 without one
and the P3 lengths of every draft point under four acceptance tables -- the tool's own
fit_acceptance_table (:474-503) on these sequences' P2 acceptances, two seeded random
tables, and the table the study recorded (docs/measurements/spec-replay.json, p3_table) --
by adaptive_lengths (:525-536; delta 0.1, 0.22, 0.55; cumulative and per position) and
cost_aware_lengths (:539-568; both tiers, with and without replay):
  q          [4][234] the tables
  s<i>/p3a   [4][3][2][n+1] adaptive lengths (table, delta, cumulative 1/0)
  s<i>/p3c   [4][2][2][n+1] cost-aware lengths (table, tier 8GB/128GB, replay 0/1)
It also writes tests/golden/study_table.json: the study file's p3_table, cost_model and
p2_defaults_from_calibration sections, as a user would hand them to
spec_table.load_study.

Usage: python tests/golden/make_drafter_golden.py [--ref <path of the reference checkout>]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_dir():
    """K3_REFERENCE, else a checkout named `reference` beside this repository."""
    return os.environ.get("K3_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
CAP = 8


def sequences(rng):
    out = []
    for n, vocab in ((400, 12), (600, 50), (500, 2000), (300, 3)):
        s = list(rng.integers(0, vocab, 40))
        while len(s) < n:
            r = rng.random()
            if r < 0.45 and len(s) > 8:                     # copy an earlier span
                a = int(rng.integers(0, len(s) - 4))
                ln = int(rng.integers(3, 24))
                s.extend(s[a:a + ln])
            elif r < 0.6:                                   # a periodic run
                per = int(rng.integers(1, 5))
                base = list(rng.integers(0, vocab, per))
                s.extend((base * 10)[:int(rng.integers(4, 20))])
            else:
                s.extend(rng.integers(0, vocab, int(rng.integers(1, 10))))
        out.append(np.asarray(s[:n], np.int32))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=reference_dir(),
                    help="the reference checkout (default: K3_REFERENCE, else `reference` beside this repository)")
    a = ap.parse_args()
    spec = importlib.util.spec_from_file_location("spec_replay", os.path.join(a.ref, "tools", "spec_replay.py"))
    sr = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sr)
    rng = np.random.default_rng(20260)
    arrays = {}
    feats = []
    for si, seq in enumerate(sequences(rng)):
        s = [int(v) for v in seq]
        n = len(s)
        p0 = np.full((n + 1, CAP), -1, np.int32)
        p0n = np.zeros(n + 1, np.int32)
        p1 = np.full((n + 1, CAP), -1, np.int32)
        p1n = np.zeros(n + 1, np.int32)
        p2 = np.full((n + 1, CAP), -1, np.int32)
        L2 = np.zeros(n + 1, np.int32)
        g2 = np.zeros(n + 1, np.int32)
        f3 = np.full((n + 1, CAP), sr.NO_DRAFT, np.uint8)
        a2 = np.zeros(n + 1, np.int64)
        sam = sr.SuffixAutomaton()
        for pos in range(n):
            v = sam.extend(s[pos], pos)
            T = pos + 1
            d = sr.spec_draft(s, T, CAP)
            p0[T, :len(d)] = d
            p0n[T] = len(d)
            d = sr.eager_draft(s, T, CAP)
            p1[T, :len(d)] = d
            p1n[T] = len(d)
            if v > 0:
                e = sam.last_end[v]
                g = pos - e
                L2[T] = sam.length[v]
                g2[T] = g
                p2[T] = sr.periodic_copy(s, e + 1, g, CAP)
                f3[T] = sr.draft_features(sam, v, sam.length[v], p2[T].tolist())
                a2[T] = sr._lcp(p2[T].tolist(), s, T, n - T)
                # the tool's own brute-force check of the automaton
                bl, be, _ = sr.longest_suffix_match(s, T)
                assert (bl, be) == (sam.length[v], e), (si, T)
            sam.commit(pos)
        arrays[f"s{si}/seq"] = seq
        arrays[f"s{si}/p0"] = p0
        arrays[f"s{si}/p0n"] = p0n
        arrays[f"s{si}/p1"] = p1
        arrays[f"s{si}/p1n"] = p1n
        arrays[f"s{si}/p2"] = p2
        arrays[f"s{si}/L2"] = L2
        arrays[f"s{si}/g2"] = g2
        arrays[f"s{si}/f3"] = f3
        feats.append((f3[1:n], a2[1:n], np.arange(n - 1, 0, -1)))
    # P3 tables: the tool's fit on these draft points, then two seeded random tables
    F = np.concatenate([f[0] for f in feats])
    A = np.concatenate([f[1] for f in feats])
    R = np.concatenate([f[2] for f in feats])
    q_fit, _ = sr.fit_acceptance_table(F, A, R)
    with open(os.path.join(a.ref, "docs", "measurements", "spec-replay.json")) as f:
        study = json.load(f)
    q_rec = np.asarray(study["p3_table"]["q"], float)
    qs = np.stack([q_fit, rng.uniform(0.05, 1.0, sr.N_CODES), rng.uniform(0.3, 1.0, sr.N_CODES), q_rec])
    sub = {k: study[k] for k in ("p3_table", "cost_model", "p2_defaults_from_calibration")}
    with open(os.path.join(HERE, "study_table.json"), "w") as f:
        json.dump(sub, f, indent=1)
    arrays["q"] = qs
    deltas = (0.1, 0.22, 0.55)
    for si in range(len(feats)):
        f3 = arrays[f"s{si}/f3"]
        p3a = np.zeros((len(qs), len(deltas), 2, len(f3)), np.int32)
        p3c = np.zeros((len(qs), 2, 2, len(f3)), np.int32)
        for qi, q in enumerate(qs):
            for di, dl in enumerate(deltas):
                p3a[qi, di, 1] = sr.adaptive_lengths(f3, q, dl, cumulative=True)
                p3a[qi, di, 0] = sr.adaptive_lengths(f3, q, dl, cumulative=False)
            for ti, tier in enumerate(("8GB", "128GB")):
                for rp in (0, 1):
                    p3c[qi, ti, rp] = sr.cost_aware_lengths(f3, q, tier, bool(rp))
        arrays[f"s{si}/p3a"] = p3a
        arrays[f"s{si}/p3c"] = p3c
    arrays["n_seq"] = np.int32(len(sequences(np.random.default_rng(20260))))
    path = os.path.join(HERE, "ref_drafters.npz")
    np.savez_compressed(path, **arrays)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
