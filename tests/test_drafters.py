"""Host drafters from the reference's drafting study (tools/spec_replay.py), CPU only.

P1 (k3_spec_draft_eager) and P2 (the incremental suffix-automaton drafter
k3_suffix_drafter_*) against golden drafts the reference tool itself produced at every
draft point of four seeded sequences with planted repeats and periodic runs
(tests/golden/ref_drafters.npz, made by tests/golden/make_drafter_golden.py), and against
the oracle's brute-force restatement on random sequences. Drafts are ids: bit-exact.
"""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))
from k3lib import load  # noqa: E402
from oracle import oracle as O  # noqa: E402

G = np.load(os.path.join(HERE, "golden", "ref_drafters.npz"))
N_SEQ = int(G["n_seq"])


@pytest.fixture(scope="module")
def k3():
    return load()


@pytest.mark.parametrize("si", range(N_SEQ))
def test_eager_draft_matches_reference_tool(k3, si):
    seq = G[f"s{si}/seq"].tolist()
    p1, p1n = G[f"s{si}/p1"], G[f"s{si}/p1n"]
    for T in range(1, len(seq) + 1):
        assert k3.spec_draft_eager(seq[:T], 8) == p1[T, :p1n[T]].tolist(), T


@pytest.mark.parametrize("si", range(N_SEQ))
def test_suffix_drafter_matches_reference_tool(k3, si):
    seq = G[f"s{si}/seq"].tolist()
    p2, L2, g2 = G[f"s{si}/p2"], G[f"s{si}/L2"], G[f"s{si}/g2"]
    d = k3.SuffixDrafter(len(seq))
    for T in range(1, len(seq) + 1):
        d.push([seq[T - 1]])
        ids, L, g = d.draft(8, min_len=1)
        assert (L, g) == (int(L2[T]), int(g2[T])), T
        assert ids == (p2[T].tolist() if L2[T] > 0 else []), T
    d.close()


def test_suffix_drafter_min_len_bulk_push_and_capacity(k3):
    rng = np.random.default_rng(3)
    seq = rng.integers(0, 4, 200).tolist()
    one, bulk = k3.SuffixDrafter(200), k3.SuffixDrafter(200)
    for i, v in enumerate(seq):
        one.push([v])
    bulk.push(seq[:77])
    bulk.push(seq[77:])
    assert len(one) == len(bulk) == 200
    assert one.draft(8, 1) == bulk.draft(8, 1)
    ids, L, g = one.draft(8, min_len=1)
    assert L > 0 and len(ids) == 8
    assert one.draft(8, min_len=L + 1) == ([], L, g)     # below min_len: no draft
    assert one.draft(3, min_len=1)[0] == ids[:3]
    with pytest.raises(k3.K3Error):
        one.push([1])                                   # past the capacity
    one.close()
    bulk.close()


@pytest.mark.parametrize("seed,vocab", [(1, 2), (2, 5), (3, 30)])
def test_drafters_vs_oracle_restatement(k3, seed, vocab):
    rng = np.random.default_rng(seed)
    seq = rng.integers(0, vocab, 160).tolist()
    d = k3.SuffixDrafter(len(seq))
    for T in range(1, len(seq) + 1):
        d.push([seq[T - 1]])
        assert k3.spec_draft_eager(seq[:T], 8) == O.eager_draft(seq, T, 8), T
        ids, L, g = d.draft(8, min_len=1)
        rids, rL, rg = O.longest_suffix_draft(seq, T, 8)
        assert (ids, L, g) == (rids, rL, rg), T
    d.close()


def test_suffix_drafter_long_history_is_linear(k3):
    """A 200k-id history with long repeats stays fast (suffix automaton, hash transitions)."""
    rng = np.random.default_rng(9)
    base = rng.integers(0, 1000, 5000).tolist()
    seq = (base * 40)[:200000]
    d = k3.SuffixDrafter(len(seq))
    d.push(seq)
    ids, L, g = d.draft(8, min_len=1)
    assert L > 1000 and g == 5000 and ids == seq[len(seq) - 5000:len(seq) - 5000 + 8]
    d.close()
