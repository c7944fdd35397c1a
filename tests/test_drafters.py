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


@pytest.mark.parametrize("seed,vocab,branch,depth,min_len",
                         [(11, 2, 2, 8, 1), (12, 3, 4, 6, 1), (13, 6, 4, 8, 2), (14, 20, 3, 5, 1)])
def test_suffix_tree_vs_oracle_restatement(k3, seed, vocab, branch, depth, min_len):
    """The draft tree at every history length against the brute-force string-counting
    restatement: same ids, same parents, same order (exact, including probability ties)."""
    rng = np.random.default_rng(seed)
    seq = rng.integers(0, vocab, 90).tolist()
    seq += seq[10:40]                                   # a planted repeat
    d = k3.SuffixDrafter(len(seq))
    for T in range(1, len(seq) + 1):
        d.push([seq[T - 1]])
        for nodes in (64, 9):
            got = d.tree(nodes, branch, depth, min_len)
            assert got == O.suffix_tree_draft(seq[:T], nodes, branch, depth, min_len), (T, nodes)
    d.close()


def test_suffix_tree_shape_and_verify_masks(k3):
    """A strictly periodic history gives one chain, P2's periodic draft; a noisy one gives
    a bushy tree whose parents precede children within the depth and branching limits and
    which fits the verify masks."""
    rng = np.random.default_rng(21)
    base = rng.integers(0, 50, 37).tolist()
    seq = base * 5 + base[:11]
    d = k3.SuffixDrafter(len(seq))
    d.push(seq)
    tok, par = d.tree(64, 3, 8, 1)
    assert tok == [seq[-1]] + d.draft(8, 1)[0] and par == list(range(-1, 8))
    assert d.tree(1, 3, 8, 1) == ([seq[-1]], [-1])
    assert d.tree(64, 3, 0, 1) == ([seq[-1]], [-1])     # depth 0: the root alone
    d.close()

    noisy = []
    for r in range(12):
        row = list(base)
        for j in rng.choice(len(row), 4, replace=False):
            row[j] = int(rng.integers(0, 6))
        noisy += row
    d = k3.SuffixDrafter(len(noisy))
    d.push(noisy)
    tok, par = d.tree(64, 3, 8, 1)
    assert tok[0] == noisy[-1] and par[0] == -1 and 9 < len(tok) <= 64
    depth = [0] * len(tok)
    for i in range(1, len(tok)):
        assert 0 <= par[i] < i
        depth[i] = depth[par[i]] + 1
        assert depth[i] <= 8
    assert max(np.bincount(par[1:])) <= 3
    assert (tok, par) == O.suffix_tree_draft(noisy, 64, 3, 8, 1)
    masks = O.tree_masks(par)                           # ancestor bitmasks for the verify
    assert masks.shape[0] == len(tok)
    d.close()
    fresh = k3.SuffixDrafter(8)
    fresh.push([5, 6, 7])                               # nothing repeats: the root alone
    assert fresh.tree() == ([7], [-1])
    fresh.close()
