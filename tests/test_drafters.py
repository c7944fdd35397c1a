"""Host drafters from the reference's drafting study (tools/spec_replay.py), CPU only.

P0 (the engine's n-gram drafter, k3_spec_draft_ngram), P1 (k3_spec_draft_eager) and P2
(the incremental suffix-automaton drafter k3_suffix_drafter_*) against golden drafts the
reference tool itself produced at every
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
def test_engine_ngram_draft_matches_reference_tool(k3, si):
    """The engine's drafter (k3_spec_draft_ngram with the engine's n = 4 then 3) against
    the tool's line-for-line port of src/cli/k3_run.c's spec_draft at every draft point;
    a smaller cap gives the same draft's prefix."""
    seq = G[f"s{si}/seq"].tolist()
    p0, p0n = G[f"s{si}/p0"], G[f"s{si}/p0n"]
    for T in range(1, len(seq) + 1):
        want = p0[T, :p0n[T]].tolist()
        assert k3.spec_draft(seq[:T], 8, 4, 3) == want, T
        assert k3.spec_draft(seq[:T], 3, 4, 3) == want[:3], T


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
    tok = (k3.C.c_int * 1)()
    assert k3.lib.k3_suffix_drafter_tree(fresh._d, 1 << 20, 4, 8, 1, tok, tok) == 0   # above 65536 nodes
    fresh.close()


# the study's two verify-cost tiers (tools/spec_replay.py:73-77): trunk streamed from an
# 8 GB machine, trunk resident at 128 GB; 896 routed experts at top-16 give ratio 56
TIERS = (("8GB", (0.78, 0.19, 0.03)), ("128GB", (0.44, 0.45, 0.11)))
DELTAS = (0.1, 0.22, 0.55)


def _cost(k3, coef):
    return k3.K3SpecCost(coef[0], coef[1], coef[2], 0.0, 56.0)


@pytest.mark.parametrize("si", range(N_SEQ))
def test_p3_features_and_lengths_match_reference_tool(k3, si):
    """P3's feature codes at every draft point, and the adaptive and cost-aware lengths
    under three tables (the tool's own fit and two random ones), against the tool."""
    seq = G[f"s{si}/seq"].tolist()
    f3, p3a, p3c, qs = G[f"s{si}/f3"], G[f"s{si}/p3a"], G[f"s{si}/p3c"], G["q"]
    d = k3.SuffixDrafter(len(seq))
    for T in range(1, len(seq) + 1):
        d.push([seq[T - 1]])
        ids, L, _ = d.draft(8, min_len=1)
        codes = d.features(ids if L > 0 else G[f"s{si}/p2"][T].tolist())
        assert codes == f3[T].tolist(), T
        for qi, q in enumerate(qs):
            for di, dl in enumerate(DELTAS):
                assert k3.spec_p3_length(codes, q, dl, True) == p3a[qi, di, 1, T], (T, qi, dl)
                assert k3.spec_p3_length(codes, q, dl, False) == p3a[qi, di, 0, T], (T, qi, dl)
            for ti, (_, coef) in enumerate(TIERS):
                for rp in (0, 1):
                    assert k3.spec_p3_cost_length(codes, q, _cost(k3, coef), rp) == p3c[qi, ti, rp, T], \
                        (T, qi, ti, rp)
        # the one-call P3 draft is P2's draft cut to the delta-rule length
        q = qs[0]
        want = p3a[0, 1, 1, T]
        assert d.draft_p3(q, 0.22) == (ids[:want] if L > 0 else [])
        assert d.draft_p3(q, 0.22, cap=2) == (ids[:min(want, 2)] if L > 0 else [])
        assert d.draft_p3(q, cost=_cost(k3, TIERS[1][1])) == (ids[:p3c[0, 1, 0, T]] if L > 0 else [])
    d.close()


def test_p3_edges(k3):
    q = np.full(k3.SPEC_P3_CODES, 0.9)
    assert k3.spec_p3_length([255] * 8, q, 0.1) == 0          # no match: no draft
    assert k3.spec_p3_length([0] * 8, q, 0.5) == 6             # 0.9^6 = 0.53 > 0.5 > 0.9^7
    assert k3.spec_p3_length([0] * 8, q, 0.5, cumulative=False) == 8
    assert k3.spec_p3_length([0] * 3, q, 0.1) == 3             # fewer positions than 8
    c = k3.K3SpecCost(0.44, 0.45, 0.11, 0.0, 56.0)
    assert k3.spec_p3_cost_length([0] * 8, np.ones(k3.SPEC_P3_CODES), c) == 8
    assert k3.spec_p3_cost_length([0] * 8, np.zeros(k3.SPEC_P3_CODES), c) == 0
    with pytest.raises(ValueError):
        k3.spec_p3_length([0], q[:10], 0.5)                    # a table of the wrong size
    d = k3.SuffixDrafter(4)
    d.push([1, 2, 3])
    assert d.features([7, 7]) == [255, 255] and d.draft_p3(q) == []
    d.close()


def test_p3_table_fit_matches_reference_tool(k3):
    """The host fit of the acceptance table reproduces the table the tool fitted on the
    golden sequences' P2 draft points (codes, accepted prefix, ids left)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "spec_table", os.path.join(os.path.dirname(HERE), "kimi-k3-for-me_b200", "spec_table.py"))
    st = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(st)
    F, A, R = [], [], []
    for si in range(N_SEQ):
        seq = G[f"s{si}/seq"].tolist()
        n = len(seq)
        for T in range(1, n):
            d = G[f"s{si}/p2"][T].tolist()
            m = 0
            while m < min(8, n - T) and seq[T + m] == d[m]:
                m += 1
            F.append(G[f"s{si}/f3"][T])
            A.append(m if G[f"s{si}/L2"][T] > 0 else 0)
            R.append(n - T)
    q = st.fit_p3_table(np.array(F), A, R)
    assert q.shape == (k3.SPEC_P3_CODES,)
    assert np.array_equal(q, G["q"][0])                  # same operations, same order: exact


def _spec_table():
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "spec_table", os.path.join(os.path.dirname(HERE), "kimi-k3-for-me_b200", "spec_table.py"))
    st = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(st)
    return st


def test_study_table_loads_and_drives_p3_as_the_tool(k3, tmp_path):
    """The table, cost tiers and P2 settings the study recorded (tests/golden/study_table.json,
    the study file's own sections) load as the library's inputs, and P3 with them gives the
    tool's lengths at every draft point (table 3 of the golden vectors is that table)."""
    import json
    st = _spec_table()
    path = os.path.join(HERE, "golden", "study_table.json")
    d = st.load_study(path)
    assert np.array_equal(d["q"], G["q"][3])
    assert d["p2_defaults"] == {"8GB": {"min_len": 5, "N": 8}, "128GB": {"min_len": 6, "N": 4}}
    for ti, (tier, coef) in enumerate(TIERS):
        c = d["costs"][tier]
        assert (c["a_T"], c["a_E"], c["a_C"], c["eps"], c["expert_ratio"]) == coef + (0.0, 56.0)
    costs = [k3.K3SpecCost(**d["costs"][tier]) for tier, _ in TIERS]
    for si in range(N_SEQ):
        seq = G[f"s{si}/seq"].tolist()
        f3, p3a, p3c = G[f"s{si}/f3"], G[f"s{si}/p3a"], G[f"s{si}/p3c"]
        for T in range(1, len(seq) + 1):
            codes = f3[T].tolist()
            assert k3.spec_p3_length(codes, d["q"], 0.22, True) == p3a[3, 1, 1, T]
            for ti in range(2):
                assert k3.spec_p3_cost_length(codes, d["q"], costs[ti], 1) == p3c[3, ti, 1, T]
    # refusals: other buckets, another formula, a short table
    raw = json.load(open(path))
    for key, val in (("length_bucket_lower_edges", [1, 2, 3, 4, 5, 6, 8, 9, 12, 16, 24, 32, 64]),
                     ("code_index", "(length_bucket*3 + depth_bucket)*6 + agreement_bucket"),
                     ("q", raw["p3_table"]["q"][:200])):
        bad = json.loads(json.dumps(raw))
        bad["p3_table"][key] = val
        q = tmp_path / f"bad_{key}.json"
        q.write_text(json.dumps(bad))
        with pytest.raises(ValueError):
            st.load_study(str(q))
