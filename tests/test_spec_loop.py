"""The speculative decode loop (k3_spec_loop_*), host only, over a greedy model on the CPU.

Two checks: the ids it generates equal plain serial greedy decoding of the same model for
every drafting policy (the property the engine's loop exists to keep,
src/cli/k3_run.c:2909-2943), and its per-step (nd, m, keep) trace, counters and final
state equal the oracle's restatement of the engine loop (oracle.spec_loop). The model is a
deterministic function of the context: mostly an order-2 table over a small vocabulary
(so drafts are often right), with context-dependent deviations (so they are often wrong).
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


@pytest.fixture(scope="module")
def k3():
    return load()


def make_model(seed, vocab=9, noise=5):
    rng = np.random.default_rng(seed)
    table = rng.integers(0, vocab, (vocab, vocab))

    def next_id(ctx):
        if len(ctx) % noise == 0 and sum(ctx[-3:]) % 3 == 0:
            return (sum(ctx[-4:]) * 7 + len(ctx)) % vocab
        return int(table[ctx[-2] if len(ctx) > 1 else 0][ctx[-1]])
    return next_id


class Fake:
    """A model that holds its consumed positions and checks the verify/commit protocol."""

    def __init__(self, next_id, consumed):
        self.next_id, self.state, self.pending = next_id, list(consumed), None
        self.calls = []

    def verify(self, ids, base, parent=None):
        assert base == len(self.state) and self.pending is None
        self.pending = (list(ids), parent)
        self.calls.append(len(ids))
        if parent is None:
            return [self.next_id(self.state + ids[:i + 1]) for i in range(len(ids))]
        assert parent[0] == -1 and all(0 <= parent[i] < i for i in range(1, len(ids)))

        def path(i):
            p = []
            while i >= 0:
                p.append(ids[i])
                i = parent[i]
            return p[::-1]
        return [self.next_id(self.state + path(i)) for i in range(len(ids))]

    def commit(self, base, keep, path=None):
        assert base == len(self.state) and self.pending is not None
        ids, parent = self.pending
        assert 0 <= keep <= len(ids)
        if path is None:
            self.state += ids[:keep]
        else:                                   # a root-first chain of the tree's nodes
            assert parent is not None and path[0] == 0
            assert all(parent[path[i]] == path[i - 1] for i in range(1, keep))
            self.state += [ids[i] for i in path]
        self.pending = None


def serial(next_id, ids, gen, tmax, stops):
    seq, out = list(ids), []
    while len(out) < gen and len(seq) < tmax:
        v = next_id(seq)
        seq.append(v)
        out.append(v)
        if v in stops:
            break
    return out


CASES = [  # policy, spec_n, min_len, gen, stop ids ("late": the ids serial decode first emits late), seed
    (0, 8, 1, 40, (), 1), (1, 8, 1, 120, (), 2), (2, 8, 1, 120, (), 3), (3, 8, 1, 120, (), 4),
    (3, 4, 3, 90, (), 5), (1, 3, 1, 200, "late", 6), (2, 8, 1, 200, "late", 7), (3, 8, 2, 200, "late", 8),
    (1, 8, 1, 7, (), 9), (3, 8, 1, 0, (), 10), (3, 8, 1, 61, (), 14), (3, 8, 1, 77, (), 15),
    (3, 6, 1, 200, "late", 16), (2, 8, 1, 53, (), 17),
    (5, 8, 1, 120, (), 18), (5, 4, 1, 150, (), 19), (5, 8, 2, 200, "late", 20), (5, 8, 1, 61, (), 22),
]


def late_stop(nid, prompt, gen):
    """Among the prompt's ids (so drafts can carry it), the one serial decode first emits
    latest (after 30 ids)."""
    out = serial(nid, prompt, gen, len(prompt) + gen + 1, ())
    first = {}
    for i, v in enumerate(out):
        if v in prompt:
            first.setdefault(v, i)
    if not first:
        return ()
    v, i = max(first.items(), key=lambda kv: kv[1])
    return (v,) if i >= 30 else ()


@pytest.mark.parametrize("policy,spec_n,min_len,gen,stops,seed", CASES)
def test_loop_equals_serial_decode_and_engine_restatement(k3, policy, spec_n, min_len, gen, stops, seed):
    nid = make_model(seed, vocab=12 if stops == "late" else 9)
    rng = np.random.default_rng(100 + seed)
    prompt = rng.integers(0, 9, 24).tolist()
    prompt += prompt[4:14]
    if stops == "late":
        stops = late_stop(nid, prompt, gen)
    tmax = len(prompt) + gen + 1 + (20 if seed % 2 == 0 else 0)   # even seeds: headroom past gen
    m = Fake(nid, [])
    loop = k3.SpecLoop(prompt, m.verify, m.commit, policy=policy, spec_n=spec_n, min_len=min_len, gen=gen,
                       tmax=tmax, stop_ids=stops)
    out, traces = loop.run()
    assert out == serial(nid, prompt, gen, tmax, stops)
    rout, rtrace, rst, rcached, rseq = O.spec_loop(nid, prompt, 0, policy, spec_n, min_len, gen, tmax, tmax,
                                                   set(stops))
    assert out == rout
    assert [(t["nd"], t["m"], t["keep"], t["fed"]) for t in traces] == rtrace
    s = loop.state()
    assert s["stats"] == rst and s["cached"] == rcached and loop.ids() == rseq
    assert m.state == rseq[:rcached]                      # the model consumed exactly the kept ids
    assert s["done"] in (k3.SPEC_LOOP_GEN, k3.SPEC_LOOP_STOP_ID, k3.SPEC_LOOP_CONTEXT)
    assert loop.step() == ([], None)                       # finished: nothing more
    if policy and len(out) > 30:
        assert s["stats"]["sweeps"] > 0 and s["stats"]["accepted"] > 0
        assert s["stats"]["partial"] > 0                   # the model does reject drafts
    loop.close()


def test_stop_id_inside_an_accepted_draft(k3):
    """A cyclic model accepts every draft; a stop id in the middle of an accepted draft cuts
    the sweep there (emit_keep), the state commits only up to it, and decoding ends."""
    nid = lambda ctx: (ctx[-1] + 1) % 6  # noqa: E731
    prompt = list(range(6)) * 3 + [0]
    for policy in (k3.DRAFT_NGRAM, k3.DRAFT_EAGER, k3.DRAFT_SUFFIX):
        m = Fake(nid, [])
        loop = k3.SpecLoop(prompt, m.verify, m.commit, policy=policy, gen=50, tmax=200, stop_ids=(4,))
        out, traces = loop.run()
        assert out == [1, 2, 3, 4] == serial(nid, prompt, 50, 200, (4,))
        s = loop.state()
        # the n-gram drafter (agreement gate) drafts only [2, 3] here: the stop id is the model's own
        assert s["done"] == k3.SPEC_LOOP_STOP_ID and s["stats"]["cut"] == (policy != k3.DRAFT_NGRAM)
        assert s["cached"] == len(prompt) + 3 and m.state == loop.ids()[:s["cached"]]
        rout, rtrace, rst, rcached, _ = O.spec_loop(nid, prompt, 0, policy, 8, 1, 50, 200, 200, {4})
        assert [(t["nd"], t["m"], t["keep"], t["fed"]) for t in traces] == rtrace and s["stats"] == rst
        loop.close()


def test_cases_reach_the_cut_paths(k3):
    """Among the cases, some sweep is cut short by the gen limit."""
    cuts = {"gen": 0, "stop": 0}
    for policy, spec_n, min_len, gen, stops, seed in CASES:
        nid = make_model(seed, vocab=12 if stops == "late" else 9)
        rng = np.random.default_rng(100 + seed)
        prompt = rng.integers(0, 9, 24).tolist()
        prompt += prompt[4:14]
        st = late_stop(nid, prompt, gen) if stops == "late" else stops
        tmax = len(prompt) + gen + 1 + (20 if seed % 2 == 0 else 0)
        out, tr, rst, _, _ = O.spec_loop(nid, prompt, 0, policy, spec_n, min_len, gen, tmax, tmax, set(st))
        if rst["cut"]:
            cuts["stop" if out and out[-1] in st else "gen"] += 1
    assert cuts["gen"] > 0, cuts


def test_loop_p3_policy_and_context_limits(k3):
    nid = make_model(11)
    prompt = list(range(9)) * 3
    q = np.full(k3.SPEC_P3_CODES, 0.8)
    for cost in (None, k3.K3SpecCost(0.44, 0.45, 0.11, 0.0, 56.0)):
        m = Fake(nid, [])
        loop = k3.SpecLoop(prompt, m.verify, m.commit, policy=k3.DRAFT_P3, gen=80, p3_q=q, p3_cost=cost)
        out, traces = loop.run()
        assert out == serial(nid, prompt, 80, len(prompt) + 81, ())
        assert max(t["nd"] for t in traces) > 0
        loop.close()
    # the context limit: drafting stops once T + spec_n + 1 reaches tmax, decoding at tmax
    m = Fake(nid, [])
    tmax = len(prompt) + 30
    loop = k3.SpecLoop(prompt, m.verify, m.commit, policy=k3.DRAFT_SUFFIX, gen=100, tmax=tmax)
    out, traces = loop.run()
    assert len(prompt) + len(out) == tmax and out == serial(nid, prompt, 100, tmax, ())
    assert loop.state()["done"] == k3.SPEC_LOOP_CONTEXT
    assert all(t["nd"] == 0 for t, T in zip(traces[1:], np.cumsum([len(prompt)] + [t["keep"] for t in traces])[1:])
               if T + 8 + 1 >= tmax)
    # a small cache: drafting needs cached + spec_n + 1 <= kv_cap
    m = Fake(nid, [])
    loop = k3.SpecLoop(prompt, m.verify, m.commit, policy=k3.DRAFT_SUFFIX, gen=40, kv_cap=len(prompt) + 5)
    out, traces = loop.run()
    assert out == serial(nid, prompt, 40, len(prompt) + 41, ()) and all(t["nd"] == 0 for t in traces)
    loop.close()


def test_loop_resume_reads_pending_plus_new_prompt(k3):
    """A resumed conversation: the model consumed all but the pending id; the first step
    feeds the pending id plus the new prompt (k3_run.c:2820-2828)."""
    nid = make_model(12)
    first = list(range(9)) * 2 + [3, 1, 4]
    m = Fake(nid, first[:-1])
    new = [1, 5, 9 % 9, 2, 6]
    loop = k3.SpecLoop(first + new, m.verify, m.commit, cached=len(first) - 1, policy=k3.DRAFT_NGRAM, gen=30)
    out, traces = loop.run()
    assert traces[0]["fed"] == len(new) + 1 and m.calls[0] == len(new) + 1
    assert out == serial(nid, first + new, 30, len(first + new) + 31, ())
    loop.close()


def test_loop_errors(k3):
    nid = make_model(13)
    m = Fake(nid, [])
    with pytest.raises(k3.K3Error):
        k3.SpecLoop([1, 2], m.verify, m.commit, cached=2)            # nothing left to read
    with pytest.raises(k3.K3Error):
        k3.SpecLoop([1, 2], m.verify, m.commit, spec_n=9)            # above the draft cap
    with pytest.raises(k3.K3Error):
        k3.SpecLoop([1, 2], m.verify, m.commit, policy=k3.DRAFT_P3)  # P3 without a table

    def bad_verify(ids, base, parent=None):
        raise RuntimeError("device lost")
    loop = k3.SpecLoop([1, 2, 3], bad_verify, m.commit)
    with pytest.raises(k3.K3Error) as e:
        loop.step()
    assert isinstance(e.value.__cause__, RuntimeError)
    loop.close()


class FakeDraft:
    """A draft model holding its consumed positions: several tentative verify calls, each
    continuing where the previous one ended, then one commit of the first `keep`."""

    def __init__(self, next_id):
        self.next_id, self.state, self.pending = next_id, [], []

    def verify(self, ids, base, parent=None):
        assert parent is None and base == len(self.state) + len(self.pending)
        out = [self.next_id(self.state + self.pending + ids[:i + 1]) for i in range(len(ids))]
        self.pending += list(ids)
        return out

    def commit(self, base, keep, path=None):
        assert path is None and base == len(self.state) and 0 <= keep <= len(self.pending)
        self.state += self.pending[:keep]
        self.pending = []


@pytest.mark.parametrize("seed,spec_n,gen,stops,noise", [(31, 8, 120, (), 3), (32, 4, 100, (), 4),
                                                          (33, 8, 77, (), 2), (34, 6, 150, "late", 3),
                                                          (35, 3, 90, (), 1)])
def test_draft_model_loop(k3, seed, spec_n, gen, stops, noise):
    """The engine's --draft mode: a second model proposes spec_n ids a round. The generated
    ids equal serial decoding of the target, the trace and every counter equal the engine
    loop's restatement, and the draft model consumed exactly a prefix of the conversation."""
    nid = make_model(seed, vocab=12 if stops == "late" else 9)
    dnid = make_model(seed, vocab=12 if stops == "late" else 9, noise=noise)   # same table, other deviations
    rng = np.random.default_rng(200 + seed)
    prompt = rng.integers(0, 9, 24).tolist()
    prompt += prompt[4:14]
    if stops == "late":
        stops = late_stop(nid, prompt, gen)
    tmax = len(prompt) + gen + 21
    m, dm = Fake(nid, []), FakeDraft(dnid)
    loop = k3.SpecLoop(prompt, m.verify, m.commit, policy=k3.DRAFT_MODEL, spec_n=spec_n, gen=gen, tmax=tmax,
                       stop_ids=stops, draft_verify=dm.verify, draft_commit=dm.commit)
    out, traces = loop.run()
    assert out == serial(nid, prompt, gen, tmax, stops)
    rout, rtrace, rst, rcached, rseq = O.spec_loop(nid, prompt, 0, 6, spec_n, 1, gen, tmax, tmax, set(stops),
                                                   draft_next=dnid)
    assert [(t["nd"], t["m"], t["keep"], t["fed"]) for t in traces] == rtrace
    s = loop.state()
    assert s["stats"] == rst and s["cached"] == rcached and loop.ids() == rseq
    assert m.state == rseq[:rcached] and dm.pending == []
    assert dm.state == rseq[:len(dm.state)] and len(dm.state) >= rcached - 1
    st = s["stats"]
    assert st["draft_rounds"] == st["sweeps"] and st["draft_drafted"] == st["drafted"]
    assert st["draft_accepted"] == st["accepted"] and st["sweeps"] > 0
    loop.close()


def test_draft_model_that_never_agrees_and_a_missing_model(k3):
    nid = make_model(41)
    prompt = list(range(9)) * 3
    m, dm = Fake(nid, []), FakeDraft(lambda ctx: (nid(ctx) + 1) % 9)      # always wrong
    loop = k3.SpecLoop(prompt, m.verify, m.commit, policy=k3.DRAFT_MODEL, gen=40, draft_verify=dm.verify,
                       draft_commit=dm.commit)
    out, traces = loop.run()
    assert out == serial(nid, prompt, 40, len(prompt) + 41, ())
    assert loop.state()["stats"]["draft_accepted"] == 0 and loop.state()["stats"]["draft_dropped"] > 0
    loop.close()
    m2 = Fake(nid, [])
    loop = k3.SpecLoop(prompt, m2.verify, m2.commit, policy=k3.DRAFT_MODEL, gen=10)
    with pytest.raises(k3.K3Error):
        loop.step()                                                      # no draft model set
    loop.close()


def test_prompt_read_in_passes_checkpoints_and_pause(k3):
    """--prefill-chunk / --checkpoint / --pause-after (src/cli/k3_run.c:1189-1240): the
    prompt is read in passes of at most N positions, a checkpoint follows every pass that
    leaves positions to go, and after pause_after checkpoints the step stops having
    emitted nothing; a new loop created at the positions read continues, and the run as a
    whole decodes exactly as serial decoding does."""
    nid = make_model(51)
    rng = np.random.default_rng(51)
    prompt = rng.integers(0, 9, 34).tolist()
    # passes of 7 with checkpoints at 7, 14, 21, 28 (not after the last pass)
    m, marks = Fake(nid, []), []
    loop = k3.SpecLoop(prompt, m.verify, m.commit, policy=k3.DRAFT_SUFFIX, gen=30, prefill_chunk=7,
                       checkpoint=marks.append)
    out, traces = loop.run()
    assert m.calls[:5] == [7, 7, 7, 7, 6] and marks == [7, 14, 21, 28]
    assert traces[0]["fed"] == 34 and out == serial(nid, prompt, 30, len(prompt) + 31, ())
    loop.close()
    # pause after 2 checkpoints, then resume from position 14
    m, marks = Fake(nid, []), []
    loop = k3.SpecLoop(prompt, m.verify, m.commit, policy=k3.DRAFT_SUFFIX, gen=30, prefill_chunk=7,
                       pause_after=2, checkpoint=marks.append)
    assert loop.step() == ([], None)
    st = loop.state()
    assert st["done"] == k3.SPEC_LOOP_PAUSED and st["cached"] == 14 and st["nout"] == 0 and marks == [7, 14]
    assert m.state == prompt[:14]
    loop.close()
    loop = k3.SpecLoop(prompt, m.verify, m.commit, cached=14, policy=k3.DRAFT_SUFFIX, gen=30, prefill_chunk=7)
    out, traces = loop.run()
    assert traces[0]["fed"] == 20 and out == serial(nid, prompt, 30, len(prompt) + 31, ())
    loop.close()
    # a pause requested before the read-in takes effect at the first checkpoint
    m, marks = Fake(nid, []), []
    loop = k3.SpecLoop(prompt, m.verify, m.commit, prefill_chunk=10, checkpoint=marks.append)
    loop.request_pause()
    loop.step()
    assert loop.state()["done"] == k3.SPEC_LOOP_PAUSED and loop.state()["cached"] == 10 and marks == [10]
    loop.close()
    # without a checkpoint callback pause_after has nothing to pause on: the read-in completes
    m = Fake(nid, [])
    loop = k3.SpecLoop(prompt, m.verify, m.commit, gen=5, prefill_chunk=10, pause_after=1)
    out, _ = loop.run()
    assert out == serial(nid, prompt, 5, len(prompt) + 6, ())
    loop.close()


def test_draft_model_reads_the_prompt_in_the_same_passes(k3):
    nid = make_model(52)
    prompt = np.random.default_rng(52).integers(0, 9, 30).tolist()
    m, dm = Fake(nid, []), FakeDraft(make_model(52, noise=3))
    calls = []

    def dverify(ids, base, parent=None):
        calls.append(len(ids))
        return dm.verify(ids, base, parent)
    loop = k3.SpecLoop(prompt, m.verify, m.commit, policy=k3.DRAFT_MODEL, gen=40, prefill_chunk=8,
                       draft_verify=dverify, draft_commit=dm.commit)
    out, _ = loop.run()
    assert calls[:4] == [8, 8, 8, 6] and out == serial(nid, prompt, 40, len(prompt) + 41, ())
    loop.close()


def test_layer_loop_plan(k3):
    """The --loop / --loop-layers / --loop-count execution order (src/cli/k3_run.c:
    2140-2182): whole AttnRes blocks only, the middle block as the preset, each executed
    position its own slot, the stride growth (R - 1) * ceil(span / block)."""
    vmap, span, extra = k3.layer_loop_plan(12, 3, 2, span=(3, 5))
    assert vmap == [0, 1, 2, 3, 4, 5, 3, 4, 5, 6, 7, 8, 9, 10, 11] and span == (3, 5) and extra == 1
    vmap, span, extra = k3.layer_loop_plan(12, 3, 3, span=(3, 8))
    assert vmap == list(range(9)) + list(range(3, 9)) * 2 + [9, 10, 11] and extra == 4
    vmap, span, extra = k3.layer_loop_plan(93, 4, 2, preset=True)       # K3: the block holding layer 46
    assert span == (44, 47) and len(vmap) == 97 and vmap[48:52] == [44, 45, 46, 47] and extra == 1
    vmap, span, _ = k3.layer_loop_plan(13, 3, 2, span=(12, 12))        # a last, partial block
    assert vmap == list(range(13)) + [12]
    for bad in ((4, 5), (3, 4), (2, 5), (3, 12)):                      # cut blocks, past the stack
        with pytest.raises(k3.K3Error):
            k3.layer_loop_plan(12, 3, 2, span=bad)
    with pytest.raises(k3.K3Error):
        k3.layer_loop_plan(12, 3, 9, span=(3, 5))                      # at most 8 passes
    vmap, _, extra = k3.layer_loop_plan(12, 3, 1, span=(3, 5))          # one pass: the plain stack
    assert vmap == list(range(12)) and extra == 0
