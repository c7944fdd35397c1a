"""The whole-model verify forward on a B200 against the reference engine's own token streams
(tests/golden/c1_golden.npz from tests/golden/make_c1_golden.py).

The checkpoint is regenerated from the same seeded call the goldens were made with; the
model is bound from it by the package's config reader, tensor index, binder and expert
loader, and runs entirely in libk3gpu.so (k3gpu_model_*). The contract (BASELINE
north_star): greedy token streams bit-identical to the reference's, logits within max-abs
2e-2 and relative L2 1e-3 of the reference's fp32 logits, the KDA state within relative L2
1e-4 -- at every acceptance count of a verify sweep (the reference's GATE 4,
tests/unit/k3_model.c:359-462, and its crafted-prompt CLI test,
tests/test_offline_cli.py:890-958).
"""
from __future__ import annotations

import importlib.util
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden", "c1_golden.npz")
LOGIT_MAX_ABS = 2e-2
LOGIT_REL_L2 = 1e-3
STATE_REL_L2 = 1e-4
SPEC = 4

pytestmark = pytest.mark.gpu


def _load(name, rel):
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def k3():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tests.k3lib import load
    return load()


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(GOLD))


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    synth = _load("k3synth_t", "kimi-k3-for-me_b200/synth.py")
    return synth.write_checkpoint(str(tmp_path_factory.mktemp("c1")), seed=0, recipe="reference")


@pytest.fixture(scope="module")
def model(k3, ckpt):
    m = k3.Model.from_checkpoint(ckpt, B=1, max_T=64, kv_cap=256)
    yield m
    m.close()


def logits_ok(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    mx = np.abs(got - ref).max()
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert mx <= LOGIT_MAX_ABS and rel <= LOGIT_REL_L2, f"{what}: logits max-abs {mx:.3g}, rel-L2 {rel:.3g}"


def ids_dev(ids):
    return torch.tensor([ids], dtype=torch.int32, device="cuda")


def test_serial_stream_and_logits(k3, model, gold):
    """The uniform-random 32-id prompt, greedy 64 ids one position at a time: every id equal
    to the reference's and every logit vector within tolerance (the first from a one-position
    sweep of the prompt's last id after reading in the rest)."""
    model.reset()
    prompt, ref_ids, ref_lg = gold["base/prompt"].tolist(), gold["base/ids"], gold["base/logits"]
    model.prefill(ids_dev(prompt[:-1]))
    pending, got = prompt[-1], []
    for i in range(len(ref_ids)):
        arg, lg = model.verify(ids_dev([pending]))
        logits_ok(lg[0, 0].cpu().numpy(), ref_lg[i], f"step {i}")
        got.append(int(arg[0, 0]))
        model.commit([1])
        assert got[i] == ref_ids[i], f"id {i}: {got[i]} vs the reference's {ref_ids[i]}"
        pending = got[-1]
    assert got == ref_ids.tolist()
    assert model.cached() == [len(prompt) + len(ref_ids) - 1]
    assert k3.device_status() == 0


def test_greedy_sweep_fused_argmax_gives_the_reference_ids(k3, model, gold):
    """The same serial stream with the lm_head fused with the argmax (no logits written,
    k3gpu_model_verify_greedy): every id equal to the reference's, and the fused argmax of a
    whole-prompt sweep equal to the argmax of that sweep's written logits."""
    model.reset()
    prompt, ref_ids = gold["base/prompt"].tolist(), gold["base/ids"]
    arg_l, lg = model.verify(ids_dev(prompt))
    want = arg_l.clone()
    arg_f, none = model.verify(ids_dev(prompt), logits=False)   # the sweep is tentative: same state
    assert none is None
    np.testing.assert_array_equal(arg_f.cpu().numpy(), want.cpu().numpy())
    model.reset()
    model.prefill(ids_dev(prompt[:-1]))
    pending, got = prompt[-1], []
    for i in range(len(ref_ids)):
        arg, _ = model.verify(ids_dev([pending]), logits=False)
        got.append(int(arg[0, 0]))
        model.commit([1])
        pending = got[-1]
    assert got == ref_ids.tolist()
    assert k3.device_status() == 0


def test_native_loop_equals_reference_and_state(k3, model, gold):
    """The engine's decode loop in C (k3_spec_loop) over the model's native callbacks, the
    reference's drafter at spec 4: the same 64 ids, no sweep fired (as in the reference
    run), and the carried state after the run equal to the state the reference saved."""
    model.reset()
    prompt, ref_ids = gold["base/prompt"].tolist(), gold["base/ids"].tolist()
    loop = model.spec_loop(prompt, policy=k3.DRAFT_NGRAM, spec_n=SPEC, gen=64, kv_cap=model.kv_cap)
    ids, _ = loop.run()
    st = loop.state()
    loop.close()
    assert ids == ref_ids
    assert st["stats"]["sweeps"] == int(gold["base/sweeps"])
    cached = int(gold["base/state_cached"])
    assert model.cached() == [cached]
    c = model.lcfg
    H, D, K = c.kda_heads, c.kda_head_dim, c.conv_k
    P = H * D
    ks = gold["base/state_kda"]
    n_mla = 0
    for layer in range(model.cfg["num_hidden_layers"]):
        if (layer + 1) in model.cfg["full_attn_layers"]:
            lat, rope = model.mla_cache(layer)
            ref_lat = gold["base/state_lat"][n_mla, :cached]
            got = (lat[0, :cached].cpu().numpy().astype(np.uint16).astype(np.uint32) << 16).view(np.float32)
            ref_rope = gold["base/state_rope"][n_mla, :cached]
            gr = (rope[0, :cached].cpu().numpy().astype(np.uint16).astype(np.uint32) << 16).view(np.float32)
            # the library keeps the cache in bf16 (relative rounding error at most 2^-9 per
            # element) over rows the reference keeps in fp32
            for name, g, r in (("latent", got, ref_lat), ("rope", gr, ref_rope)):
                rel = np.linalg.norm(g - r) / np.linalg.norm(r)
                assert rel <= 2.0 ** -8, f"layer {layer} {name} cache rel-L2 {rel:.3g}"
            n_mla += 1
            continue
        state, hist = model.kda_state(layer)
        ref_s = ks[layer, :H * D * D]
        ref_h = ks[layer, H * D * D:H * D * D + 3 * P * (K - 1)]
        got_s = state[0].reshape(-1).cpu().numpy()
        got_h = hist[0].reshape(-1).cpu().numpy()
        rel_s = np.linalg.norm(got_s - ref_s) / np.linalg.norm(ref_s)
        rel_h = np.linalg.norm(got_h - ref_h) / np.linalg.norm(ref_h)
        assert rel_s <= STATE_REL_L2, f"layer {layer} KDA state rel-L2 {rel_s:.3g}"
        assert rel_h <= STATE_REL_L2, f"layer {layer} ShortConv history rel-L2 {rel_h:.3g}"
    assert k3.device_status() == 0


@pytest.mark.parametrize("accept", range(SPEC + 1))
def test_crafted_sweep_accepts_as_the_reference(k3, model, gold, accept):
    """A prompt whose first verify sweep drafts 4 ids of which the reference accepted exactly
    `accept`: the native loop's stream and trace equal the reference's, and the sweep's
    logits for the kept positions equal the reference's within tolerance."""
    prompt = gold[f"craft{accept}/prompt"].tolist()
    ref_ids = gold[f"craft{accept}/ids"].tolist()
    ref_trace = gold[f"craft{accept}/trace"].tolist()
    model.reset()
    loop = model.spec_loop(prompt, policy=k3.DRAFT_NGRAM, spec_n=SPEC, gen=len(ref_ids), kv_cap=model.kv_cap)
    ids, trace = [], []
    while True:
        kept, tr = loop.step()
        if not kept:
            break
        ids += kept
        if tr and tr["nd"] > 0:
            trace.append([tr["nd"], tr["m"], tr["keep"]])
    loop.close()
    assert ids == ref_ids
    assert trace == ref_trace
    # the first sweep by hand: the pending id and the reference's four drafts in one pass
    model.reset()
    nxt = int(model.prefill(ids_dev(prompt)).item())
    assert nxt == ref_ids[0]
    seq = prompt + [nxt]
    d = k3.spec_draft(seq, SPEC)
    assert len(d) == SPEC
    arg, lg = model.verify(ids_dev([nxt] + d))
    ref_lg = gold[f"craft{accept}/logits"]
    for i in range(accept + 1):
        logits_ok(lg[0, i].cpu().numpy(), ref_lg[1 + i], f"sweep position {i}")
        assert int(arg[0, i]) == ref_ids[1 + i]
    m = 0
    while m < SPEC and int(arg[0, m]) == d[m]:
        m += 1
    assert m == accept
    model.commit([m + 1])
    assert k3.device_status() == 0


def test_forced_drafts_every_acceptance_count(k3, model, gold):
    """GATE 4 on the device: drafts are the reference's own continuation with one planted
    wrong id at position p (none for p = SPEC); each sweep accepts exactly p, commits p + 1
    positions, and the stream, every kept position's logits and the final KDA state equal
    the serial run's."""
    prompt, ref_ids, ref_lg = gold["base/prompt"].tolist(), gold["base/ids"].tolist(), gold["base/logits"]
    model.reset()
    nxt = int(model.prefill(ids_dev(prompt)).item())
    out = [nxt]
    step = 0
    while len(out) < len(ref_ids) - SPEC - 1:
        p = step % (SPEC + 1)
        n = len(out)
        drafts = list(ref_ids[n:n + SPEC])
        if p < SPEC:
            drafts[p] = (drafts[p] + 1) % model.vocab
        arg, lg = model.verify(ids_dev([out[-1]] + drafts))
        a = arg[0].tolist()
        m = 0
        while m < SPEC and a[m] == drafts[m]:
            m += 1
        assert m == p, f"step {step}: accepted {m}, planted the wrong id at {p}"
        emit = drafts[:m] + [a[m]]
        for i in range(m + 1):
            logits_ok(lg[0, i].cpu().numpy(), ref_lg[n + i], f"step {step} position {i}")
        model.commit([m + 1])
        out += emit
        assert out == ref_ids[:len(out)], f"stream diverged at step {step}"
        step += 1
    assert step >= 2 * (SPEC + 1)
    assert k3.device_status() == 0


def test_batched_sequences_are_independent(k3, ckpt, gold):
    """B = 2: the reference's prompt beside another, one sweep per step for both; the first
    sequence's stream equals the reference's, the second equals its own B = 1 run."""
    other = [(7 * i + 3) % 1024 for i in range(32)]
    prompt = gold["base/prompt"].tolist()
    ref_ids = gold["base/ids"].tolist()[:16]
    m1 = k3.Model.from_checkpoint(ckpt, B=1, max_T=8, kv_cap=64)
    nxt = int(m1.prefill(ids_dev(other)).item())
    solo = [nxt]
    for _ in range(15):
        arg, _ = m1.verify(ids_dev([solo[-1]]))
        m1.commit([1])
        solo.append(int(arg[0, 0]))
    m1.close()
    m2 = k3.Model.from_checkpoint(ckpt, B=2, max_T=8, kv_cap=64)
    nxt = m2.prefill(torch.tensor([prompt, other], dtype=torch.int32, device="cuda")).tolist()
    outs = [[nxt[0]], [nxt[1]]]
    for _ in range(15):
        arg, _ = m2.verify(torch.tensor([[outs[0][-1]], [outs[1][-1]]], dtype=torch.int32, device="cuda"))
        m2.commit([1, 1])
        outs[0].append(int(arg[0, 0]))
        outs[1].append(int(arg[1, 0]))
    m2.close()
    assert outs[0] == ref_ids
    assert outs[1] == solo
    assert k3.device_status() == 0


def test_tree_sweep_through_kda_and_mla_layers(k3, model, gold):
    """A draft TREE over the reference's continuation with decoy branches, verified in one
    sweep through the 3 KDA layers (recurrence and ShortConv along each node's ancestors)
    and the MLA layer (ancestor masks): the nodes on the true branch carry the reference's
    serial logits, a decoy node's logits equal a chain sweep of its own path, the on-device
    greedy tree walk accepts the true branch, and after the path's commit the stream goes on
    exactly as the reference's."""
    prompt, y, ref_lg = gold["base/prompt"].tolist(), gold["base/ids"].tolist(), gold["base/logits"]
    V = model.vocab
    w = [(y[1] + 11) % V, (y[1] + 23) % V, (y[2] + 5) % V, (y[3] + 7) % V, 3]
    #        0     1     2     3     4     5     6     7     8
    tok = [y[0], w[0], y[1], w[1], w[4], y[2], w[2], w[3], y[3]]
    parent = [-1, 0, 0, 0, 1, 2, 2, 5, 5]
    model.reset()
    assert int(model.prefill(ids_dev(prompt)).item()) == y[0]
    arg, lg = model.verify(ids_dev(tok), parent=parent)
    for node, ref_row in ((0, 1), (2, 2), (5, 3), (8, 4)):
        logits_ok(lg[0, node].cpu().numpy(), ref_lg[ref_row], f"true-branch node {node}")
        assert int(arg[0, node]) == y[ref_row]
    tree_lg = lg[0].cpu().numpy().copy()
    # the decoy node 4 (path 0 -> 1 -> 4) against a chain sweep of that path
    arg_c, lg_c = model.verify(ids_dev([tok[0], tok[1], tok[4]]))
    got, ref = tree_lg[4].astype(np.float64), lg_c[0, 2].cpu().numpy().astype(np.float64)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5
    # the tree again, accepted on the device, and its path committed
    arg, lg = model.verify(ids_dev(tok), parent=parent)
    emit, n_emit, path, _ = k3.accept_tree_greedy(lg, ids_dev(tok), torch.tensor(parent, dtype=torch.int32,
                                                                                    device="cuda"))
    n = int(n_emit[0])
    assert n == 4 and emit[0, :n].tolist() == y[1:5]
    assert path[0, :n].tolist() == [0, 2, 5, 8]
    model.commit([n], [path[0].tolist()])
    out = y[:5]
    for i in range(5, 14):
        a, lgs = model.verify(ids_dev([out[-1]]))
        logits_ok(lgs[0, 0].cpu().numpy(), ref_lg[i], f"step {i} after the tree commit")
        model.commit([1])
        out.append(int(a[0, 0]))
    assert out == y[:14]
    assert k3.device_status() == 0
