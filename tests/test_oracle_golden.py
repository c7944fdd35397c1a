"""Pin the CPU restatement (oracle/k3_oracle.c) to the reference's own golden vectors.

No GPU. Every check here compares liborc.so with either a fixture the reference checks in
(converted into tests/golden/ops_fixtures.npz and mxfp4_fixture.npz) or with outputs of
the reference's own C kernels on seeded inputs (tests/golden/ref_*.npz). Bit-exact where
the oracle promises the reference's arithmetic; the reference fixtures' own tolerance
(abs 1e-5, rel 1e-4, tests/fixtures/ops/MANIFEST.json of the reference) where the
fixture came from torch.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.golden import inputs as GI

G = os.path.join(os.path.dirname(__file__), "golden")
OPS = np.load(os.path.join(G, "ops_fixtures.npz"))


def fx(name, key):
    return np.ascontiguousarray(OPS[f"{name}/{key}"], np.float32)


def close(got, want, atol=1e-5, rtol=1e-4):
    np.testing.assert_allclose(got, want, atol=atol, rtol=rtol)


# ------------------------------------------------------------------------- router --
def test_router_fixture():
    x, W, b = fx("router", "in"), fx("router", "gate_weight"), fx("router", "bias")
    k = int(OPS["router/top_k"])
    idx, w = O.router(x, W, b, k)
    np.testing.assert_array_equal(idx, OPS["router/topk_idx"].astype(np.int32))
    close(w, fx("router", "topk_weight"))


@pytest.mark.parametrize("case", GI.ROUTER_CASES, ids=lambda c: c["name"])
def test_router_bitexact_vs_reference_kernel(case):
    g = np.load(os.path.join(G, "ref_router.npz"))
    x, W, b = GI.router_inputs(case)
    idx, w = O.router(x, W, b, case["topk"])
    np.testing.assert_array_equal(idx, g[case["name"] + "/idx"])
    np.testing.assert_array_equal(w.view(np.uint32), g[case["name"] + "/w"].view(np.uint32))


def test_router_ties_take_first_index():
    case = [c for c in GI.ROUTER_CASES if c["name"] == "ties"][0]
    x, W, b = GI.router_inputs(case)
    idx, _ = O.router(x, W, b, case["topk"])
    for row in idx:
        for e in row:
            if e % 2 == 1:   # the odd twin may only follow its even twin
                assert (e - 1) in row.tolist()[: row.tolist().index(e)]


# -------------------------------------------------------------------------- MXFP4 --
def test_mxfp4_dequant_released_bytes_exact():
    d = np.load(os.path.join(G, "mxfp4_fixture.npz"))
    rows, width = int(d["rows"]), int(d["logical_width"])
    out = np.zeros((rows, width), np.float32)
    O.orc().orc_mxfp4_dequant(out, d["packed"], d["scales"], rows, width)
    np.testing.assert_array_equal(out.view(np.uint32), d["expected"].view(np.uint32))
    # the swapped nibble order must NOT reproduce (the fixture records what it gives)
    assert not np.array_equal(out.ravel()[:64], d["swapped_first64"])


@pytest.mark.parametrize("case", GI.MXFP4_CASES, ids=lambda c: c["name"])
def test_mxfp4_matmul_vs_reference_kernel(case):
    g = np.load(os.path.join(G, "ref_mxfp4.npz"))
    packed, scales, x = GI.mxfp4_inputs(case)
    y = np.zeros(case["rows"], np.float32)
    O.orc().orc_matmul_mxfp4(y, x, packed, scales, case["in"], case["rows"])
    # double accumulation in another order: agreement to ~1 ulp of float
    np.testing.assert_allclose(y, g[case["name"] + "/y"], rtol=2e-7, atol=1e-9)


# ---------------------------------------------------------------------------- KDA --
@pytest.mark.parametrize("name", ["kda_recur1", "kda_recur8"])
def test_kda_recurrence_fixture(name):
    q, k, v = fx(name, "q"), fx(name, "k"), fx(name, "v")
    al, be = fx(name, "alpha"), fx(name, "beta")
    T, H, D = q.shape
    st0 = np.zeros((H, D, D), np.float32)
    o = O.kda_verify(st0, q, k, v, al, be, float(OPS[f"{name}/q_scale"]))
    close(o, fx(name, "out"))
    st = O.kda_commit(st0, k, v, al, be, T)
    close(st, fx(name, "state_out"))


@pytest.mark.parametrize("case", GI.KDA_CASES, ids=lambda c: c["name"])
def test_kda_verify_and_commit_bitexact_vs_reference_kernel(case):
    g = np.load(os.path.join(G, "ref_kda.npz"))
    st0, q, k, v, al, be = GI.kda_inputs(case)
    D = q.shape[2]
    o = O.kda_verify(st0, q, k, v, al, be, np.float32(1.0) / np.sqrt(np.float32(D)))
    np.testing.assert_array_equal(o.view(np.uint32), g[case["name"] + "/o"].view(np.uint32))
    for n in case["commits"]:
        st = O.kda_commit(st0, k, v, al, be, n)
        np.testing.assert_array_equal(st.view(np.uint32),
                                      g[case["name"] + f"/state_n{n}"].view(np.uint32))


def test_kda_decay_fixture():
    z, A, dt = fx("kda_decay", "z"), fx("kda_decay", "A_log"), fx("kda_decay", "dt_bias")
    H, D = A.shape[0], dt.shape[0] // A.shape[0]
    zf = z.reshape(-1, H * D)
    g = np.zeros_like(zf)
    a = np.zeros_like(zf)
    for t in range(zf.shape[0]):
        gt, at = np.zeros(H * D, np.float32), np.zeros(H * D, np.float32)
        O.orc().orc_kda_decay(gt, at, np.ascontiguousarray(zf[t]), A, dt, H, D,
                              float(OPS["kda_decay/lower_bound"]))
        g[t], a[t] = gt, at
    close(g.ravel(), fx("kda_decay", "g").ravel())
    close(a.ravel(), fx("kda_decay", "alpha").ravel())


def test_shortconv_fixture_with_carried_history():
    w = fx("shortconv", "weight").reshape(64, 4)
    x = fx("shortconv", "in")[0]
    hist = np.zeros((64, 3), np.float32)
    y = np.zeros_like(x)
    O.orc().orc_shortconv(y, x, w, hist.ctypes.data, 64, 4, x.shape[0])
    close(y, fx("shortconv", "out")[0])
    close(hist, fx("shortconv", "state_after")[0])
    xn = fx("shortconv", "in_next")[0]
    yn = np.zeros_like(xn)
    O.orc().orc_shortconv(yn, xn, w, hist.ctypes.data, 64, 4, 1)
    close(yn, fx("shortconv", "out_next")[0])


def test_kda_layer_fixture_composition():
    """The whole KDA layer (src/core/k3_ops.c:2231-2385) composed from the oracle's
    prologue, recurrence and norm/gate with double-accumulated projections."""
    for name in ("kda_layer1", "kda_layer8"):
        x = fx(name, "in")[0]
        T, E = x.shape
        H, D, K = int(OPS[f"{name}/H"]), int(OPS[f"{name}/d_k"]), int(OPS[f"{name}/conv_k"])
        P = H * D
        q = O.matmul_d(x, fx(name, "q_proj"))
        k = O.matmul_d(x, fx(name, "k_proj"))
        v = O.matmul_d(x, fx(name, "v_proj"))
        b = O.matmul_d(x, fx(name, "b_proj"))
        z = O.matmul_d(O.matmul_d(x, fx(name, "f_a")), fx(name, "f_b"))
        al = np.zeros((T, P), np.float32)
        be = np.zeros((T, H), np.float32)
        hist = np.zeros((3, P, K - 1), np.float32)
        O.orc().orc_kda_prologue(q, k, v, al, be, z, b, fx(name, "q_conv").reshape(P, K),
                                 fx(name, "k_conv").reshape(P, K), fx(name, "v_conv").reshape(P, K),
                                 hist.ctypes.data, fx(name, "A_log"), fx(name, "dt_bias"), T, H, D,
                                 K, float(OPS[f"{name}/lower_bound"]))
        st0 = np.zeros((H, D, D), np.float32)
        sh = (T, H, D)
        o = O.kda_verify(st0, q.reshape(sh), k.reshape(sh), v.reshape(sh), al.reshape(sh), be,
                         np.float32(1.0) / np.sqrt(np.float32(D)))
        st = O.kda_commit(st0, k.reshape(sh), v.reshape(sh), al.reshape(sh), be, T)
        gate = O.matmul_d(x, fx(name, "g_proj"))
        o = np.ascontiguousarray(o)
        O.orc().orc_kda_norm_gate(o, gate, fx(name, "o_norm"), T, H, D, float(OPS[f"{name}/rms_eps"]))
        out = O.matmul_d(o.reshape(T, P), fx(name, "o_proj"))
        close(out, fx(name, "out")[0])
        close(st, fx(name, "state_out")[0])


# ------------------------------------------------------------------- small ops ---
def test_situ_glu_rmsnorm_attnres_fixtures():
    x = fx("situ_glu", "in")
    n = x.shape[1] // 2
    for r in range(x.shape[0]):
        y = np.zeros(n, np.float32)
        O.orc().orc_situ_glu(y, np.ascontiguousarray(x[r]), n, 4.0, 25.0)
        close(y, fx("situ_glu", "out")[r])
    close(O.rmsnorm(fx("rmsnorm", "in"), fx("rmsnorm", "weight"), 1e-5), fx("rmsnorm", "out"))
    fold = fx("attnres", "norm_weight") * fx("attnres", "proj_weight")
    ps, br = fx("attnres", "prefix_sum"), fx("attnres", "block_residual")
    for t in range(ps.shape[0]):
        src = np.ascontiguousarray(np.concatenate([br[t], ps[t:t + 1]], 0))
        out = np.zeros(ps.shape[1], np.float32)
        O.orc().orc_attn_res(out, src, fold.astype(np.float32), src.shape[0], src.shape[1], 1e-5)
        close(out, fx("attnres", "out")[t])


# ---------------------------------------------------------------------------- MLA --
def test_mla_fixture_absorbed_composition():
    """orc_mla_absorbed inside the whole gated NoPE MLA, against the reference's torch
    fixture (expanded attention; absorption is exact in real arithmetic)."""
    cfg = dict(n_heads=int(OPS["mla/n_heads"]), qk_nope=int(OPS["mla/qk_nope"]),
               qk_rope=int(OPS["mla/qk_rope"]), v_head=int(OPS["mla/v_head"]),
               kv_lora=int(OPS["mla/kv_lora"]), eps=float(OPS["mla/rms_eps"]))
    wts = dict(q_a=fx("mla", "q_a_proj_weight"), q_a_norm=fx("mla", "q_a_layernorm_weight"),
               q_b=fx("mla", "q_b_proj_weight"), kv_a=fx("mla", "kv_a_proj_with_mqa_weight"),
               kv_a_norm=fx("mla", "kv_a_layernorm_weight"), kv_b=fx("mla", "kv_b_proj_weight"),
               o=fx("mla", "o_proj_weight"), g=fx("mla", "g_proj_weight"))
    out = O.mla_forward(fx("mla", "in")[0], wts, cfg)
    close(out, fx("mla", "out")[0])


def test_mla_tree_mask_equals_chain_on_a_chain():
    rng = np.random.default_rng(5)
    T, H, qn, qr, vh, kvl, cached = 5, 3, 16, 8, 16, 32, 7
    qn_, qr_ = rng.standard_normal((T, H, qn), dtype=np.float32), rng.standard_normal((T, H, qr), dtype=np.float32)
    kvb = rng.standard_normal((H * (qn + vh), kvl), dtype=np.float32) * np.float32(0.2)
    lat = rng.standard_normal((cached + T, kvl), dtype=np.float32)
    rope = rng.standard_normal((cached + T, qr), dtype=np.float32)
    a = O.mla_absorbed(qn_, qr_, kvb, lat, rope, cached, O.chain_masks(T), 0.2, vh)
    b = O.mla_absorbed(qn_, qr_, kvb, lat, rope, cached, O.tree_masks([-1, 0, 1, 2, 3]), 0.2, vh)
    np.testing.assert_array_equal(a, b)
    # a sibling must not see its brother: node 2 under root 0 next to node 1
    c = O.mla_absorbed(qn_, qr_, kvb, lat, rope, cached, O.tree_masks([-1, 0, 0, 1, 2]), 0.2, vh)
    assert not np.array_equal(a[2], c[2])
    np.testing.assert_array_equal(a[:2], c[:2])


def _random_tree(rng, T):
    return [-1] + [int(rng.integers(0, i)) for i in range(1, T)]


def test_mla_tree_node_equals_its_ancestor_chain():
    """What a tree mask means: node i's output equals a plain causal run over just the
    path root .. i (its ancestors' rows, in order), for every node of random trees."""
    rng = np.random.default_rng(8)
    H, qn, qr, vh, kvl, cached = 3, 16, 8, 16, 32, 9
    for T in (6, 17, 40):
        parent = _random_tree(rng, T)
        qn_ = rng.standard_normal((T, H, qn), dtype=np.float32)
        qr_ = rng.standard_normal((T, H, qr), dtype=np.float32)
        kvb = rng.standard_normal((H * (qn + vh), kvl), dtype=np.float32) * np.float32(0.2)
        lat = rng.standard_normal((cached + T, kvl), dtype=np.float32)
        rope = rng.standard_normal((cached + T, qr), dtype=np.float32)
        tree = O.mla_absorbed(qn_, qr_, kvb, lat, rope, cached, O.tree_masks(parent), 0.2, vh)
        for i in range(T):
            path, j = [], i
            while j >= 0:
                path.append(j)
                j = parent[j]
            path = path[::-1]
            n = len(path)
            lat_c = np.concatenate([lat[:cached], lat[cached + np.array(path)]])
            rope_c = np.concatenate([rope[:cached], rope[cached + np.array(path)]])
            chain = O.mla_absorbed(qn_[path], qr_[path], kvb, lat_c, rope_c, cached, O.chain_masks(n), 0.2, vh)
            np.testing.assert_allclose(tree[i], chain[n - 1], rtol=1e-6, atol=1e-6)


def _greedy_walk(lg, tok, parent):
    """The definition of greedy tree acceptance: from the root, emit the current node's
    argmax (first index of the maximum); move to the lowest-index child carrying it."""
    node, emit, path = 0, [], [0]
    while True:
        a = int(np.argmax(lg[node]))
        emit.append(a)
        kids = [c for c in range(len(parent)) if parent[c] == node and tok[c] == a]
        if not kids:
            return emit, path
        node = kids[0]
        path.append(node)


def test_tree_accept_is_the_greedy_walk_and_a_chain_on_a_chain():
    rng = np.random.default_rng(9)
    V = 7
    for T in (1, 5, 23, 64):
        for trial in range(20):
            parent = _random_tree(rng, T)
            tok = rng.integers(0, V, T).astype(np.int32)
            lg = rng.standard_normal((T, V), dtype=np.float32)
            # steer some nodes' argmax onto one of their children so paths get deep
            for c in range(1, T):
                if rng.random() < 0.6:
                    lg[parent[c], tok[c]] = 5.0 + rng.random()
            emit = np.zeros(T, np.int32)
            path = np.zeros(T, np.int32)
            n = O.orc().orc_accept_tree_greedy(emit, path, np.ascontiguousarray(lg), tok,
                                               np.asarray(parent, np.int32), T, V)
            want_emit, want_path = _greedy_walk(lg, tok, parent)
            assert emit[:n].tolist() == want_emit and path[:len(want_path)].tolist() == want_path
    # a chain-shaped tree accepts exactly as the chain rule does
    nd = 6
    d = rng.integers(0, V, nd).astype(np.int32)
    for m_want in range(nd + 1):
        lg = rng.standard_normal((nd + 1, V), dtype=np.float32)
        for i in range(nd + 1):
            lg[i, d[i] if i < m_want else ((d[i] + 1) % V if i < nd else 3)] = 10.0
        e1, e2 = np.zeros(nd + 1, np.int32), np.zeros(nd + 1, np.int32)
        arg, acc, path = np.zeros(nd + 1, np.int32), O.C.c_int(0), np.zeros(nd + 1, np.int32)
        n1 = O.orc().orc_accept_greedy(e1, O.C.byref(acc), arg, lg, d, nd, V)
        tok = np.concatenate([[0], d]).astype(np.int32)
        n2 = O.orc().orc_accept_tree_greedy(e2, path, lg, tok, np.arange(-1, nd, dtype=np.int32), nd + 1, V)
        assert n1 == n2 == m_want + 1 and e1[:n1].tolist() == e2[:n2].tolist()


def _mxfp4_decode(packed, scales, rows, cols):
    """Independent numpy decode of MXFP4: E2M1 magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}
    with sign bit 8, low nibble the even element, times 2^(S - 127) per 32 columns."""
    mag = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float64)
    p = packed.reshape(rows, cols // 2)
    nib = np.empty((rows, cols), np.uint8)
    nib[:, 0::2], nib[:, 1::2] = p & 0xF, p >> 4
    v = mag[nib & 7] * np.where(nib & 8, -1.0, 1.0)
    sc = np.exp2(scales.reshape(rows, cols // 32).astype(np.float64) - 127.0)
    return v * np.repeat(sc, 32, axis=1)


def test_swiglu_experts_against_an_independent_restatement():
    """The SwiGLU experts the benchmark configurations use (no reference implementation;
    the reference's experts are SiTU-GLU): the checker's expert stream equals a float64
    numpy restatement -- decode each expert, gate and up from w1 and w3, silu(gate) * up,
    down through w2, routed contributions weighted in top-k order, shared ones added."""
    rng = np.random.default_rng(12)
    L, I, n, ns, k, T = 64, 96, 6, 1, 2, 5
    bank, lay = O.make_bank(rng, n + ns, L, I, std=0.05, w13_std=0.3)
    z = rng.standard_normal((T, L), dtype=np.float32)
    W = rng.standard_normal((n, L), dtype=np.float32) * np.float32(0.05)
    idx, wt = O.router(z, W, np.zeros(n, np.float32), k)
    got = O.moe_routed(z, idx, wt, bank, lay, L, I, k, n, ns, 1)
    stride = int(lay[6])

    def expert(e, x):
        run = bank[e * stride:(e + 1) * stride]
        w1 = _mxfp4_decode(run[lay[0]:lay[0] + I * L // 2], run[lay[1]:lay[1] + I * L // 32], I, L)
        w2 = _mxfp4_decode(run[lay[2]:lay[2] + L * I // 2], run[lay[3]:lay[3] + L * I // 32], L, I)
        w3 = _mxfp4_decode(run[lay[4]:lay[4] + I * L // 2], run[lay[5]:lay[5] + I * L // 32], I, L)
        g, u = w1 @ x, w3 @ x
        return w2 @ (g / (1.0 + np.exp(-g)) * u)
    want = np.zeros((T, L))
    for t in range(T):
        x = z[t].astype(np.float64)
        for j in range(k):
            want[t] += float(wt[t, j]) * expert(int(idx[t, j]), x)
        for s_ in range(ns):
            want[t] += expert(n + s_, x)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-5


# ---------------------------------------------------------------------------- MoE --
def test_latent_moe_composition_vs_reference_k3_moe():
    """orc_moe_routed inside the LatentMoE of the reference's k3_moe
    (src/core/k3_ops.c:1862-1952), against k3_moe itself with MXFP4 experts."""
    p = GI.latent_moe_inputs()
    g = np.load(os.path.join(G, "ref_moe.npz"))
    x = p["x"]
    idx, wt = O.router(x, p["gate"], p["bias"], p["topk"])
    z = O.matmul_d(x, p["down"])
    acc = O.moe_routed(z, idx, wt, p["bank"], p["lay"], p["L"], p["I"], p["topk"],
                       p["n_experts"], 0, 0, latent_norm=p["latent_norm"])
    out = O.matmul_d(acc, p["up"])
    gu = np.concatenate([O.matmul_d(x, p["sh1"]), O.matmul_d(x, p["sh3"])], 1)
    h = np.zeros((x.shape[0], p["I"]), np.float32)
    for t in range(x.shape[0]):
        ht = np.zeros(p["I"], np.float32)
        O.orc().orc_situ_glu(ht, np.ascontiguousarray(gu[t]), p["I"], 4.0, 25.0)
        h[t] = ht
    out = out + O.matmul_d(h, p["sh2"])
    np.testing.assert_allclose(out, g["out"], rtol=1e-5, atol=1e-6)


# ------------------------------------------------------------- drafter / accept ---
def draft(seq, cap=8, nmax=4, nmin=3):
    seq = np.asarray(seq, np.int32)
    out = np.zeros(max(cap, 1), np.int32)
    nd = O.orc().orc_spec_draft(seq, len(seq), cap, nmax, nmin, out)
    return out[:nd].tolist()


def test_spec_draft_rules():
    # a repeated 4-gram whose two occurrences agree on what follows; the older history
    # ends where the newer match begins (m2 + n + i >= m1 stops the draft)
    s = [1, 2, 3, 4, 5, 6, 9, 1, 2, 3, 4, 5, 6, 9, 1, 2, 3, 4]
    assert draft(s) == [5, 6, 9]
    # the two histories disagree at once: no draft
    s = [7, 1, 2, 3, 4, 8, 0, 1, 2, 3, 4, 9, 0, 1, 2, 3, 4]
    assert draft(s) == []
    # only one earlier occurrence: draft its continuation up to the cap
    s = [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 1, 2, 3, 4]
    assert draft(s, cap=3) == [5, 6, 7]
    # no 4-gram match but a 3-gram one (n = 4 then 3)
    s = [0, 2, 3, 4, 5, 6, 9, 2, 3, 4]
    assert draft(s) == [5, 6, 9, 2, 3, 4]
    # the benchmark's rule n = 3 only
    assert draft([5, 1, 2, 3, 9, 1, 2, 3], nmax=3) == [9, 1, 2, 3]
    assert draft([1, 2]) == []


def test_accept_greedy_every_count():
    rng = np.random.default_rng(3)
    nd, V = 4, 50
    d = rng.integers(0, V, nd).astype(np.int32)
    for m_want in range(nd + 1):
        lg = rng.standard_normal((nd + 1, V), dtype=np.float32)
        for i in range(nd + 1):
            tgt = d[i] if i < m_want else (d[i] + 1) % V if i < nd else 7
            lg[i, tgt] = 10.0
        emit = np.zeros(nd + 1, np.int32)
        arg = np.zeros(nd + 1, np.int32)
        acc = O.C.c_int(0)
        n = O.orc().orc_accept_greedy(emit, O.C.byref(acc), arg, lg, d, nd, V)
        assert acc.value == m_want and n == m_want + 1
        assert emit[:m_want].tolist() == d[:m_want].tolist()
        assert emit[m_want] == arg[m_want]


def test_reference_library_matches_goldens_when_built():
    lib = O.ref()
    if lib is None:
        pytest.skip("oracle/_ref/libk3ref.so not built (no reference tree)")
    g = np.load(os.path.join(G, "ref_router.npz"))
    case = GI.ROUTER_CASES[1]
    x, W, b = GI.router_inputs(case)
    idx, w = O.router(x, W, b, case["topk"], lib=lib)
    np.testing.assert_array_equal(idx, g[case["name"] + "/idx"])


def test_reference_isa_builds_agree_bit_for_bit():
    """The x86-64-v4 build of the reference's numeric core (its AVX-512 paths), which the
    timed CPU baselines use on hosts that have them, gives the same bits as the x86-64-v3
    build that the parity checks use, as the reference's floating-point contract promises
    for its ISA paths (src/core/k3_ops.c:8-25): the router, the MXFP4 matmul, the batched
    bf16 matmul and the KDA step."""
    v3, v4 = O.ref(), O.ref_v4_if_runnable()
    if v3 is None or v4 is None:
        pytest.skip("needs both reference builds and an x86-64-v4 host")
    for case in GI.ROUTER_CASES:
        x, W, b = GI.router_inputs(case)
        i3, w3 = O.router(x, W, b, case["topk"], lib=v3)
        i4, w4 = O.router(x, W, b, case["topk"], lib=v4)
        np.testing.assert_array_equal(i3, i4)
        np.testing.assert_array_equal(w3.view(np.uint32), w4.view(np.uint32))
    for case in GI.MXFP4_CASES:
        packed, scales, x = GI.mxfp4_inputs(case)
        rows, n_in = case["rows"], case["in"]
        y = [np.zeros(rows, np.float32) for _ in range(2)]
        for lib, out in zip((v3, v4), y):
            lib.k3_matmul_mxfp4(out, x, packed, scales, n_in, rows, 32)
        np.testing.assert_array_equal(y[0].view(np.uint32), y[1].view(np.uint32))
    rng = np.random.default_rng(41)
    T, n_in, n_out = 9, 1024, 96
    X = rng.standard_normal((T, n_in)).astype(np.float32)
    Wb = ((rng.standard_normal((n_out, n_in)).astype(np.float32) * np.float32(0.02)).view(np.uint32) >> 16) \
        .astype(np.uint16)
    Y = [np.zeros((T, n_out), np.float32) for _ in range(2)]
    for lib, out in zip((v3, v4), Y):
        lib.k3_matmul_bf16_batch_ld(out, n_out, X, n_in, Wb.ctypes.data, n_in, n_out, T)
    np.testing.assert_array_equal(Y[0].view(np.uint32), Y[1].view(np.uint32))
    D = 128
    S0 = (rng.standard_normal((D, D)) * 0.1).astype(np.float32)
    q, k, v = (rng.standard_normal(D).astype(np.float32) for _ in range(3))
    al = rng.uniform(0.9, 0.999, D).astype(np.float32)
    outs = []
    for lib in (v3, v4):
        S, o = S0.copy(), np.zeros(D, np.float32)
        for _ in range(4):
            lib.k3_kda_step(S, o, q, k, v, al, 0.4, D, D)
        outs.append((S, o))
    np.testing.assert_array_equal(outs[0][0].view(np.uint32), outs[1][0].view(np.uint32))
    np.testing.assert_array_equal(outs[0][1].view(np.uint32), outs[1][1].view(np.uint32))
