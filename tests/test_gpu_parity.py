"""GPU parity: every kernel through the C ABI against the CPU oracle and the reference's
golden vectors. Tolerances are written per test; integer work (routing indices, drafts,
accepted ids, cache data movement) and the KDA recurrence are bit-exact."""
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests import k3lib
from tests.golden import inputs as GI

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(__file__), "golden")

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def k3():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return k3lib.load()


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def assert_clean(k3):
    assert k3.device_status(0) == 0, "a kernel flagged an out-of-range index"


# ------------------------------------------------------------------------- router --
@pytest.mark.parametrize("case", GI.ROUTER_CASES, ids=lambda c: c["name"])
def test_router_indices_bitexact_vs_reference(k3, case):
    g = np.load(os.path.join(G, "ref_router.npz"))
    x, W, b = GI.router_inputs(case)
    idx, w = k3.router(dev(x), dev(W), dev(b), case["topk"])
    np.testing.assert_array_equal(host(idx), g[case["name"] + "/idx"])
    # weights: the reference's glibc expf differs from a correctly rounded exp in ~6e-4
    # of inputs by one ulp, which reaches the weight through the renormaliser
    np.testing.assert_allclose(host(w), g[case["name"] + "/w"], rtol=1e-6, atol=0)
    assert_clean(k3)


def test_router_fixture(k3):
    ops = np.load(os.path.join(G, "ops_fixtures.npz"))
    x, W, b = ops["router/in"], ops["router/gate_weight"], ops["router/bias"]
    idx, w = k3.router(dev(x), dev(W), dev(b), int(ops["router/top_k"]))
    np.testing.assert_array_equal(host(idx), ops["router/topk_idx"].astype(np.int32))
    np.testing.assert_allclose(host(w), ops["router/topk_weight"], atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("T", [5, 72, 320, 1024])   # the one-wave kernel (5, 72) and the tiled one
def test_router_c2_batches_vs_oracle(k3, T):
    rng = np.random.default_rng(100 + T)
    x = GI.bf16_round(rng.standard_normal((T, 7168), dtype=np.float32))
    W = rng.standard_normal((384, 7168), dtype=np.float32) * np.float32(0.02)
    b = rng.standard_normal(384, dtype=np.float32) * np.float32(0.01)
    idx, w = k3.router(dev(x), dev(W), dev(b), 8)
    ri, rw = O.router(x, W, b, 8)
    np.testing.assert_array_equal(host(idx), ri)
    np.testing.assert_allclose(host(w), rw, rtol=1e-6, atol=0)


# -------------------------------------------------------------------------- MXFP4 --
def test_mxfp4_dequant_released_bytes_exact(k3):
    d = np.load(os.path.join(G, "mxfp4_fixture.npz"))
    out = k3.mxfp4_dequant(dev(d["packed"]), dev(d["scales"]))
    np.testing.assert_array_equal(host(out).view(np.uint32), d["expected"].view(np.uint32))


def test_mxfp4_dequant_every_code_and_scale(k3):
    # all 256 byte values in every one of the 256 scale bytes, incl. 0 (2^-127) and 255
    packed = np.tile(np.arange(256, dtype=np.uint8), (256, 1)).reshape(256, 256)
    scales = np.repeat(np.arange(256, dtype=np.uint8), 16).reshape(256, 16)
    out = k3.mxfp4_dequant(dev(packed), dev(scales))
    want = np.zeros((256, 512), np.float32)
    O.orc().orc_mxfp4_dequant(want, packed, scales, 256, 512)
    np.testing.assert_array_equal(host(out).view(np.uint32), want.view(np.uint32))


# ---------------------------------------------------------------------------- MoE --
def moe_case(seed, L, I, n_routed, n_shared, topk, T, act, std=0.02, w13_std=None):
    rng = np.random.default_rng(seed)
    bank, lay = O.make_bank(rng, n_routed + n_shared, L, I, std=std, w13_std=w13_std)
    x = GI.bf16_round(rng.standard_normal((T, L), dtype=np.float32))
    W = rng.standard_normal((n_routed, L), dtype=np.float32) * np.float32(0.02)
    bias = rng.standard_normal(n_routed, dtype=np.float32) * np.float32(0.01)
    return bank, lay, x, W, bias


@pytest.mark.parametrize("act", [0, 1], ids=["situ", "swiglu"])
def test_moe_layer_tiny_config_vs_oracle(k3, act):
    """Benchmark config 1 MoE shape: d 512, 16 experts top-2, 1 shared, FFN 256."""
    L, I, n, ns, k, T = 512, 256, 16, 1, 2, 5
    bank, lay, x, W, bias = moe_case(7, L, I, n, ns, k, T, act, std=0.05, w13_std=0.3)
    kb = k3.ExpertBank(dev(bank), n + ns, L, I)
    out, idx, wt = k3.moe_layer(dev(x), dev(W), dev(bias), kb, k, n, ns, act)
    ri, rw = O.router(x, W, bias, k)
    np.testing.assert_array_equal(host(idx), ri)
    ref = O.moe_routed(x, ri, rw, bank, lay, L, I, k, n, ns, act)
    got = host(out)
    assert rel_l2(got, ref) < 1e-5, rel_l2(got, ref)
    np.testing.assert_allclose(got, ref, atol=1e-5 * np.abs(ref).max(), rtol=0)
    assert_clean(k3)


def test_moe_latent_norm_and_dropped_slot(k3):
    L, I, n, ns, k, T = 256, 128, 12, 0, 3, 6
    bank, lay, x, W, bias = moe_case(8, L, I, n, ns, k, T, 0, std=0.05, w13_std=0.3)
    ri, rw = O.router(x, W, bias, k)
    ri[2, 1] = -1                     # a dropped expert, as after a failed load
    ln = (1.0 + 0.1 * np.random.default_rng(1).standard_normal(L)).astype(np.float32)
    kb = k3.ExpertBank(dev(bank), n, L, I)
    out = k3.moe_experts(dev(x), dev(ri), dev(rw), kb, k, n, ns, 0, latent_norm=dev(ln))
    ref = O.moe_routed(x, ri, rw, bank, lay, L, I, k, n, ns, 0, latent_norm=ln)
    assert rel_l2(host(out), ref) < 1e-5


def test_moe_c2_width_vs_oracle(k3):
    """Benchmark config 2 widths (d 7168, FFN 2048, SwiGLU) on 24 experts, 5 tokens."""
    L, I, n, ns, k, T = 7168, 2048, 24, 1, 8, 5
    bank, lay, x, W, bias = moe_case(9, L, I, n, ns, k, T, 1)
    kb = k3.ExpertBank(dev(bank), n + ns, L, I)
    out, idx, wt = k3.moe_layer(dev(x), dev(W), dev(bias), kb, k, n, ns, 1)
    ri, rw = O.router(x, W, bias, k)
    np.testing.assert_array_equal(host(idx), ri)
    ref = O.moe_routed(x, ri, rw, bank, lay, L, I, k, n, ns, 1)
    assert rel_l2(host(out), ref) < 1e-5, rel_l2(host(out), ref)


@pytest.mark.parametrize("which", [0, 1], ids=["tensor", "cudacore"])
def test_moe_expert_kernels_fp32_inputs_many_tokens(k3, which):
    """Both expert streams on tensor-core-eligible shapes (L, I multiples of 512) with
    fp32 (not bf16) inputs, so the lo half of the f16 split is live, and up to 48 tokens
    per expert: several 8-token chunks and a second pass over the weights."""
    L, I, n, ns, k, T = 1024, 512, 4, 1, 3, 64
    rng = np.random.default_rng(21)
    bank, lay = O.make_bank(rng, n + ns, L, I, std=0.05, w13_std=0.1)
    x = rng.standard_normal((T, L), dtype=np.float32)
    W = rng.standard_normal((n, L), dtype=np.float32) * np.float32(0.02)
    bias = np.zeros(n, np.float32)
    kb = k3.ExpertBank(dev(bank), n + ns, L, I)
    k3.check(k3.lib.k3gpu_moe_select_kernels(which), "select")
    try:
        out, idx, wt = k3.moe_layer(dev(x), dev(W), dev(bias), kb, k, n, ns, 1)
    finally:
        k3.check(k3.lib.k3gpu_moe_select_kernels(0), "select")
    ri, rw = O.router(x, W, bias, k)
    np.testing.assert_array_equal(host(idx), ri)
    ref = O.moe_routed(x, ri, rw, bank, lay, L, I, k, n, ns, 1)
    assert rel_l2(host(out), ref) < 1e-5, rel_l2(host(out), ref)
    assert_clean(k3)


@pytest.mark.parametrize("shape", [2, 3], ids=["dense32", "sparse8"])
@pytest.mark.parametrize("fp32_inputs", [False, True], ids=["bf16in", "fp32in"])
def test_moe_tcgen05_pass_shapes_many_tokens(k3, shape, fp32_inputs):
    """The tcgen05 expert kernels forced into each pass shape on a certified bank with many
    tokens per expert: 8 routed experts top-3 over 100 tokens (37.5 an expert on average,
    so the dense shape's 32-token pass needs a second pass on some and the sparse shape
    five), with and without live lo halves, and the automatic choice beside them."""
    L, I, n, ns, k, T = 1024, 512, 8, 1, 3, 100
    rng = np.random.default_rng(61 + shape)
    bank, lay = O.make_bank(rng, n + ns, L, I, std=0.05, w13_std=0.1)
    x = rng.standard_normal((T, L), dtype=np.float32)
    if not fp32_inputs:
        x = GI.bf16_round(x)
    W = rng.standard_normal((n, L), dtype=np.float32) * np.float32(0.02)
    bias = rng.standard_normal(n, dtype=np.float32) * np.float32(0.01)
    kb = k3.ExpertBank(dev(bank), n + ns, L, I)
    assert kb.scan() == 0
    ri, rw = O.router(x, W, bias, k)
    ref = O.moe_routed(x, ri, rw, bank, lay, L, I, k, n, ns, 1)
    for which in (shape, 0):
        k3.check(k3.lib.k3gpu_moe_select_kernels(which), "select")
        try:
            out, idx, wt = k3.moe_layer(dev(x), dev(W), dev(bias), kb, k, n, ns, 1)
        finally:
            k3.check(k3.lib.k3gpu_moe_select_kernels(0), "select")
        np.testing.assert_array_equal(host(idx), ri)
        assert rel_l2(host(out), ref) < 1e-5, (which, rel_l2(host(out), ref))
    assert_clean(k3)


@pytest.mark.parametrize("fp32_inputs", [False, True], ids=["bf16in", "fp32in"])
def test_moe_tcgen05_path_vs_oracle(k3, fp32_inputs):
    """The tcgen05 expert kernels (bank certified by k3gpu_bank_scan): benchmark config-2
    widths on 24 experts, then a 1024/512 case with up to 48 tokens per expert (three
    16-token passes) and, for fp32 inputs, the lo halves of the f16 split."""
    for (L, I, n, ns, k, T, seed) in ((7168, 2048, 24, 1, 8, 6, 31), (1024, 512, 4, 1, 3, 64, 32)):
        rng = np.random.default_rng(seed)
        bank, lay = O.make_bank(rng, n + ns, L, I, std=0.05, w13_std=0.1)
        x = rng.standard_normal((T, L), dtype=np.float32)
        if not fp32_inputs:
            x = GI.bf16_round(x)
        W = rng.standard_normal((n, L), dtype=np.float32) * np.float32(0.02)
        bias = rng.standard_normal(n, dtype=np.float32) * np.float32(0.01)
        kb = k3.ExpertBank(dev(bank), n + ns, L, I)
        assert kb.scan() == 0                       # every expert certified
        out, idx, wt = k3.moe_layer(dev(x), dev(W), dev(bias), kb, k, n, ns, 1)
        ri, rw = O.router(x, W, bias, k)
        np.testing.assert_array_equal(host(idx), ri)
        ref = O.moe_routed(x, ri, rw, bank, lay, L, I, k, n, ns, 1)
        assert rel_l2(host(out), ref) < 1e-5, (L, rel_l2(host(out), ref))
    assert_clean(k3)


def test_moe_mixed_bank_tcgen05_and_sync_paths(k3):
    """One expert carries E8M0 bytes outside the f16-exact range (141), so the scan leaves
    it to the mma.sync kernels while the rest run on tcgen05; the sum must not care."""
    L, I, n, ns, k, T = 1024, 512, 6, 1, 2, 24
    rng = np.random.default_rng(33)
    bank, lay = O.make_bank(rng, n + ns, L, I, std=0.05, w13_std=0.1)
    stride = int(lay[6])
    bank[2 * stride + int(lay[1]) + 5] = 141          # expert 2, one w1 scale byte
    x = GI.bf16_round(rng.standard_normal((T, L), dtype=np.float32))
    W = rng.standard_normal((n, L), dtype=np.float32) * np.float32(0.02)
    bias = np.zeros(n, np.float32)
    kb = k3.ExpertBank(dev(bank), n + ns, L, I)
    assert kb.scan() == 1
    assert host(kb.safe).tolist() == [1, 1, 0, 1, 1, 1, 1]
    out, idx, wt = k3.moe_layer(dev(x), dev(W), dev(bias), kb, k, n, ns, 1)
    ri, rw = O.router(x, W, bias, k)
    ref = O.moe_routed(x, ri, rw, bank, lay, L, I, k, n, ns, 1)
    assert rel_l2(host(out), ref) < 1e-5, rel_l2(host(out), ref)
    assert_clean(k3)


def test_moe_c2_width_cudacore_path(k3):
    L, I, n, ns, k, T = 7168, 2048, 12, 1, 8, 3
    bank, lay, x, W, bias = moe_case(19, L, I, n, ns, k, T, 1)
    kb = k3.ExpertBank(dev(bank), n + ns, L, I)
    k3.check(k3.lib.k3gpu_moe_select_kernels(1), "select")
    try:
        out, idx, wt = k3.moe_layer(dev(x), dev(W), dev(bias), kb, k, n, ns, 1)
    finally:
        k3.check(k3.lib.k3gpu_moe_select_kernels(0), "select")
    ri, rw = O.router(x, W, bias, k)
    ref = O.moe_routed(x, ri, rw, bank, lay, L, I, k, n, ns, 1)
    assert rel_l2(host(out), ref) < 1e-5


def test_moe_many_tokens_per_expert(k3):
    """Odd and even token counts per expert (the 2-token and 1-token paths)."""
    L, I, n, ns, k, T = 256, 64, 4, 1, 3, 33
    bank, lay, x, W, bias = moe_case(10, L, I, n, ns, k, T, 0, std=0.05, w13_std=0.3)
    kb = k3.ExpertBank(dev(bank), n + ns, L, I)
    out, idx, wt = k3.moe_layer(dev(x), dev(W), dev(bias), kb, k, n, ns, 0)
    ri, rw = O.router(x, W, bias, k)
    ref = O.moe_routed(x, ri, rw, bank, lay, L, I, k, n, ns, 0)
    assert rel_l2(host(out), ref) < 1e-5


# ---------------------------------------------------------------------------- KDA --
@pytest.mark.parametrize("case", GI.KDA_CASES, ids=lambda c: c["name"])
def test_kda_verify_commit_bitexact_vs_reference(k3, case):
    g = np.load(os.path.join(G, "ref_kda.npz"))
    st0, q, k, v, al, be = GI.kda_inputs(case)
    T, H, D = q.shape
    qs = np.float32(1.0) / np.sqrt(np.float32(D))
    S = dev(st0[None])
    o = k3.kda_verify(S, dev(q[None]), dev(k[None]), dev(v[None]), dev(al[None]), dev(be[None]), qs)
    np.testing.assert_array_equal(host(o)[0].view(np.uint32), g[case["name"] + "/o"].view(np.uint32))
    np.testing.assert_array_equal(host(S)[0], st0)          # verify never writes the state
    for n in case["commits"]:
        S = dev(st0[None])
        k3.kda_commit(S, dev(k[None]), dev(v[None]), dev(al[None]), dev(be[None]),
                      dev(np.array([n], np.int32)))
        np.testing.assert_array_equal(host(S)[0].view(np.uint32),
                                      g[case["name"] + f"/state_n{n}"].view(np.uint32))
    assert_clean(k3)


def test_kda_batched_rollback_c3_shape(k3):
    """Benchmark config 3: 32 heads x 128, chunk 1+k = 9, four sequences, rollback
    lengths drawn in [0, k]; each sequence bit-identical to the oracle."""
    B, T, H, D = 4, 9, 32, 128
    rng = np.random.default_rng(77)
    case = dict(seed=78, T=T, H=H, D=D)
    ins = [GI.kda_inputs(dict(case, seed=78 + b)) for b in range(B)]
    st0 = np.stack([i[0] for i in ins])
    q, k, v, al, be = (np.stack([i[j] for i in ins]) for j in range(1, 6))
    qs = np.float32(1.0) / np.sqrt(np.float32(D))
    o = k3.kda_verify(dev(st0), dev(q), dev(k), dev(v), dev(al), dev(be), qs)
    n = rng.integers(0, T + 1, B).astype(np.int32)
    S = dev(st0)
    k3.kda_commit(S, dev(k), dev(v), dev(al), dev(be), dev(n))
    og, Sg = host(o), host(S)
    for b in range(B):
        ref_o = O.kda_verify(st0[b], q[b], k[b], v[b], al[b], be[b], qs)
        np.testing.assert_array_equal(og[b].view(np.uint32), ref_o.view(np.uint32))
        ref_s = O.kda_commit(st0[b], k[b], v[b], al[b], be[b], int(n[b]))
        np.testing.assert_array_equal(Sg[b].view(np.uint32), ref_s.view(np.uint32))


def test_kda_prologue_conv_commit_norm_gate_vs_oracle(k3):
    B, T, H, D, K = 2, 5, 4, 64, 4
    P = H * D
    rng = np.random.default_rng(5)
    q, k, v, z = (rng.standard_normal((B, T, P), dtype=np.float32) for _ in range(4))
    b = rng.standard_normal((B, T, H), dtype=np.float32)
    qc, kc, vc = (rng.standard_normal((P, K), dtype=np.float32) * np.float32(0.4) for _ in range(3))
    hist = rng.standard_normal((B, 3, P, K - 1), dtype=np.float32)
    A = np.linspace(-0.4, 1.2, H).astype(np.float32)
    dt = rng.standard_normal(P, dtype=np.float32) * np.float32(0.5)
    tq, tk, tv = dev(q), dev(k), dev(v)
    al, be, pre = k3.kda_prologue(tq, tk, tv, dev(z), dev(b), dev(qc), dev(kc), dev(vc), dev(hist),
                                  dev(A), dev(dt), H, D, K, -5.0)
    for bb in range(B):
        rq, rk, rv = q[bb].copy(), k[bb].copy(), v[bb].copy()
        ral, rbe = np.zeros((T, P), np.float32), np.zeros((T, H), np.float32)
        h = hist[bb].copy()
        O.orc().orc_kda_prologue(rq, rk, rv, ral, rbe, np.ascontiguousarray(z[bb]),
                                 np.ascontiguousarray(b[bb]), qc, kc, vc, h.ctypes.data, A, dt, T,
                                 H, D, K, -5.0)
        for got, want in ((tq, rq), (tk, rk), (tv, rv), (al, ral), (be, rbe)):
            np.testing.assert_allclose(host(got)[bb], want, rtol=2e-6, atol=1e-6)
        np.testing.assert_array_equal(host(pre)[bb][:, 0], q[bb])
    # conv-history commit: pure data movement, exact
    n = np.array([2, 5], np.int32)
    th = dev(hist)
    k3.kda_commit_conv(th, pre, dev(n), H, D, K)
    for bb in range(B):
        h = hist[bb].copy()
        prer = np.ascontiguousarray(np.stack([q[bb], k[bb], v[bb]], 1))
        O.orc().orc_kda_commit_conv(h, prer, int(n[bb]), P, K)
        np.testing.assert_array_equal(host(th)[bb], h)
    # head-wise RMSNorm then the sigmoid gate
    o = rng.standard_normal((B * T, H, D), dtype=np.float32)
    gate = rng.standard_normal((B * T, P), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    to = dev(o)
    k3.kda_norm_gate(to, dev(gate), dev(w), H, D, 1e-5)
    ro = o.copy()
    O.orc().orc_kda_norm_gate(ro, gate, w, B * T, H, D, 1e-5)
    np.testing.assert_allclose(host(to), ro, rtol=2e-6, atol=1e-7)


# ---------------------------------------------------------------------------- MLA --
def mla_case(seed, B, T, H, qn, qr, vh, kvl, cached):
    rng = np.random.default_rng(seed)
    qnope = rng.standard_normal((B, T, H, qn), dtype=np.float32)
    qrope = rng.standard_normal((B, T, H, qr), dtype=np.float32)
    kvb = rng.standard_normal((H * (qn + vh), kvl), dtype=np.float32) * np.float32(0.05)
    cap = max(cached) + T + 3
    lat = GI.bf16_round(rng.standard_normal((B, cap, kvl), dtype=np.float32))
    rope = GI.bf16_round(rng.standard_normal((B, cap, qr), dtype=np.float32))
    return qnope, qrope, kvb, lat, rope, cap


def to_bf16_bits(a):
    return np.ascontiguousarray((np.ascontiguousarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16))


@pytest.mark.parametrize("tree", [False, True], ids=["chain", "tree"])
def test_mla_absorbed_vs_oracle(k3, tree):
    B, T, H, qn, qr, vh, kvl = 2, 9, 8, 32, 16, 32, 128
    cached = [700, 37]
    qnope, qrope, kvb, lat, rope, cap = mla_case(3, B, T, H, qn, qr, vh, kvl, cached)
    if tree:
        parent = [-1, 0, 0, 1, 1, 2, 3, 5, 5]
        masks = O.tree_masks(parent)
    else:
        masks = O.chain_masks(T)
    scale = 1.0 / np.sqrt(qn + qr)
    out = k3.mla_absorbed(dev(qnope), dev(qrope), dev(kvb), dev(to_bf16_bits(lat).view(np.int16)),
                          dev(to_bf16_bits(rope).view(np.int16)), dev(np.array(cached, np.int32)),
                          dev(masks.view(np.int64)), vh, cap, scale)
    got = host(out)
    for b in range(B):
        ref = O.mla_absorbed(qnope[b], qrope[b], kvb, lat[b], rope[b], cached[b], masks, scale, vh)
        assert rel_l2(got[b], ref) < 1e-4, rel_l2(got[b], ref)
    assert_clean(k3)


# The tcgen05 path (kv_lora 128/256/512, qk_rope 0 or 64): ragged 128-row query tiles,
# several context slices, a partial last tile, and NaN garbage in the cache rows past
# cached + T (the kernel zeroes them before they enter the value product). The bar is
# relative L2 1e-4 (5e-4 for the wide-score case, whose scores spread over +-40 and whose
# running max is rescaled along the context).
@pytest.mark.parametrize("kvl,qr,B,T,H,cached,tree,qscale", [
    (512, 64, 2, 9, 16, [700, 37], True, 1.0),     # K3 widths, 2 query tiles (144 rows)
    (128, 0, 1, 5, 8, [3000], False, 1.0),         # no rope, many slices
    (256, 64, 1, 4, 32, [5000], True, 4.0),        # wide scores: lazy-max rescale
    (512, 64, 1, 64, 4, [130], False, 1.0),        # 64 chain nodes, cache shorter than a tile pair
], ids=["k3_2seq", "norope_slices", "rescale", "t64"])
def test_mla_absorbed_tensor_core(k3, kvl, qr, B, T, H, cached, tree, qscale):
    qn, vh = 32, 48
    qnope, qrope, kvb, lat, rope, cap = mla_case(17 + kvl + T, B, T, H, qn, qr, vh, kvl, cached)
    qnope *= np.float32(qscale)
    for b in range(B):                      # unspecified rows past the new ones
        lat[b, cached[b] + T:] = np.nan
        rope[b, cached[b] + T:] = np.nan
    if tree:
        parent = [-1] + [(i - 1) // 2 for i in range(1, T)]
        masks = O.tree_masks(parent)
    else:
        masks = O.chain_masks(T)
    scale = 1.0 / np.sqrt(qn + qr)
    # qk_rope = 0: empty rope tensors (NULL pointers at the C ABI)
    out = k3.mla_absorbed(dev(qnope), dev(qrope), dev(kvb), dev(to_bf16_bits(lat).view(np.int16)),
                          dev(to_bf16_bits(rope).view(np.int16)), dev(np.array(cached, np.int32)),
                          dev(masks.view(np.int64)), vh, cap, scale)
    got = host(out)
    tol = 5e-4 if qscale > 1 else 1e-4
    for b in range(B):
        ref = O.mla_absorbed(qnope[b], qrope[b], kvb, lat[b], rope[b], cached[b], masks, scale, vh)
        assert np.isfinite(got[b]).all()
        assert rel_l2(got[b], ref) < tol, rel_l2(got[b], ref)
    assert_clean(k3)


# Dozens of context slices to merge, output rows in two 128-row tiles (v_head 160) and a
# q_nope width that leaves a partial 32-wide chunk (40). qk_rope 16 runs the CUDA-core
# attention (512 positions a slice: 40 slices), qk_rope 0 with kv_lora 128 the tcgen05 one
# (47 slices).
@pytest.mark.parametrize("qr,cached", [(16, 20000), (0, 6000)], ids=["cuda_core_40", "tcgen05_47"])
def test_mla_absorbed_many_slices(k3, qr, cached):
    B, T, H, qn, vh, kvl = 1, 3, 4, 40, 160, 128
    qnope, qrope, kvb, lat, rope, cap = mla_case(29 + qr, B, T, H, qn, qr, vh, kvl, [cached])
    masks = O.chain_masks(T)
    scale = 1.0 / np.sqrt(qn + qr)
    out = k3.mla_absorbed(dev(qnope), dev(qrope), dev(kvb), dev(to_bf16_bits(lat).view(np.int16)),
                          dev(to_bf16_bits(rope).view(np.int16)), dev(np.array([cached], np.int32)),
                          dev(masks.view(np.int64)), vh, cap, scale)
    got = host(out)
    ref = O.mla_absorbed(qnope[0], qrope[0], kvb, lat[0], rope[0], cached, masks, scale, vh)
    assert rel_l2(got[0], ref) < 1e-4, rel_l2(got[0], ref)
    assert_clean(k3)


# ------------------------------------------------------------------------- accept --
def test_accept_greedy_every_acceptance_count(k3):
    B, nd, V = 6, 5, 1000
    rng = np.random.default_rng(11)
    d = rng.integers(0, V, (B, nd)).astype(np.int32)
    lg = rng.standard_normal((B, nd + 1, V), dtype=np.float32)
    for b in range(B):      # sequence b accepts exactly min(b, nd) drafts
        for i in range(nd + 1):
            if i < min(b, nd):
                lg[b, i, d[b, i]] = 9.0
            elif i < nd:
                lg[b, i, (d[b, i] + 1) % V] = 9.0
    lg[0, 0, 3] = lg[0, 0].max()          # an exact tie: the first index must win
    emit, n_emit, arg = k3.accept_greedy(dev(lg), dev(d))
    emit, n_emit, arg = host(emit), host(n_emit), host(arg)
    for b in range(B):
        e = np.zeros(nd + 1, np.int32)
        a = np.zeros(nd + 1, np.int32)
        m = O.C.c_int(0)
        n = O.orc().orc_accept_greedy(e, O.C.byref(m), a, np.ascontiguousarray(lg[b]),
                                      np.ascontiguousarray(d[b]), nd, V)
        assert n_emit[b] == n == min(b, nd) + 1
        np.testing.assert_array_equal(emit[b, :n], e[:n])
        np.testing.assert_array_equal(arg[b], a)


@pytest.mark.parametrize("V", [163840, 1001, 5], ids=["c4_vocab", "ragged", "tiny"])
def test_argmax_ties_nans_and_chunk_edges(k3, V):
    """The row is scanned by several CTAs in chunks: ties that straddle chunk edges, NaN at
    index 0 (the sequential scan keeps 0), NaNs elsewhere, an all-NaN row, and vocab sizes
    with empty chunks or no 16-byte path must all give the reference's argmax_."""
    rows = 7
    rng = np.random.default_rng(V)
    lg = rng.standard_normal((rows, V), dtype=np.float32)
    per = -(-V // 8)                       # chunk width of the 8-CTA split (elements)
    top = np.float32(50.0)
    lg[0, [V - 1, min(per, V - 1), 0]] = top            # tie: index 0 must win
    if V > 2:
        lg[1, [V - 2, V - 1]] = top                     # tie inside the last chunk
    lg[2, 0] = np.nan                                   # NaN first: index 0
    lg[3, 1::2] = np.nan                                # scattered NaNs
    lg[4, :] = np.nan                                   # all NaN: index 0
    lg[5, -1] = top                                     # maximum at the very end
    lg[6, :] = top                                      # all equal: index 0
    emit, n_emit, arg = k3.accept_greedy(dev(lg.reshape(1, rows, V)), dev(np.zeros((1, rows - 1), np.int32)))
    got = host(arg).reshape(-1)
    want = [O.orc().orc_argmax(np.ascontiguousarray(lg[r]), V) for r in range(rows)]
    np.testing.assert_array_equal(got, want)


def test_accept_tree_greedy_vs_oracle(k3):
    # 64-node tree, branching 4, depth 3 (+ root): benchmark config 4's draft tree shape
    parent = [-1]
    level = [0]
    while len(parent) < 64:
        nxt = []
        for p in level:
            for _ in range(4):
                if len(parent) < 64:
                    parent.append(p)
                    nxt.append(len(parent) - 1)
        level = nxt
    T, V, B = len(parent), 4096, 3
    rng = np.random.default_rng(12)
    lg = rng.standard_normal((B, T, V), dtype=np.float32)
    tok = rng.integers(0, V, (B, T)).astype(np.int32)
    for b in range(B):     # make a path of depth b+1 acceptable
        c = 0
        for _ in range(b + 1):
            kids = [i for i in range(T) if parent[i] == c]
            if not kids:
                break
            ch = kids[b % len(kids)]
            lg[b, c, tok[b, ch]] = 20.0
            c = ch
    emit, n_emit, path, arg = k3.accept_tree_greedy(dev(lg), dev(tok), dev(np.array(parent, np.int32)))
    emit, n_emit, path = host(emit), host(n_emit), host(path)
    for b in range(B):
        e = np.zeros(T, np.int32)
        pth = np.zeros(T, np.int32)
        n = O.orc().orc_accept_tree_greedy(e, pth, np.ascontiguousarray(lg[b]),
                                           np.ascontiguousarray(tok[b]), np.array(parent, np.int32), T, V)
        assert n_emit[b] == n
        np.testing.assert_array_equal(emit[b, :n], e[:n])
        np.testing.assert_array_equal(path[b, :n], pth[:n])


def test_accept_sample_matches_oracle_and_rejection_rule(k3):
    B, nd, V = 64, 4, 512
    rng = np.random.default_rng(13)
    lg = (rng.standard_normal((B, nd + 1, V), dtype=np.float32) * 2).astype(np.float32)
    d = np.argmax(lg[:, :nd], axis=2).astype(np.int32)      # likely drafts
    d[::3, 1] = 7                                            # and some unlikely ones
    emit, n_emit = k3.accept_sample(dev(lg), dev(d), 0.7, seed=1234, offset=5)
    emit, n_emit = host(emit), host(n_emit)
    for b in range(B):
        e = np.zeros(nd + 1, np.int32)
        n = O.orc().orc_accept_sample(e, np.ascontiguousarray(lg[b]), np.ascontiguousarray(d[b]),
                                      nd, V, 0.7, 1234, 5, b)
        assert n_emit[b] == n
        np.testing.assert_array_equal(emit[b, :n], e[:n])
        assert np.all(emit[b, : n - 1] == d[b, : n - 1])    # accepted prefix = drafts
