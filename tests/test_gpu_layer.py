"""The KDA layer and the KDA + MoE decoder layer (k3gpu_kda_layer_verify,
k3gpu_decoder_layer_kda_verify) against an oracle composition.

The oracle side composes the pinned restatements in the reference's order
(k3_kda_layer_log, src/core/k3_ops.c:2231-2385; k3_decoder_layer_core, :2485-2592):
projections as double matmuls of the same bf16 weights (k3_matmul_bf16_batch's contract),
orc_kda_prologue, orc_kda_verify, orc_kda_norm_gate, orc_attn_res, orc_rmsnorm, the router
and the MoE. The device projections agree with double sums to ~1e-5 relative, so the bar
is rel-L2 <= 1e-4 on layer outputs and log operands (the sweep's logits tolerance is
1e-3, the KDA state's 1e-4); the routing is checked for identity.
"""
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))
from k3lib import load  # noqa: E402
from oracle import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu

E, H, D, K = 512, 4, 64, 4
P = H * D
LB, EPS = -5.0, 1e-5


@pytest.fixture(scope="module")
def k3():
    return load()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rel(got, ref):
    return float(np.linalg.norm(np.asarray(got, np.float64) - ref) / max(np.linalg.norm(ref), 1e-30))


def bf16_bits(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def kda_weights(rng):
    w = {}
    for n, shape, sd in (("q", (P, E), 0.05), ("k", (P, E), 0.05), ("v", (P, E), 0.05), ("b", (H, E), 0.05),
                         ("f_a", (D, E), 0.05), ("f_b", (P, D), 0.1), ("g", (P, E), 0.05), ("o", (E, P), 0.05)):
        w[n] = bf16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(sd))
    for n in ("q_conv", "k_conv", "v_conv"):
        w[n] = rng.standard_normal((P, K), dtype=np.float32) * np.float32(0.4)
    w["A_log"] = np.linspace(-0.4, 1.2, H).astype(np.float32)
    w["dt_bias"] = rng.standard_normal(P, dtype=np.float32) * np.float32(0.5)
    w["o_norm"] = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    return w


def to_dev(w):
    return {n: (dev(a.view(np.int16)) if a.dtype == np.uint16 else dev(a)) for n, a in w.items()}


def mmd(x, wbits):
    return O.matmul_d(x, O.bf16_bits_to_f32(wbits))


def oracle_kda_layer(x, w, state, hist):
    """One sequence: x [T][E] -> out [T][E], log (k, v, alpha, beta)."""
    T = x.shape[0]
    q, k, v = mmd(x, w["q"]), mmd(x, w["k"]), mmd(x, w["v"])
    bt = mmd(x, w["b"])
    z = mmd(mmd(x, w["f_a"]), w["f_b"])
    al, be = np.zeros((T, P), np.float32), np.zeros((T, H), np.float32)
    h = np.ascontiguousarray(hist.copy())
    O.orc().orc_kda_prologue(q, k, v, al, be, z, bt, w["q_conv"], w["k_conv"], w["v_conv"], h.ctypes.data,
                             w["A_log"], w["dt_bias"], T, H, D, K, LB)
    hd = lambda a: np.ascontiguousarray(a.reshape(T, H, D))
    o = O.kda_verify(state, hd(q), hd(k), hd(v), hd(al), be, np.float32(1.0) / np.sqrt(np.float32(D)))
    o = np.ascontiguousarray(o.reshape(T, P))
    g = mmd(x, w["g"])
    O.orc().orc_kda_norm_gate(o, g, w["o_norm"], T, H, D, EPS)
    return mmd(o, w["o"]), (k, v, al, be)


def cfg(k3, **kw):
    base = dict(hidden=E, kda_heads=H, kda_head_dim=D, conv_k=K, gate_lb=LB, rms_eps=EPS, attn_res_block=2,
                max_blocks=4, n_routed=16, n_shared=1, topk=2, moe_inter=256, act=k3.ACT_SWIGLU, renorm=1,
                routed_scale=1.0, situ_b1=4.0, situ_b2=25.0)
    base.update(kw)
    return k3.layer_cfg(**base)


def test_kda_layer_verify_vs_oracle(k3):
    B, T = 2, 5
    rng = np.random.default_rng(11)
    w = kda_weights(rng)
    x = rng.standard_normal((B * T, E), dtype=np.float32)
    state = rng.standard_normal((B, H, D, D), dtype=np.float32) * np.float32(0.1)
    hist = rng.standard_normal((B, 3, P, K - 1), dtype=np.float32)
    wd = to_dev(w)
    out, lt = k3.kda_layer_verify(dev(x), wd, cfg(k3), dev(state), dev(hist), B, T)
    got = out.cpu().numpy()
    for b in range(B):
        ref, (k, v, al, be) = oracle_kda_layer(x[b * T:(b + 1) * T], w, state[b], hist[b])
        assert rel(got[b * T:(b + 1) * T], ref) < 1e-4
        assert rel(lt["k"].cpu().numpy()[b], k) < 1e-4
        assert rel(lt["v"].cpu().numpy()[b], v) < 1e-4
        assert rel(lt["alpha"].cpu().numpy()[b], al) < 1e-4
        assert rel(lt["beta"].cpu().numpy()[b], be) < 1e-4


@pytest.mark.parametrize("layer_idx", [2, 3], ids=["boundary", "inner"])
def test_decoder_layer_kda_verify_vs_oracle(k3, layer_idx):
    B, T, maxb = 2, 4, 4
    R = B * T
    c = cfg(k3)
    rng = np.random.default_rng(20 + layer_idx)
    w = kda_weights(rng)
    for n in ("attn_res_fold", "mlp_res_fold"):
        w[n] = rng.standard_normal(E, dtype=np.float32) * np.float32(0.05)
    for n in ("in_norm", "post_norm"):
        w[n] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    w["gate_W"] = rng.standard_normal((c.n_routed, E), dtype=np.float32) * np.float32(0.2)
    w["gate_bias"] = rng.standard_normal(c.n_routed, dtype=np.float32) * np.float32(0.01)
    bank, lay = O.make_bank(rng, c.n_routed + c.n_shared, E, c.moe_inter, std=0.05, w13_std=0.3)
    h0 = rng.standard_normal((R, E), dtype=np.float32)
    br0 = rng.standard_normal((R, maxb, E), dtype=np.float32)
    nb0 = np.array([0, 1, 2, 3, 1, 2, 0, 3], np.int32)
    state = rng.standard_normal((B, H, D, D), dtype=np.float32) * np.float32(0.1)
    hist = rng.standard_normal((B, 3, P, K - 1), dtype=np.float32)

    wd = to_dev(w)
    kb = k3.ExpertBank(dev(bank), c.n_routed + c.n_shared, E, c.moe_inter)
    h, br, nb = dev(h0), dev(br0), dev(nb0)
    idx, wt, _ = k3.decoder_layer_kda_verify(h, br, nb, wd, kb, c, layer_idx, dev(state), dev(hist), B, T)

    # the oracle composition of k3_decoder_layer_core
    def attn_res(fold, brr, nbr, cur):
        out = np.empty_like(cur)
        for t in range(R):
            src = np.ascontiguousarray(np.concatenate([brr[t, :nbr[t]], cur[t:t + 1]]))
            O.orc().orc_attn_res(out[t], src, fold, src.shape[0], E, EPS)
        return out

    pref = h0.copy()
    hh = attn_res(w["attn_res_fold"], br0, nb0, pref)
    brr, nbr = br0.copy(), nb0.copy()
    boundary = layer_idx % c.attn_res_block == 0
    if boundary:
        for t in range(R):
            brr[t, nbr[t]] = pref[t]
            nbr[t] += 1
    hin = O.rmsnorm(hh, w["in_norm"], EPS)
    tmp = np.concatenate([oracle_kda_layer(hin[b * T:(b + 1) * T], w, state[b], hist[b])[0] for b in range(B)])
    pref = tmp if boundary else pref + tmp
    hh = attn_res(w["mlp_res_fold"], brr, nbr, pref)
    hin = O.rmsnorm(hh, w["post_norm"], EPS)
    ri, rw = O.router(hin, w["gate_W"], w["gate_bias"], c.topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    moe = O.moe_routed(hin, ri, rw, bank, lay, E, c.moe_inter, c.topk, c.n_routed, c.n_shared, c.act)
    ref = pref + moe

    assert rel(h.cpu().numpy(), ref) < 1e-4
    np.testing.assert_array_equal(nb.cpu().numpy(), nbr)
    np.testing.assert_array_equal(br.cpu().numpy(), brr)


def oracle_moe_k3(x, w, bank, lay, L, I, topk, n_routed, SI, act, eps=EPS):
    """k3_moe_prefill composed from the oracle: route on x, experts on down(x) at L with
    the latent norm, up-projection, plus the dense shared expert on x."""
    z = mmd(x, w["down"])
    ri, rw = O.router(x, w["gate_W"], w["gate_bias"], topk)
    acc = O.moe_routed(z, ri, rw, bank, lay, L, I, topk, n_routed, 0, act, latent_norm=w.get("latent_norm"),
                       eps=eps)
    out = mmd(acc, w["up"])
    if SI:
        gu = np.ascontiguousarray(np.concatenate([mmd(x, w["sh1"]), mmd(x, w["sh3"])], axis=1))
        a = np.empty((x.shape[0], SI), np.float32)
        for t in range(x.shape[0]):
            if act == 0:
                O.orc().orc_situ_glu(a[t], np.ascontiguousarray(gu[t]), SI, 4.0, 25.0)
            else:
                O.orc().orc_swiglu(a[t], np.ascontiguousarray(gu[t]), SI)
        out = out + mmd(a, w["sh2"])
    return out, ri


def k3_moe_weights(rng, E, L, SI, n_routed):
    w = {"down": bf16_bits(rng.standard_normal((L, E), dtype=np.float32) * np.float32(0.05)),
         "up": bf16_bits(rng.standard_normal((E, L), dtype=np.float32) * np.float32(0.05)),
         "sh1": bf16_bits(rng.standard_normal((SI, E), dtype=np.float32) * np.float32(0.05)),
         "sh3": bf16_bits(rng.standard_normal((SI, E), dtype=np.float32) * np.float32(0.05)),
         "sh2": bf16_bits(rng.standard_normal((E, SI), dtype=np.float32) * np.float32(0.05)),
         "gate_W": rng.standard_normal((n_routed, E), dtype=np.float32) * np.float32(0.2),
         "gate_bias": rng.standard_normal(n_routed, dtype=np.float32) * np.float32(0.01),
         "latent_norm": (1 + 0.1 * rng.standard_normal(L)).astype(np.float32)}
    return w


def test_moe_prefill_k3_form_vs_oracle(k3):
    """E 1024, latent 512, FFN 512 (tensor-core experts), 8 experts top-2, a 512-wide
    dense SiTU shared expert, 12 positions."""
    E2, L, I, n_routed, topk, SI, T = 1024, 512, 512, 8, 2, 512, 12
    rng = np.random.default_rng(31)
    w = k3_moe_weights(rng, E2, L, SI, n_routed)
    bank, lay = O.make_bank(rng, n_routed, L, I, std=0.05, w13_std=0.1)
    x = rng.standard_normal((T, E2), dtype=np.float32)
    c = k3.K3GpuMoeCfg(hidden=E2, latent=L, moe_inter=I, shared_inter=SI, n_routed=n_routed, topk=topk, act=0,
                       renorm=1, routed_scale=1.0, situ_b1=4.0, situ_b2=25.0, rms_eps=EPS)
    kb = k3.ExpertBank(dev(bank), n_routed, L, I)
    kb.scan()
    out, idx, _ = k3.moe_prefill(dev(x), to_dev(w), kb, c)
    ref, ri = oracle_moe_k3(x, w, bank, lay, L, I, topk, n_routed, SI, 0)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    assert rel(out.cpu().numpy(), ref) < 1e-4


def test_decoder_layer_with_k3_moe_form(k3):
    B, T, maxb = 2, 3, 4
    R = B * T
    L, I, SI = 256, 256, 256
    c = cfg(k3, latent=L, shared_inter=SI, moe_inter=I, n_routed=8, topk=2, act=0)
    rng = np.random.default_rng(41)
    w = kda_weights(rng)
    for n in ("attn_res_fold", "mlp_res_fold"):
        w[n] = rng.standard_normal(E, dtype=np.float32) * np.float32(0.05)
    for n in ("in_norm", "post_norm"):
        w[n] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    m = k3_moe_weights(rng, E, L, SI, c.n_routed)
    w["gate_W"], w["gate_bias"] = m["gate_W"], m["gate_bias"]
    bank, lay = O.make_bank(rng, c.n_routed, L, I, std=0.05, w13_std=0.3)
    h0 = rng.standard_normal((R, E), dtype=np.float32)
    br0 = rng.standard_normal((R, maxb, E), dtype=np.float32)
    nb0 = np.array([1, 0, 2, 3, 1, 2], np.int32)
    state = rng.standard_normal((B, H, D, D), dtype=np.float32) * np.float32(0.1)
    hist = rng.standard_normal((B, 3, P, K - 1), dtype=np.float32)
    kb = k3.ExpertBank(dev(bank), c.n_routed, L, I)
    h, br, nb = dev(h0), dev(br0), dev(nb0)
    idx, _, _ = k3.decoder_layer_kda_verify(h, br, nb, to_dev(w), kb, c, 3, dev(state), dev(hist), B, T,
                                            moe=to_dev(m))

    def attn_res(fold, cur):
        out = np.empty_like(cur)
        for t in range(R):
            src = np.ascontiguousarray(np.concatenate([br0[t, :nb0[t]], cur[t:t + 1]]))
            O.orc().orc_attn_res(out[t], src, fold, src.shape[0], E, EPS)
        return out

    pref = h0.copy()                                   # layer 3: not a block boundary
    hin = O.rmsnorm(attn_res(w["attn_res_fold"], pref), w["in_norm"], EPS)
    pref = pref + np.concatenate([oracle_kda_layer(hin[b * T:(b + 1) * T], w, state[b], hist[b])[0]
                                  for b in range(B)])
    hin = O.rmsnorm(attn_res(w["mlp_res_fold"], pref), w["post_norm"], EPS)
    moe, ri = oracle_moe_k3(hin, m, bank, lay, L, I, c.topk, c.n_routed, SI, 0)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    assert rel(h.cpu().numpy(), pref + moe) < 1e-4


# ---------------------------------------------------------------------------- MLA --
# k3_mla_cached (src/core/k3_ops.c:1115-1615) in the absorbed latent layout: the oracle
# composes the double matmuls of the bf16 weights, orc_rmsnorm, the bf16 rounding of the
# appended cache rows (this library's cache is bf16), orc_mla_absorbed with the node masks,
# the sigmoid gate and o. Bar: rel-L2 <= 1e-4 on the output; the appended rows agree to a
# bf16 ulp plus 1e-4 of the row scale (their inputs come from the device projection, whose
# error is relative to the row); every other cache row untouched.
MH, QL, QN, VH = 4, 128, 32, 32


def mla_weights(rng, kvl, qr):
    w = {"q_a": bf16_bits(rng.standard_normal((QL, E), dtype=np.float32) * np.float32(0.05)),
         "q_b": bf16_bits(rng.standard_normal((MH * (QN + qr), QL), dtype=np.float32) * np.float32(0.1)),
         "kv_a": bf16_bits(rng.standard_normal((kvl + qr, E), dtype=np.float32) * np.float32(0.05)),
         "g": bf16_bits(rng.standard_normal((MH * VH, E), dtype=np.float32) * np.float32(0.05)),
         "o": bf16_bits(rng.standard_normal((E, MH * VH), dtype=np.float32) * np.float32(0.1)),
         "q_a_norm": (1 + 0.1 * rng.standard_normal(QL)).astype(np.float32),
         "kv_a_norm": (1 + 0.1 * rng.standard_normal(kvl)).astype(np.float32),
         "kv_b": rng.standard_normal((MH * (QN + VH), kvl), dtype=np.float32) * np.float32(0.1)}
    return w


def mla_cfg(k3, kvl, qr, **kw):
    return cfg(k3, mla_heads=MH, q_lora=QL, kv_lora=kvl, qk_nope=QN, qk_rope=qr, v_head=VH, **kw)


def bf16_round(a):
    return O.bf16_bits_to_f32(bf16_bits(a))


def oracle_mla_layer(x, w, lat, rope, cached, masks, kvl, qr):
    """One sequence: x [T][E] -> out [T][E]; lat/rope [cap][.] float, updated in place."""
    T = x.shape[0]
    q = mmd(O.rmsnorm(mmd(x, w["q_a"]), w["q_a_norm"], EPS), w["q_b"]).reshape(T, MH, QN + qr)
    ct = mmd(x, w["kv_a"])
    lat[cached:cached + T] = bf16_round(O.rmsnorm(np.ascontiguousarray(ct[:, :kvl]), w["kv_a_norm"], EPS))
    rope[cached:cached + T] = bf16_round(ct[:, kvl:])
    acc = O.mla_absorbed(np.ascontiguousarray(q[..., :QN]), np.ascontiguousarray(q[..., QN:]), w["kv_b"], lat,
                         rope, cached, masks, 1.0 / np.sqrt(np.float32(QN + qr)), VH).reshape(T, MH * VH)
    g = mmd(x, w["g"])
    acc = (acc * (1.0 / (1.0 + np.exp(-g.astype(np.float64))))).astype(np.float32)
    return mmd(acc, w["o"])


@pytest.mark.parametrize("kvl,qr,tree", [(512, 64, True), (128, 64, False), (128, 16, True)],
                         ids=["k3_tree", "chain", "cudacore_rope16"])
def test_mla_layer_verify_vs_oracle(k3, kvl, qr, tree):
    B, T = 2, 9
    cached = [300, 41]
    cap = max(cached) + T + 5
    rng = np.random.default_rng(60 + kvl + qr)
    w = mla_weights(rng, kvl, qr)
    x = rng.standard_normal((B * T, E), dtype=np.float32)
    lat0 = bf16_round(rng.standard_normal((B, cap, kvl), dtype=np.float32))
    rope0 = bf16_round(rng.standard_normal((B, cap, qr), dtype=np.float32))
    for b in range(B):                                  # unspecified rows past the new ones
        lat0[b, cached[b] + T:] = np.nan
        rope0[b, cached[b] + T:] = np.nan
    masks = O.tree_masks([-1, 0, 0, 1, 1, 2, 2, 3, 3]) if tree else O.chain_masks(T)
    lat_d, rope_d = dev(bf16_bits(lat0).view(np.int16)), dev(bf16_bits(rope0).view(np.int16))
    out = k3.mla_layer_verify(dev(x), to_dev(w), mla_cfg(k3, kvl, qr), lat_d, rope_d,
                              dev(np.array(cached, np.int32)), dev(masks.view(np.int64)), cap, B, T)
    got = out.cpu().numpy()
    lat_g = O.bf16_bits_to_f32(lat_d.cpu().numpy().view(np.uint16))
    rope_g = O.bf16_bits_to_f32(rope_d.cpu().numpy().view(np.uint16))
    for b in range(B):
        lat, rope = lat0[b].copy(), rope0[b].copy()
        ref = oracle_mla_layer(x[b * T:(b + 1) * T], w, lat, rope, cached[b], masks, kvl, qr)
        assert np.isfinite(got[b * T:(b + 1) * T]).all()
        assert rel(got[b * T:(b + 1) * T], ref) < 1e-4, rel(got[b * T:(b + 1) * T], ref)
        new = slice(cached[b], cached[b] + T)
        for gc, rc in ((lat_g[b], lat), (rope_g[b], rope)):
            # a bf16 ulp, plus the projection's ~1e-5 error measured on the row scale
            np.testing.assert_allclose(gc[new], rc[new], rtol=2 ** -7, atol=1e-4 * np.abs(rc[new]).max())
            keep = np.r_[0:cached[b]]
            np.testing.assert_array_equal(gc[keep], rc[keep])
            assert np.isnan(gc[cached[b] + T:]).all()
    assert k3.device_status(0) == 0


def test_decoder_layer_mla_verify_vs_oracle(k3):
    """An MLA + MoE decoder layer on a block-boundary layer index (snapshot taken)."""
    B, T, maxb = 2, 4, 4
    R = B * T
    kvl, qr = 512, 64
    c = mla_cfg(k3, kvl, qr)
    cached = [200, 33]
    cap = max(cached) + T
    rng = np.random.default_rng(71)
    w = mla_weights(rng, kvl, qr)
    for n in ("attn_res_fold", "mlp_res_fold"):
        w[n] = rng.standard_normal(E, dtype=np.float32) * np.float32(0.05)
    for n in ("in_norm", "post_norm"):
        w[n] = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    w["gate_W"] = rng.standard_normal((c.n_routed, E), dtype=np.float32) * np.float32(0.2)
    w["gate_bias"] = rng.standard_normal(c.n_routed, dtype=np.float32) * np.float32(0.01)
    bank, lay = O.make_bank(rng, c.n_routed + c.n_shared, E, c.moe_inter, std=0.05, w13_std=0.3)
    h0 = rng.standard_normal((R, E), dtype=np.float32)
    br0 = rng.standard_normal((R, maxb, E), dtype=np.float32)
    nb0 = np.array([0, 1, 2, 3, 1, 2, 0, 3], np.int32)
    lat0 = bf16_round(rng.standard_normal((B, cap, kvl), dtype=np.float32))
    rope0 = bf16_round(rng.standard_normal((B, cap, qr), dtype=np.float32))
    masks = O.chain_masks(T)
    kb = k3.ExpertBank(dev(bank), c.n_routed + c.n_shared, E, c.moe_inter)
    h, br, nb = dev(h0), dev(br0), dev(nb0)
    lat_d, rope_d = dev(bf16_bits(lat0).view(np.int16)), dev(bf16_bits(rope0).view(np.int16))
    idx, _ = k3.decoder_layer_mla_verify(h, br, nb, to_dev(w), kb, c, 2, lat_d, rope_d,
                                         dev(np.array(cached, np.int32)), dev(masks.view(np.int64)), cap, B, T)

    def attn_res(fold, brr, nbr, cur):
        out = np.empty_like(cur)
        for t in range(R):
            src = np.ascontiguousarray(np.concatenate([brr[t, :nbr[t]], cur[t:t + 1]]))
            O.orc().orc_attn_res(out[t], src, fold, src.shape[0], E, EPS)
        return out

    pref = h0.copy()
    hh = attn_res(w["attn_res_fold"], br0, nb0, pref)
    brr, nbr = br0.copy(), nb0.copy()
    for t in range(R):                                   # layer 2: a block boundary
        brr[t, nbr[t]] = pref[t]
        nbr[t] += 1
    hin = O.rmsnorm(hh, w["in_norm"], EPS)
    pref = np.concatenate([oracle_mla_layer(hin[b * T:(b + 1) * T], w, lat0[b].copy(), rope0[b].copy(), cached[b],
                                            masks, kvl, qr) for b in range(B)])
    hin = O.rmsnorm(attn_res(w["mlp_res_fold"], brr, nbr, pref), w["post_norm"], EPS)
    ri, rw = O.router(hin, w["gate_W"], w["gate_bias"], c.topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    moe = O.moe_routed(hin, ri, rw, bank, lay, E, c.moe_inter, c.topk, c.n_routed, c.n_shared, c.act)
    assert rel(h.cpu().numpy(), pref + moe) < 1e-4
    np.testing.assert_array_equal(nb.cpu().numpy(), nbr)
    np.testing.assert_array_equal(br.cpu().numpy(), brr)
