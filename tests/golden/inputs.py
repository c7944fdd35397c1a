"""Seeded input generators shared by tests/golden/make_golden.py and the tests.

The golden files store only outputs; the inputs are rebuilt here from fixed seeds with
numpy's PCG64 generator, whose streams are stable across numpy versions. Distributions
follow the benchmark configurations (router/expert weights N(0, 0.02) quantised to
MXFP4, activations bf16 N(0, 1), router bias N(0, 0.01); KDA state N(0, 0.1), q and k
L2-normalised bf16, v N(0, 1), decay U(0.9, 0.999), beta = sigmoid(N(0, 1))).
"""
from __future__ import annotations

import numpy as np

from oracle import oracle as O


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even), returned as fp32."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


ROUTER_CASES = [
    # Benchmark config 2 router: 384 experts over d_model 7168, top-8, 16 tokens
    dict(name="c2_t16", seed=11, T=16, hidden=7168, n=384, topk=8, wstd=0.02, bstd=0.01),
    # Benchmark config 1 router: 16 experts over 512, top-2
    dict(name="c1_t9", seed=12, T=9, hidden=512, n=16, topk=2, wstd=0.02, bstd=0.01),
    # exact ties: duplicated gate rows and a zero bias, so the first-index rule decides
    dict(name="ties", seed=13, T=8, hidden=96, n=64, topk=6, wstd=0.05, bstd=0.0, dup=True),
]


def router_inputs(case):
    rng = np.random.default_rng(case["seed"])
    x = bf16_round(rng.standard_normal((case["T"], case["hidden"]), dtype=np.float32))
    W = rng.standard_normal((case["n"], case["hidden"]), dtype=np.float32) * np.float32(case["wstd"])
    if case.get("dup"):
        W[1::2] = W[0::2]          # experts 2i and 2i+1 score identically
    bias = (rng.standard_normal(case["n"], dtype=np.float32) * np.float32(case["bstd"])
            if case["bstd"] > 0 else np.zeros(case["n"], np.float32))
    return np.ascontiguousarray(x), np.ascontiguousarray(W), np.ascontiguousarray(bias)


MXFP4_CASES = [
    dict(name="w1_7168", seed=21, rows=256, **{"in": 7168}),
    dict(name="w2_2048", seed=22, rows=192, **{"in": 2048}),
]


def mxfp4_inputs(case):
    rng = np.random.default_rng(case["seed"])
    W = rng.standard_normal((case["rows"], case["in"]), dtype=np.float32) * np.float32(0.02)
    packed, scales = O.mxfp4_quant(W)
    x = bf16_round(rng.standard_normal(case["in"], dtype=np.float32))
    return packed, scales, x


KDA_CASES = [
    # Benchmark config 3 geometry (head dim 128) at k = 16, two heads to keep files small
    dict(name="d128_k16", seed=31, T=17, H=2, D=128, commits=[0, 1, 5, 9, 17]),
    dict(name="d64_k4", seed=32, T=5, H=4, D=64, commits=[0, 2, 5]),
]


def l2n(a):
    n = np.sqrt((a.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6)
    return (a / n).astype(np.float32)


def kda_inputs(case):
    rng = np.random.default_rng(case["seed"])
    T, H, D = case["T"], case["H"], case["D"]
    st = rng.standard_normal((H, D, D), dtype=np.float32) * np.float32(0.1)
    q = bf16_round(l2n(rng.standard_normal((T, H, D), dtype=np.float32)))
    k = bf16_round(l2n(rng.standard_normal((T, H, D), dtype=np.float32)))
    v = rng.standard_normal((T, H, D), dtype=np.float32)
    al = rng.uniform(0.9, 0.999, (T, H, D)).astype(np.float32)
    be = (1.0 / (1.0 + np.exp(-rng.standard_normal((T, H))))).astype(np.float32)
    # a few exact zeros in k and q: the recurrence skips those rows (k3_ops.c:333,354)
    k[0, 0, :3] = 0.0
    q[1, 0, 5:9] = 0.0
    return st, q, k, v, al, be


def latent_moe_inputs():
    """A small LatentMoE (hidden 128, latent 64, 8 experts top-2, one shared expert of
    intermediate 64) with MXFP4 routed experts, fp32 trunk matrices."""
    rng = np.random.default_rng(41)
    E, L, I, n, topk, ns = 128, 64, 64, 8, 2, 1
    bank, lay = O.make_bank(rng, n, L, I, std=0.1, w13_std=0.5)
    p = dict(E=E, L=L, I=I, n_experts=n, topk=topk, n_shared=ns, bank=bank, lay=lay)
    p["gate"] = rng.standard_normal((n, E), dtype=np.float32) * np.float32(0.1)
    p["bias"] = np.linspace(-0.15, 0.15, n).astype(np.float32)
    p["latent_norm"] = (1.0 + 0.1 * rng.standard_normal(L)).astype(np.float32)
    p["down"] = rng.standard_normal((L, E), dtype=np.float32) * np.float32(0.1)
    p["up"] = rng.standard_normal((E, L), dtype=np.float32) * np.float32(0.1)
    SI = I * ns
    p["sh1"] = rng.standard_normal((SI, E), dtype=np.float32) * np.float32(0.3)
    p["sh3"] = rng.standard_normal((SI, E), dtype=np.float32) * np.float32(0.3)
    p["sh2"] = rng.standard_normal((E, SI), dtype=np.float32) * np.float32(0.1)
    p["x"] = rng.standard_normal((5, E), dtype=np.float32)
    return p
