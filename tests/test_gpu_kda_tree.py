"""The KDA recurrence and ShortConv over a draft TREE on a B200 (no counterpart in the
reference, whose sweeps are chains): every node must see exactly what a chain along its own
ancestor path sees. The recurrence is held bit-exact to the oracle's restatement of
k3_kda_step (src/core/k3_ops.c:303-360) run on each node's path; the prologue to the
oracle's ShortConv / L2 norm / decay chain (src/core/k3_ops.c:171-221, 2286-2303) on each
node's path with the carried history."""
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from oracle import oracle as O  # noqa: E402
from tests.golden import inputs as GI  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def k3():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tests.k3lib import load
    return load()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def random_tree(rng, T, max_back=4):
    parent = [-1]
    for i in range(1, T):
        parent.append(int(rng.integers(max(0, i - max_back), i)))
    return parent


def path_of(parent, t):
    p = []
    while t >= 0:
        p.append(t)
        t = parent[t]
    return p[::-1]


def best_first_tree(T=64, branch=4, depth=4):
    """The benchmark's draft-tree shape: nodes grown best-first under a branching and depth
    cap (most nodes are leaves, internal nodes at every depth)."""
    parent, dep = [-1], [0]
    frontier = [0]
    while len(parent) < T and frontier:
        p = frontier.pop(0)
        for _ in range(branch):
            if len(parent) >= T:
                break
            parent.append(p)
            dep.append(dep[p] + 1)
            if dep[-1] < depth:
                frontier.append(len(parent) - 1)
    return parent


TREES = {
    "random": None,
    "best_first": lambda rng, T: best_first_tree(T),
    "star": lambda rng, T: [-1] + [0] * (T - 1),
    # several roots on the carried state, some of them leaves
    "forest": lambda rng, T: [-1] + [(-1 if i % 5 == 0 else int(rng.integers(max(0, i - 3), i))) for i in range(1, T)],
}


@pytest.mark.parametrize("D,T,kind", [(128, 17, "random"), (64, 40, "random"), (32, 64, "random"),
                                      (128, 64, "best_first"), (128, 33, "star"), (64, 45, "forest"),
                                      (16, 64, "best_first")])
def test_kda_verify_tree_bitexact_on_every_path(k3, D, T, kind):
    rng = np.random.default_rng(D + T)
    B, H = 2, 3
    parent = random_tree(rng, T) if TREES[kind] is None else TREES[kind](rng, T)
    st = rng.standard_normal((B, H, D, D), dtype=np.float32) * np.float32(0.1)
    q = GI.bf16_round(GI.l2n(rng.standard_normal((B, T, H, D), dtype=np.float32)))
    k = GI.bf16_round(GI.l2n(rng.standard_normal((B, T, H, D), dtype=np.float32)))
    v = rng.standard_normal((B, T, H, D), dtype=np.float32)
    al = rng.uniform(0.9, 0.999, (B, T, H, D)).astype(np.float32)
    be = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H))))).astype(np.float32)
    k[0, 2, 1, :5] = 0.0                       # zero rows are skipped as in the chain
    k[1, T - 1, 2, 3:9] = 0.0                  # (a leaf's too)
    q[1, T - 2, 0, :7] = 0.0
    qs = np.float32(1.0) / np.sqrt(np.float32(D))
    o = k3.kda_verify_tree(dev(st), dev(q), dev(k), dev(v), dev(al), dev(be),
                           dev(np.asarray(parent, np.int32)), qs).cpu().numpy()
    for b in range(B):
        for t in range(T):
            p = path_of(parent, t)
            want = O.kda_verify(st[b], q[b][p], k[b][p], v[b][p], al[b][p], be[b][p], qs)[-1]
            np.testing.assert_array_equal(o[b, t], want, err_msg=f"sequence {b} node {t} path {p}")
    # a chain given as parents is the chain
    chain = list(range(-1, T - 1))
    oc = k3.kda_verify_tree(dev(st), dev(q), dev(k), dev(v), dev(al), dev(be),
                            dev(np.asarray(chain, np.int32)), qs).cpu().numpy()
    o_chain = k3.kda_verify(dev(st), dev(q), dev(k), dev(v), dev(al), dev(be), qs).cpu().numpy()
    np.testing.assert_array_equal(oc, o_chain)
    assert k3.device_status() == 0


def test_kda_prologue_tree_is_the_chain_along_each_path(k3):
    rng = np.random.default_rng(77)
    B, T, H, D, K = 2, 21, 4, 64, 4
    P = H * D
    parent = random_tree(rng, T, max_back=6)
    q, k, v, z = (rng.standard_normal((B, T, P), dtype=np.float32) for _ in range(4))
    b = rng.standard_normal((B, T, H), dtype=np.float32)
    qc, kc, vc = (rng.standard_normal((P, K), dtype=np.float32) * np.float32(0.4) for _ in range(3))
    hist = rng.standard_normal((B, 3, P, K - 1), dtype=np.float32)
    A = np.linspace(-0.4, 1.2, H).astype(np.float32)
    dt = rng.standard_normal(P, dtype=np.float32) * np.float32(0.5)
    tq, tk, tv = dev(q), dev(k), dev(v)
    al, be, pre = k3.kda_prologue_tree(tq, tk, tv, dev(z), dev(b), dev(qc), dev(kc), dev(vc), dev(hist),
                                       dev(A), dev(dt), dev(np.asarray(parent, np.int32)), H, D, K, -5.0)
    got = [x.cpu().numpy() for x in (tq, tk, tv, al, be, pre)]
    for bb in range(B):
        for t in range(T):
            p = path_of(parent, t)
            n = len(p)
            rq, rk, rv = q[bb][p].copy(), k[bb][p].copy(), v[bb][p].copy()
            ral, rbe = np.zeros((n, P), np.float32), np.zeros((n, H), np.float32)
            h = hist[bb].copy()
            O.orc().orc_kda_prologue(rq, rk, rv, ral, rbe, np.ascontiguousarray(z[bb][p]),
                                     np.ascontiguousarray(b[bb][p]), qc, kc, vc, h.ctypes.data, A, dt, n,
                                     H, D, K, -5.0)
            for g, want in ((got[0], rq), (got[1], rk), (got[2], rv), (got[3], ral), (got[4], rbe)):
                np.testing.assert_allclose(g[bb, t], want[-1], rtol=2e-6, atol=1e-6,
                                           err_msg=f"sequence {bb} node {t} path {p}")
        np.testing.assert_array_equal(got[5][bb][:, 0], q[bb])
    assert k3.device_status() == 0
