"""Temperature sampling's checker (oracle.orc_accept_sample, which the device kernel
k3gpu_accept_sample equals bit for bit on a B200), CPU only. The reference decodes
greedily, so there is no reference output to pin it to; instead:

* its Philox4x32-10 is checked against the generator's published known-answer vectors
  (Salmon et al., SC'11; the Random123 distribution's kat_vectors), through the uniform
  it derives from the first two output words;
* the speculative rejection rule must leave the model's distribution unchanged whatever
  the drafts: over many seeds the first emitted id follows softmax(logits_0 / temp), and,
  given the first draft was accepted, the second follows softmax(logits_1 / temp)
  (chi-square, fixed seeds, bounds far from the observed values).
"""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from oracle import oracle as O  # noqa: E402

# (counter words c0..c3, key words k0 k1) -> first two output words
PHILOX_KAT = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D)),
              ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E)),
              ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
               (0xD16CFE09, 0x94FDCCEB))]


def test_philox_known_answers():
    for (c0, c1, c2, c3), (k0, k1), (o0, o1) in PHILOX_KAT:
        want = (((o0 >> 5) << 26) | (o1 >> 6)) / 9007199254740992.0    # the 53-bit uniform
        got = O.orc().orc_philox_uniform(k0 | (k1 << 32), c0 | (c1 << 32), c2, c3 // 2, c3 % 2)
        assert got == want


def _softmax(l, temp):
    z = np.exp((l - l.max()) / temp)
    return z / z.sum()


def _chi2(counts, p):
    n = counts.sum()
    e = p * n
    return float(((counts - e) ** 2 / e).sum())


def test_rejection_rule_keeps_the_model_distribution():
    rng = np.random.default_rng(61)
    V, nd, temp, N = 6, 3, 0.7, 20000
    lg = rng.standard_normal((nd + 1, V)).astype(np.float32) * np.float32(1.5)
    d = np.array([int(np.argsort(lg[0])[-2]), 1, 4], np.int32)        # a plausible, not the top, draft
    emit = np.zeros(nd + 1, np.int32)
    first, second = np.zeros(V), np.zeros(V)
    for seed in range(N):
        n = O.orc().orc_accept_sample(emit, np.ascontiguousarray(lg), d, nd, V, temp, seed, 0, 0)
        first[emit[0]] += 1
        if emit[0] == d[0] and n >= 2:
            second[emit[1]] += 1
    p0, p1 = _softmax(lg[0], temp), _softmax(lg[1], temp)
    # 5 degrees of freedom: 20.5 is p = 0.001; a rule that ignored the draft's probability
    # or sampled the residual without removing d lands in the thousands
    assert _chi2(first, p0) < 20.5
    assert second.sum() > 0.5 * N * p0[d[0]] and _chi2(second, p1) < 20.5
