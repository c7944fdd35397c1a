"""The chunked (UT-transform) form of the KDA recurrence against the sequential one, CPU.

oracle.kda_chunked is the checker a chunked prefill kernel will be held to; here it is
itself held to the sequential recurrence (oracle.kda_verify / kda_commit, bit-exact with
the reference's k3_kda_step): outputs and the end state within rel-L2 1e-5 (the
sequential side rounds in fp32 at every step, the chunked side is float64), for ragged
chunks, strong and weak decay, and chunk sizes from 1 to the whole sequence.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from oracle import oracle as O  # noqa: E402


def inputs(seed, T, H, D, decay):
    rng = np.random.default_rng(seed)
    st = rng.standard_normal((H, D, D), dtype=np.float32) * np.float32(0.1)
    q, k, v = (rng.standard_normal((T, H, D), dtype=np.float32) for _ in range(3))
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    lo, hi = decay
    al = rng.uniform(lo, hi, (T, H, D)).astype(np.float32)
    be = rng.uniform(0.1, 0.9, (T, H)).astype(np.float32)
    return st, q, k, v, al, be


def rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("T,H,D,chunk,decay", [
    (1, 2, 64, 64, (0.9, 0.999)), (37, 2, 64, 16, (0.9, 0.999)), (130, 2, 64, 64, (0.9, 0.999)),
    (100, 1, 128, 32, (0.3, 0.7)), (64, 3, 32, 64, (0.995, 1.0)), (90, 2, 64, 90, (0.05, 0.3)),
])
def test_chunked_equals_sequential(T, H, D, chunk, decay):
    st, q, k, v, al, be = inputs(T * 7 + D, T, H, D, decay)
    qs = np.float32(1.0) / np.sqrt(np.float32(D))
    o_seq = O.kda_verify(st, q, k, v, al, be, qs)
    s_seq = O.kda_commit(st, k, v, al, be, T)
    o_ch, s_ch = O.kda_chunked(st, q, k, v, al, be, qs, chunk)
    assert rel(o_ch, o_seq) < 1e-5
    assert rel(s_ch, s_seq) < 1e-5


def test_chunk_size_does_not_matter():
    st, q, k, v, al, be = inputs(5, 75, 2, 64, (0.8, 0.99))
    ref_o, ref_s = O.kda_chunked(st, q, k, v, al, be, 0.125, 75)
    for c in (1, 8, 16, 64):
        o, s = O.kda_chunked(st, q, k, v, al, be, 0.125, c)
        assert rel(o, ref_o) < 1e-6 and rel(s, ref_s) < 1e-6, c


def test_full_decay_zero_alpha_is_finite():
    """alpha = 0 in a channel (a decay that underflowed in fp32) forgets that channel."""
    st, q, k, v, al, be = inputs(6, 20, 1, 32, (0.5, 0.9))
    al[7, 0, :5] = 0.0
    o_ch, s_ch = O.kda_chunked(st, q, k, v, al, be, 0.25, 8)
    assert np.isfinite(o_ch).all() and np.isfinite(s_ch).all()
    assert rel(o_ch, O.kda_verify(st, q, k, v, al, be, np.float32(0.25))) < 1e-5
    assert rel(s_ch, O.kda_commit(st, k, v, al, be, 20)) < 1e-5


@pytest.mark.parametrize("T,H,D,decay", [
    (128, 2, 128, (0.9, 0.999)), (128, 2, 128, (0.3, 0.7)), (128, 2, 128, (0.05, 0.3)),
    (96, 2, 64, (0.995, 1.0)), (64, 2, 128, (0.001, 0.01)), (50, 1, 32, (0.5, 0.99)),
])
def test_factored_float32_form_equals_sequential(T, H, D, decay):
    """The form a tensor-core prefill computes -- float32, decay ratios factored about the
    chunk's middle so the pair sums are plain products, the exact per-pair form where the
    chunk's decay range passes 100 (log2) -- stays within rel-L2 1e-5 of the sequential
    recurrence; the strongest decay here (range ~260) takes the fallback."""
    st, q, k, v, al, be = inputs(T * 3 + D, T, H, D, decay)
    qs = np.float32(1.0) / np.sqrt(np.float32(D))
    o_f, s_f = O.kda_chunked_factored_f32(st, q, k, v, al, be, qs, 32)
    assert rel(o_f, O.kda_verify(st, q, k, v, al, be, qs)) < 1e-5
    assert rel(s_f, O.kda_commit(st, k, v, al, be, T)) < 1e-5
