"""The chunked KDA prefill (k3gpu_kda_prefill) against the sequential recurrence.

The sequential checker is oracle.kda_verify / kda_commit, bit-exact with the reference's
k3_kda_step chained over t; the float64 chunked restatement oracle.kda_chunked is checked
too. The kernel reorders the sums (chunked form, fp32), so the bar is the north_star's KDA
state tolerance, rel-L2 <= 1e-4, for the state and the outputs: ragged chunks, one
position, strong and weak decay, D 32/64/128, a prompt split over two calls.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests import k3lib

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def k3():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return k3lib.load()


def inputs(seed, B, T, H, D, decay):
    rng = np.random.default_rng(seed)
    st = rng.standard_normal((B, H, D, D), dtype=np.float32) * np.float32(0.1)
    q, k, v = (rng.standard_normal((B, T, H, D), dtype=np.float32) for _ in range(3))
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    al = rng.uniform(decay[0], decay[1], (B, T, H, D)).astype(np.float32)
    be = rng.uniform(0.1, 0.9, (B, T, H)).astype(np.float32)
    return st, q, k, v, al, be


def rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("B,T,H,D,decay", [
    (2, 1, 2, 128, (0.9, 0.999)), (1, 37, 3, 128, (0.9, 0.999)), (2, 100, 2, 64, (0.3, 0.7)),
    (1, 257, 2, 128, (0.05, 0.4)), (1, 64, 4, 32, (0.995, 1.0)),
])
def test_prefill_equals_sequential(k3, B, T, H, D, decay):
    st, q, k, v, al, be = inputs(B * 1000 + T * 7 + D, B, T, H, D, decay)
    qs = np.float32(1.0) / np.sqrt(np.float32(D))
    S = torch.from_numpy(st).cuda()
    o = k3.kda_prefill(S, *(torch.from_numpy(a).cuda() for a in (q, k, v, al, be)), qs)
    torch.cuda.synchronize()
    got_o, got_s = o.cpu().numpy(), S.cpu().numpy()
    for b in range(B):
        ref_o = O.kda_verify(st[b], q[b], k[b], v[b], al[b], be[b], qs)
        ref_s = O.kda_commit(st[b], k[b], v[b], al[b], be[b], T)
        assert rel(got_o[b], ref_o) < 1e-4, b
        assert rel(got_s[b], ref_s) < 1e-4, b
        ch_o, ch_s = O.kda_chunked(st[b], q[b], k[b], v[b], al[b], be[b], qs, 32)
        assert rel(got_o[b], ch_o) < 1e-4 and rel(got_s[b], ch_s) < 1e-4, b
    assert k3.device_status(0) == 0


def test_prefill_split_and_state_only(k3):
    """A prompt read in two calls (60 then 40 positions), and without outputs, ends in the
    same state as one call."""
    st, q, k, v, al, be = inputs(7, 1, 100, 2, 128, (0.8, 0.99))
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    S1 = t(st)
    k3.kda_prefill(S1, t(q), t(k), t(v), t(al), t(be), 0.125)
    S2 = t(st)
    for a, b in ((0, 60), (60, 100)):
        k3.kda_prefill(S2, t(q[:, a:b]), t(k[:, a:b]), t(v[:, a:b]), t(al[:, a:b]), t(be[:, a:b]), 0.125,
                       outputs=False)
    torch.cuda.synchronize()
    ref = O.kda_commit(st[0], k[0], v[0], al[0], be[0], 100)
    assert rel(S1.cpu().numpy()[0], ref) < 1e-4 and rel(S2.cpu().numpy()[0], ref) < 1e-4
