"""The tcgen05 bf16 trunk matmul (k3gpu_matmul_bf16_batch) against the reference.

Reference: k3_matmul_bf16_batch_ld (src/core/k3_ops.c:953), run from oracle/_ref when it
was built, else the oracle's double matmul (they agree exactly on these inputs, see
test_oracle_golden). The device path takes the activations as two bf16 pieces and sums
in fp32, so the bar is relative L2 <= 5e-5 and max-abs <= 1e-4 of the output scale --
inside the sweep's logits tolerance (rel-L2 1e-3) by a wide margin. bf16-exact
activations take one piece (products exact), same bar.
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


@pytest.fixture(scope="module")
def k3():
    return load()


def bf16_bits(a):
    """Round fp32 to bf16 (nearest even) and return the uint16 bit patterns."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def reference(X, Wb):
    r = O.matmul_bf16_ref(X, Wb)
    return r if r is not None else O.matmul_d(X, O.bf16_bits_to_f32(Wb))


def check(got, ref):
    scale = max(float(np.abs(ref).max()), 1e-30)
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
    assert rel <= 5e-5, rel
    assert float(np.abs(got - ref).max()) <= 1e-4 * scale


def wdev(Wb):
    return torch.from_numpy(Wb.view(np.int16)).cuda()


# the last three: a tree batch's position tiles (1024 = 8 tiles), two launches with a ragged
# second (2100 = 2048 + 52), and K splits over many position tiles of a narrow output
@pytest.mark.parametrize("T,n_in,n_out", [(72, 7168, 1024), (5, 512, 300), (200, 1024, 256),
                                          (300, 256, 130), (9, 520, 64), (1, 2048, 7168),
                                          (1024, 1024, 512), (2100, 256, 130), (1000, 7168, 64)])
def test_matmul_bf16_fp32_activations(k3, T, n_in, n_out):
    rng = np.random.default_rng(T * 131 + n_in + n_out)
    X = rng.standard_normal((T, n_in), dtype=np.float32)
    Wb = bf16_bits(rng.standard_normal((n_out, n_in), dtype=np.float32) * np.float32(0.03))
    got = k3.matmul_bf16(torch.from_numpy(X).cuda(), wdev(Wb)).cpu().numpy()
    check(got, reference(X, Wb))


def test_matmul_bf16_exact_activations_and_strides(k3):
    """bf16-valued X (one piece), written into a column slice of a wider Y with a row
    stride, from a row-strided X: the _ld form."""
    rng = np.random.default_rng(5)
    T, n_in, n_out = 40, 1536, 512
    Xw = bf16_bits(rng.standard_normal((T, n_in + 64), dtype=np.float32))
    Xw = O.bf16_bits_to_f32(Xw)
    Wb = bf16_bits(rng.standard_normal((n_out, n_in), dtype=np.float32) * np.float32(0.05))
    Yw = torch.full((T, 2 * n_out), 7.0, device="cuda")
    Xd = torch.from_numpy(np.ascontiguousarray(Xw)).cuda()
    k3.matmul_bf16(Xd[:, :n_in], wdev(Wb), out=Yw[:, n_out:])
    got = Yw.cpu().numpy()
    assert np.all(got[:, :n_out] == 7.0)                      # the other half untouched
    check(got[:, n_out:], reference(np.ascontiguousarray(Xw[:, :n_in]), Wb))


def test_matmul_bf16_argument_checks(k3):
    X = torch.zeros((2, 12), device="cuda")
    W = torch.zeros((4, 12), dtype=torch.int16, device="cuda")
    Y = torch.zeros((2, 4), device="cuda")
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    lib = k3.lib
    # in % 8 != 0
    assert lib.k3gpu_matmul_bf16_batch(Y.data_ptr(), 4, X.data_ptr(), 12, W.data_ptr(), 12, 4, 2,
                                       ws.data_ptr(), ws.numel(), None) == k3.K3GPU_EINVAL
    # ldy < out
    assert lib.k3gpu_matmul_bf16_batch(Y.data_ptr(), 3, X.data_ptr(), 12, W.data_ptr(), 8, 4, 2,
                                       ws.data_ptr(), ws.numel(), None) == k3.K3GPU_EINVAL
    # workspace too small
    assert lib.k3gpu_matmul_bf16_batch(Y.data_ptr(), 4, X.data_ptr(), 12, W.data_ptr(), 8, 4, 2,
                                       ws.data_ptr(), 16, None) == k3.K3GPU_ECAPACITY


def first_argmax(logits):
    """argmax_ (src/cli/k3_run.c:138-139) per row: best = 0, then every later value that
    compares greater -- so the first maximum, NaN never chosen, and 0 when row[0] is NaN."""
    out = np.zeros(logits.shape[0], np.int32)
    for t, row in enumerate(logits):
        if not (np.isnan(row[0]) or np.isnan(row).all()):
            out[t] = int(np.nanargmax(row))   # the first occurrence of the non-NaN maximum
    return out


@pytest.mark.parametrize("T,vocab", [(37, 1000), (130, 4096)])
def test_lm_head_argmax_exact_ties_and_nans(k3, T, vocab):
    """The lm_head fused with the argmax on integer-valued inputs, whose logits are exact
    in any summation order: the first maximum wins on ties inside a 128-row block and
    across blocks, NaN logits are never chosen, and a NaN at id 0 gives 0 -- as argmax_
    finds them on the written logits. A partial last row block (vocab % 128 != 0) too."""
    rng = np.random.default_rng(T + vocab)
    n_in = 512
    X = rng.integers(-2, 3, (T, n_in)).astype(np.float32)
    Wf = rng.integers(-3, 4, (vocab, n_in)).astype(np.float32)
    Wf[700 % vocab] = Wf[5] = 3.0                      # the largest rows, tied, in two blocks
    Wf[9] = Wf[5]                                      # and inside block 0
    X[3] = np.nan                                      # a position whose logits are all NaN
    X[4, :] = 0.0                                      # a position whose logits all tie at 0
    Wb = bf16_bits(Wf)
    logits = (X.astype(np.float64) @ Wf.T.astype(np.float64)).astype(np.float32)
    want = first_argmax(logits)
    got = k3.lm_head_argmax(torch.from_numpy(X).cuda(), torch.from_numpy(Wb.view(np.int16)).cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, want)
    # against the written logits' argmax, through the unfused matmul
    Y = k3.matmul_bf16(torch.from_numpy(X).cuda(), torch.from_numpy(Wb.view(np.int16)).cuda())
    np.testing.assert_array_equal(got, k3.argmax(Y).cpu().numpy())
    # a NaN at id 0 alone: every position gives 0
    Wf0 = Wf.copy()
    Wf0[0, 7] = np.nan
    got0 = k3.lm_head_argmax(torch.from_numpy(X).cuda(), torch.from_numpy(bf16_bits(Wf0).view(np.int16)).cuda())
    assert (got0.cpu().numpy() == 0).all()
    assert k3.device_status(0) == 0


def test_lm_head_argmax_random_matches_written_logits(k3):
    """Random fp32 activations (two bf16 pieces) over a config-4-sized vocabulary slice: the
    fused argmax equals the argmax of the unfused matmul's logits wherever the two largest
    logits are not within the matmuls' rounding of each other."""
    rng = np.random.default_rng(77)
    T, n_in, vocab = 72, 7168, 16384
    X = rng.standard_normal((T, n_in)).astype(np.float32)
    Wb = bf16_bits(rng.standard_normal((vocab, n_in)).astype(np.float32) * np.float32(0.02))
    Wd = torch.from_numpy(Wb.view(np.int16)).cuda()
    got = k3.lm_head_argmax(torch.from_numpy(X).cuda(), Wd).cpu().numpy()
    Y = k3.matmul_bf16(torch.from_numpy(X).cuda(), Wd).cpu().numpy()
    want = first_argmax(Y)
    top2 = np.sort(Y, axis=1)[:, -2:]
    close = (top2[:, 1] - top2[:, 0]) <= 1e-4 * np.abs(top2[:, 1])
    assert ((got == want) | close).all()
    assert (got == want).mean() > 0.95
