"""RMSNorm and AttnRes kernels (k3gpu_rmsnorm, k3gpu_attn_res) against the oracle.

The oracle restates k3_rmsnorm (src/core/k3_ops.c:132-140) and k3_attn_res (:1722-1753)
and is pinned to the reference's golden vectors (tests/test_oracle_golden.py). The device
kernels take their double sums as block reductions, so they agree to an ulp of float:
the tolerance is 2e-6 relative to the output's scale.
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


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def close(got, ref, rel=2e-6):
    scale = max(float(np.abs(ref).max()), 1e-30)
    np.testing.assert_allclose(got, ref, atol=rel * scale, rtol=0)


@pytest.mark.parametrize("n", [512, 7168, 100])
def test_rmsnorm_rows_vs_oracle(k3, n):
    rng = np.random.default_rng(n)
    T = 9
    x = rng.standard_normal((T, n), dtype=np.float32) * np.float32(3.0)
    x[3] = 0.0                                   # an all-zero row: inv = 1/sqrt(eps)
    w = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    y = k3.rmsnorm(dev(x), dev(w), 1e-5).cpu().numpy()
    ref = O.rmsnorm(x, w, 1e-5)
    close(y, ref)
    # in place, as the reference allows
    xd = dev(x)
    k3.rmsnorm(xd, dev(w), 1e-5, out=xd)
    close(xd.cpu().numpy(), ref)


@pytest.mark.parametrize("n,maxb", [(512, 4), (7168, 4), (7168, 48), (510, 12), (8192, 6), (3000, 9)])
def test_attn_res_source_stacks_vs_oracle(k3, n, maxb):
    """Up to 49 sources (a 93-layer stack's snapshots); rows held in registers (the
    single-pass kernel, widths up to 7168 with ragged last columns at 3000) and the two-pass
    kernel (8192 wide, and a width that is not a multiple of four: scalar loads)."""
    rng = np.random.default_rng(7 + n + maxb)
    T = 6
    nb = np.array([0, 1, 2, 3, maxb, maxb // 2], np.int32)
    br = rng.standard_normal((T, maxb, n), dtype=np.float32)
    cur = rng.standard_normal((T, n), dtype=np.float32) * np.float32(2.0)
    fold = (rng.standard_normal(n) * 0.05).astype(np.float32)
    got = k3.attn_res(dev(br), dev(cur), dev(fold), dev(nb), 1e-5).cpu().numpy()
    for t in range(T):
        src = np.ascontiguousarray(np.concatenate([br[t, :nb[t]], cur[t:t + 1]]))
        ref = np.empty(n, np.float32)
        O.orc().orc_attn_res(ref, src, fold, src.shape[0], n, 1e-5)
        close(got[t], ref)


@pytest.mark.parametrize("n", [7168, 8192])
def test_attn_res_spread_scores_vs_oracle(k3, n):
    """Sources of very different scales and a large fold: the scores span tens of units and
    the maximum rises at several sources, so the single-pass kernel rescales its sums
    (7168) -- held to the same bar as the two-pass kernel (8192)."""
    rng = np.random.default_rng(11 + n)
    T, maxb = 8, 30
    nb = np.array([30, 29, 17, 5, 1, 0, 30, 12], np.int32)
    scale = rng.uniform(0.1, 10.0, (T, maxb, 1)).astype(np.float32)
    br = (rng.standard_normal((T, maxb, n), dtype=np.float32) * scale).astype(np.float32)
    cur = rng.standard_normal((T, n), dtype=np.float32)
    fold = rng.standard_normal(n).astype(np.float32) * np.float32(0.3)
    got = k3.attn_res(dev(br), dev(cur), dev(fold), dev(nb), 1e-5).cpu().numpy()
    for t in range(T):
        src = np.ascontiguousarray(np.concatenate([br[t, :nb[t]], cur[t:t + 1]]))
        ref = np.empty(n, np.float32)
        O.orc().orc_attn_res(ref, src, fold, src.shape[0], n, 1e-5)
        close(got[t], ref)


def test_attn_res_no_snapshots_and_bad_count(k3):
    """maxb = 0 (no block_residual): the output is cur itself (one source, p = 1).
    A count past maxb is clamped and flagged in the device status word."""
    rng = np.random.default_rng(3)
    T, n = 3, 256
    cur = rng.standard_normal((T, n), dtype=np.float32)
    fold = rng.standard_normal(n).astype(np.float32)
    got = k3.attn_res(None, dev(cur), dev(fold), dev(np.zeros(T, np.int32)), 1e-5).cpu().numpy()
    np.testing.assert_array_equal(got, cur)
    k3.device_status()                           # clear
    br = rng.standard_normal((T, 2, n), dtype=np.float32)
    got = k3.attn_res(dev(br), dev(cur), dev(fold), dev(np.array([0, 5, 2], np.int32)), 1e-5).cpu().numpy()
    assert k3.device_status() & 2
    src = np.ascontiguousarray(np.concatenate([br[1, :2], cur[1:2]]))
    ref = np.empty(n, np.float32)
    O.orc().orc_attn_res(ref, src, fold, 3, n, 1e-5)
    close(got[1], ref)


def test_norm_argument_checks(k3):
    x = torch.zeros((2, 8), device="cuda")
    assert k3.lib.k3gpu_rmsnorm(None, k3.ptr(x), k3.ptr(x[0]), 2, 8, 1e-5, None) == k3.K3GPU_EINVAL
    assert k3.lib.k3gpu_attn_res(k3.ptr(x), None, k3.ptr(x), k3.ptr(x[0]), None, 2, 0, 8, 1e-5,
                                 None) == k3.K3GPU_EINVAL
    nbv = torch.zeros(2, dtype=torch.int32, device="cuda")
    assert k3.lib.k3gpu_attn_res(k3.ptr(x), k3.ptr(x), k3.ptr(x), k3.ptr(x[0]), k3.ptr(nbv), 2, 300,
                                 8, 1e-5, None) == k3.K3GPU_ECAPACITY
