"""The allocation-free router (k3gpu_router_noalloc) against the ordinary router.

Some callers cannot allocate device memory -- their own allocator has reserved the HBM,
or they run where cudaMalloc's possible device synchronisation is not allowed -- so they
cannot hand k3gpu_router its score workspace. k3gpu_router_noalloc keeps those scores in
a fixed array inside the library instead. This file checks, through the C ABI, that two
calls in a row give exactly what k3gpu_router gives on the same inputs (the same kernels
and arithmetic, so bit-identical), and that an oversize request is refused. It runs last
(file name) so that a failure here comes after every other test has run, and it passes
both alone in a fresh process and after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest

from tests import k3lib
from tests.golden import inputs as GI

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _router_pair(k3, x, W, b, topk):
    """(noalloc idx, w), (workspace idx, w) for the same inputs on the current stream."""
    T, hidden = x.shape
    n = W.shape[0]
    dx, dW, db = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (x, W, b))
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    i1 = torch.empty((T, topk), dtype=torch.int32, device="cuda")
    w1 = torch.empty((T, topk), dtype=torch.float32, device="cuda")
    st = k3.lib.k3gpu_router_noalloc(C.c_void_p(i1.data_ptr()), C.c_void_p(w1.data_ptr()),
                                     C.c_void_p(dx.data_ptr()), C.c_void_p(dW.data_ptr()),
                                     C.c_void_p(db.data_ptr()), T, hidden, n, topk, 1, 1.0, s)
    assert st == k3.K3GPU_OK, k3.lib.k3gpu_strerror(st)
    i2, w2 = k3.router(dx, dW, db, topk)
    torch.cuda.synchronize()
    return (i1.cpu().numpy(), w1.cpu().numpy()), (i2.cpu().numpy(), w2.cpu().numpy())


def test_router_noalloc_matches_workspace_router_twice():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    k3 = k3lib.load()
    # two different calls in a row: the second must not see anything the first left in
    # the shared array (benchmark config 2 router shape, then a larger batch)
    for case in (dict(name="a", seed=11, T=16, hidden=7168, n=384, topk=8, wstd=0.02, bstd=0.01),
                 dict(name="b", seed=91, T=72, hidden=7168, n=384, topk=8, wstd=0.02, bstd=0.01)):
        x, W, b = GI.router_inputs(case)
        (ia, wa), (ib, wb) = _router_pair(k3, x, W, b, case["topk"])
        np.testing.assert_array_equal(ia, ib)
        np.testing.assert_array_equal(wa.view(np.uint32), wb.view(np.uint32))
    assert k3.device_status(0) == 0


def test_router_noalloc_refuses_oversize_request():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    k3 = k3lib.load()
    n = 384
    T = 524288 // n + 1   # one token past K3GPU_ROUTER_NOALLOC_MAX_SCORES
    p = C.c_void_p(16)   # never dereferenced: the size check comes first
    st = k3.lib.k3gpu_router_noalloc(p, p, p, p, p, T, 7168, n, 8, 1, 1.0, None)
    assert st == k3.K3GPU_ECAPACITY
