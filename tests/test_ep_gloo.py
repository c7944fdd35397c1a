"""Expert-parallel dispatch/combine (kimi-k3-for-me_b200/ep.py) on CPU with gloo ranks.

The expert compute is a stand-in (a different non-linear map per global expert id), so
these tests cover the host logic the GPU run shares: the send plan (rows deduplicated per
destination, local ids, dropped slots), the count and row all-to-alls, the combine, and
the shared experts -- against the single-process formula
    out[t] = sum_k wt[t,k] * f_{idx[t,k]}(x[t]) + shared(x[t]).
"""
import importlib.util
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
EP_PATH = os.path.join(os.path.dirname(HERE), "kimi-k3-for-me_b200", "ep.py")


def load_ep():
    spec = importlib.util.spec_from_file_location("k3b200_ep", EP_PATH)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def f_expert(e, z):
    return torch.tanh(z * (0.3 + 0.1 * e) + 0.01 * e)


def shared(x):
    return 0.5 * x + 0.25


def route(x, W, topk, drop):
    """Top-k of x @ W with a deterministic dropped slot: (idx int32, wt)."""
    s = torch.sigmoid(x @ W)
    wt, idx = torch.topk(s, topk, dim=1)
    idx = idx.to(torch.int32)
    if drop:
        idx[0, -1] = -1
        wt[0, -1] = 0.0
    return idx, wt / wt.sum(dim=1, keepdim=True)


def reference(x, idx, wt):
    out = shared(x).clone()
    for t in range(x.shape[0]):
        for k in range(idx.shape[1]):
            e = int(idx[t, k])
            if e >= 0:
                out[t] += wt[t, k] * f_expert(e, x[t])
    return out


def _worker(rank, world, port, n_routed, topk, T, L, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ep = load_ep()
        g = torch.Generator().manual_seed(7)
        W = torch.randn(L, n_routed, generator=g)                # replicated gate
        x = torch.randn(T + rank, L, generator=torch.Generator().manual_seed(100 + rank))
        n_local = n_routed // world

        def experts(z, idx, wt):
            out = torch.zeros_like(z)
            for r in range(z.shape[0]):
                for k in range(idx.shape[1]):
                    e = int(idx[r, k])
                    if e >= 0:
                        out[r] += wt[r, k] * f_expert(rank * n_local + e, z[r])
            return out

        layer = ep.EPMoELayer(lambda v: route(v, W, topk, drop=(rank == 0)), experts, shared,
                              n_routed, topk)
        out, idx, wt = layer(x)
        ref = reference(x, idx, wt)
        results[rank] = float((out - ref).abs().max())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,n_routed,topk", [(2, 8, 3), (2, 6, 6), (4, 8, 2)])
def test_ep_layer_matches_single_process(world, n_routed, topk):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), n_routed, topk, 5, 16, results),
                       nprocs=world, join=True, start_method="spawn")
    assert len(results) == world
    for r in range(world):
        assert results[r] < 1e-5, (r, results[r])


def test_plan_dispatch_dedups_per_destination():
    ep = load_ep()
    # 2 ranks x 4 local experts; token 0 -> experts 1, 2 (rank 0) and 5 (rank 1);
    # token 1 -> 6, 7 (rank 1) and a dropped slot; token 2 -> 0, 3, 4
    idx = torch.tensor([[1, 2, 5], [6, -1, 7], [0, 3, 4]], dtype=torch.int32)
    wt = torch.tensor([[0.5, 0.3, 0.2], [0.6, 0.0, 0.4], [0.1, 0.2, 0.7]])
    tok, counts, midx, mwt = ep.plan_dispatch(idx, wt, 4, 2)
    assert counts.tolist() == [2, 3]                 # rank 0: tokens 0, 2; rank 1: 0, 1, 2
    assert tok.tolist() == [0, 2, 0, 1, 2]
    assert midx.tolist() == [[1, 2, -1], [0, 3, -1], [-1, -1, 1], [2, -1, 3], [-1, -1, 0]]
    assert torch.equal(mwt, torch.tensor([[0.5, 0.3, 0.0], [0.1, 0.2, 0.0], [0.0, 0.0, 0.2],
                                          [0.6, 0.0, 0.4], [0.0, 0.0, 0.7]]))


def test_pack_roundtrip_keeps_int_bits():
    ep = load_ep()
    rows = torch.randn(3, 8)
    midx = torch.tensor([[5, -1], [0, 2147483647], [-2147483648, 7]], dtype=torch.int32)
    mwt = torch.rand(3, 2)
    r, i, w = ep._unpack(ep._pack(rows, midx, mwt), 8, 2)
    assert torch.equal(r, rows) and torch.equal(i, midx) and torch.equal(w, mwt)
