"""Expert-parallel MoE layer on 2 GPUs (NCCL, and the peer-memory transport) against the
single-GPU layer.

Each rank holds half of the routed experts of one bank (plus the replicated shared
expert) and verifies its own tokens; rank 0 also runs k3gpu_moe_layer over the whole bank
on every rank's tokens, and the EP outputs must match it to fp32 rounding (the EP sum over
a token's experts runs per owning rank, then across ranks). Skipped with fewer than two
GPUs.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import importlib.util
    from datetime import timedelta

    import torch.distributed as dist
    from k3lib import load
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        k3 = load()
        spec = importlib.util.spec_from_file_location("k3b200_ep", os.path.join(
            os.path.dirname(HERE), "kimi-k3-for-me_b200", "ep.py"))
        ep = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(ep)
        L, I, n, ns, topk, T = 1024, 512, 8, 1, 3, 24
        rng = np.random.default_rng(41)
        bank, lay = O.make_bank(rng, n + ns, L, I, std=0.05, w13_std=0.1)
        stride = int(lay[6])
        W = (rng.standard_normal((n, L), dtype=np.float32) * np.float32(0.02))
        bias = rng.standard_normal(n, dtype=np.float32) * np.float32(0.01)
        xs = [rng.standard_normal((T, L), dtype=np.float32) for _ in range(world)]
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        nl = n // world
        local = d(bank[rank * nl * stride:(rank + 1) * nl * stride])
        shared = d(bank[n * stride:(n + ns) * stride])
        kb_l = k3.ExpertBank(local, nl, L, I)
        kb_s = k3.ExpertBank(shared, ns, L, I)
        layer = ep.EPMoELayer.from_k3(k3, kb_l, kb_s, d(W), d(bias), n, topk, k3.ACT_SWIGLU)
        out, idx, wt = layer(d(xs[rank]))
        torch.cuda.synchronize()
        outs = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(outs, out)
        if rank == 0:
            kb = k3.ExpertBank(d(bank), n + ns, L, I)
            ref, ridx, _ = k3.moe_layer(d(np.concatenate(xs)), d(W), d(bias), kb, topk, n, ns,
                                        k3.ACT_SWIGLU)
            got = torch.cat(outs)
            results["rel"] = float((got - ref).norm() / ref.norm())
            results["idx_local_ok"] = bool(torch.equal(idx, ridx[:T]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _worker_p2p(rank, world, port, results):
    """The peer-memory transport: three steps with new tokens each (the exchange arena and
    its sequence flags are reused), a different token count on each rank."""
    import importlib.util
    from datetime import timedelta

    import torch.distributed as dist
    from k3lib import load
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    layer = None
    try:
        k3 = load()
        spec = importlib.util.spec_from_file_location("k3b200_ep", os.path.join(
            os.path.dirname(HERE), "kimi-k3-for-me_b200", "ep.py"))
        ep = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(ep)
        L, I, n, ns, topk, cap = 1024, 512, 8, 1, 3, 32
        Ts = [24, 17]
        rng = np.random.default_rng(43)
        bank, lay = O.make_bank(rng, n + ns, L, I, std=0.05, w13_std=0.1)
        stride = int(lay[6])
        W = (rng.standard_normal((n, L), dtype=np.float32) * np.float32(0.02))
        bias = rng.standard_normal(n, dtype=np.float32) * np.float32(0.01)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        nl = n // world
        kb_l = k3.ExpertBank(d(bank[rank * nl * stride:(rank + 1) * nl * stride]), nl, L, I)
        kb_s = k3.ExpertBank(d(bank[n * stride:(n + ns) * stride]), ns, L, I)
        layer = ep.P2PMoELayer(k3, kb_l, kb_s, d(W), d(bias), n, topk, k3.ACT_SWIGLU, cap)
        kb = k3.ExpertBank(d(bank), n + ns, L, I) if rank == 0 else None
        rels, idx_ok = [], True
        for step in range(3):
            xs = [rng.standard_normal((Ts[r], L), dtype=np.float32) for r in range(world)]
            out, idx, _ = layer(d(xs[rank]))
            torch.cuda.synchronize()
            outs = [torch.empty((Ts[r], L), dtype=torch.float32, device=dev) for r in range(world)]
            # gather rank 1's rows on rank 0 (ragged sizes: pad to cap)
            pad = torch.zeros((cap, L), dtype=torch.float32, device=dev)
            pad[:out.shape[0]] = out
            gath = [torch.empty_like(pad) for _ in range(world)]
            dist.all_gather(gath, pad)
            if rank == 0:
                got = torch.cat([gath[r][:Ts[r]] for r in range(world)])
                ref, ridx, _ = k3.moe_layer(d(np.concatenate(xs)), d(W), d(bias), kb, topk, n, ns, k3.ACT_SWIGLU)
                rels.append(float((got - ref).norm() / ref.norm()))
                idx_ok = idx_ok and bool(torch.equal(idx, ridx[:Ts[0]]))
        if rank == 0:
            results["rels"] = rels
            results["idx_ok"] = idx_ok
        results[f"status{rank}"] = k3.device_status(rank)
        dist.barrier()
    finally:
        if layer is not None:
            layer.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_gpus_peer_memory_transport():
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_worker_p2p, args=(2, _free_port(), results), nprocs=2, join=True,
                       start_method="spawn")
    assert results["idx_ok"]
    assert results["status0"] == 0 and results["status1"] == 0
    assert max(results["rels"]) < 1e-5, results["rels"]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_gpus_matches_single_gpu_layer():
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_worker, args=(2, _free_port(), results), nprocs=2, join=True,
                       start_method="spawn")
    assert results["idx_local_ok"]
    assert results["rel"] < 1e-5, results["rel"]



def test_ep_exchange_wait_runs_out_and_reports():
    """One GPU, a world of two: rank 0's arena and a second arena on the same GPU standing
    in for a peer that never signals. With a short wait limit, receive and combine give up
    on the silent peer: the timeout bit is set, its receive slots are all dropped, its owner
    flag is 0, and the output holds exactly rank 0's own partial rows. Every wait is
    bounded, so the kernels return; nothing else waits on them."""
    import ctypes as C

    from k3lib import load

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    k3 = load()
    lib = k3.lib
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L, K, cap, T, n_local = 64, 2, 8, 5, 4
    nbytes = lib.k3gpu_ep_arena_bytes(2, cap, L, K)
    arenas = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(2)]
    assert all(a.data_ptr() % 256 == 0 for a in arenas)
    g = k3.K3GpuEpGroup()
    g.world, g.rank, g.cap, g.L, g.K, g.n_local = 2, 0, cap, L, K, n_local
    g.arena[0], g.arena[1] = arenas[0].data_ptr(), arenas[1].data_ptr()
    torch.cuda.synchronize()
    k3.device_status(0)                                     # clear
    k3.check(lib.k3gpu_ep_set_wait_limit(2000), "k3gpu_ep_set_wait_limit")
    try:
        x = torch.randn((T, L), device=dev)
        # tokens 0, 2, 4 use an expert of rank 0 (ids 0..3); every token one of rank 1 (4..7)
        idx = torch.tensor([[1, 5], [6, 7], [0, 4], [5, 6], [3, 7]], dtype=torch.int32, device=dev)
        wt = torch.full((T, K), 0.5, device=dev)
        pos = torch.empty(2 * T, dtype=torch.int32, device=dev)
        sp = k3.stream_ptr()
        k3.check(lib.k3gpu_ep_dispatch(C.byref(g), k3.ptr(x), k3.ptr(idx), k3.ptr(wt), T, 1, k3.ptr(pos), sp),
                 "k3gpu_ep_dispatch")
        k3.check(lib.k3gpu_ep_receive(C.byref(g), 1, sp), "k3gpu_ep_receive")
        torch.cuda.synchronize()
        assert k3.device_status(0) & 8, "the receive wait on the silent peer did not run out"
        xr, ir, wr = C.c_void_p(), C.c_void_p(), C.c_void_p()
        k3.check(lib.k3gpu_ep_recv_views(C.byref(g), C.byref(xr), C.byref(ir), C.byref(wr)), "views")
        off = ir.value - arenas[0].data_ptr()
        recv_idx = arenas[0][off:off + 4 * 2 * cap * K].view(torch.int32).view(2, cap, K).cpu()
        assert torch.all(recv_idx[1] == -1), "the silent peer's receive slots were not dropped"
        assert recv_idx[0, :3].tolist() == [[1, -1], [0, -1], [3, -1]]   # tokens 0, 2, 4: local ids
        assert torch.all(recv_idx[0, 3:] == -1)
        part = torch.randn((2 * cap, L), device=dev)
        k3.check(lib.k3gpu_ep_return(C.byref(g), k3.ptr(part), 1, sp), "k3gpu_ep_return")
        out0 = torch.randn((T, L), device=dev)
        out = out0.clone()
        ok = torch.empty(2, dtype=torch.int32, device=dev)
        k3.check(lib.k3gpu_ep_combine(C.byref(g), k3.ptr(out), k3.ptr(pos), T, 1, k3.ptr(ok), sp),
                 "k3gpu_ep_combine")
        torch.cuda.synchronize()
        assert ok.tolist() == [1, 0]
        assert k3.device_status(0) & 8, "the combine wait on the silent peer did not run out"
        want = out0.clone()
        for t, p in enumerate(pos[:T].tolist()):
            if p >= 0:
                want[t] += part[p]
        assert torch.equal(out, want)
    finally:
        lib.k3gpu_ep_set_wait_limit(1 << 24)
        torch.cuda.synchronize()
        k3.device_status(0)
