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
