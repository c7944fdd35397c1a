"""Expert-parallel MoE layer on 2 GPUs (NCCL) against the single-GPU layer.

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


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_gpus_matches_single_gpu_layer():
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_worker, args=(2, _free_port(), results), nprocs=2, join=True,
                       start_method="spawn")
    assert results["idx_local_ok"]
    assert results["rel"] < 1e-5, results["rel"]
