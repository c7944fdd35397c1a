#!/usr/bin/env python3
"""Benchmark: speculative verification on the K3-shaped 8-layer slice (benchmark config 4).

A step is one verify sweep of B = 16 sequences, each scoring a 64-node draft tree
(branching 4, depth 4) against a 32,768-position MLA cache, through the library's C ABI:
embed -> 6 KDA + 2 MLA decoder layers (each with a 384-expert top-8 + shared MXFP4 MoE,
d_model 7168, FFN 2048 SwiGLU) -> final norm -> lm_head (vocab 163,840) -> per-node argmax
-> the greedy tree walk on the device -> the commit (KDA log replay along the accepted
path, MLA rows gathered, cached advanced). Weights, cache and drafts are synthetic and
seeded; each tree's most probable branch carries the model's own greedy continuation, so
every step accepts its 4 drafts plus the bonus id (the reference's GATE 4 forcing).

value  accepted ids per second over all sequences (device-timed, CUDA events)
e2e    the same through the public calls with the draft ids copied from pinned host memory
       and the accepted ids read back inside the timed region
rows   config 2 (one MoE layer at every M = B(1+k)), config 3 (KDA verify / commit, the
       chunked prefill), the MLA attention, trunk matmuls, lm_head, router and accept,
       each with its roofline fraction and, where the reference has the kernel, its CPU
       baseline; integer outputs carry FNV-1a fingerprints
N > 1  expert parallel: every layer's 384 routed experts split 384/N per GPU, token rows
       exchanged through peer memory inside the model's MoE steps; each rank verifies its
       own 16 sequences (weak scaling); the max over ranks of the device time.

--impl reference times the reference engine's own C kernels (compiled from its sources
into oracle/_ref) on the host cores for the same slice, one sequence's chain at a time.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L_DIM, I_DIM, N_ROUTED, N_SHARED, TOPK = 7168, 2048, 384, 1, 8
METRIC = "accepted tok/s (spec decode) & verify-step ms; expert-GEMM HBM GB/s vs peak"


def load_pkg():
    import importlib.util
    spec = importlib.util.spec_from_file_location("k3b200", os.path.join(ROOT, "kimi-k3-for-me_b200", "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["k3b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks_tensor():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d.get("bf16_tflops", 1590.0))
    return 1590.0


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# --------------------------------------------------------------------- workload ----
def bank_layout(L, I):
    pw, sw, pd, sd = I * (L // 2), I * (L // 32), L * (I // 2), L * (I // 32)
    offs = dict(p1=0, s1=pw, p2=pw + sw, s2=pw + sw + pd, p3=pw + sw + pd + sd,
                s3=pw + sw + pd + sd + pw)
    run = pw + sw + pd + sd + pw + sw
    # the library's stride (k3gpu_bank_layout): run rounded up to lcm(L/2, I/2, 256)
    import math
    q = math.lcm(256, L // 2, I // 2)
    return offs, (run + q - 1) // q * q


def quant_mxfp4_torch(w):
    """MXFP4 by the reference generator's rule (tools/make_tiny_checkpoint.py:88-138):
    per 32 elements scale 2^(floor(log2 amax) - 2), nearest E2M1 magnitude (lower level
    on exact ties), low nibble = even element. Returns (packed u8 [R][C/2], scales u8)."""
    import torch
    R, Cc = w.shape
    g = w.view(R, Cc // 32, 32)
    amax = g.abs().amax(dim=2).clamp_min(1e-30)
    ex = (torch.floor(torch.log2(amax)) - 2).clamp(-127, 127)
    scales = (ex + 127).to(torch.uint8)
    xq = g / torch.exp2(ex).unsqueeze(2)
    mids = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], device=w.device)
    mag = torch.bucketize(xq.abs().contiguous(), mids, right=False).to(torch.uint8)
    nib = mag | ((xq < 0).to(torch.uint8) << 3)
    nib = nib.view(R, Cc)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).contiguous()
    return packed, scales.view(R, Cc // 32).contiguous()


def make_bank_device(n_experts, L, I, seed, device, chunk=16):
    """A device MXFP4 bank in the library's run layout, w1/w2/w3 ~ N(0, 0.02) quantised by
    the reference generator's rule, drawn `chunk` experts at a time (one torch generator
    seeded with `seed`: w1 of the chunk, then w2, then w3)."""
    import torch
    offs, stride = bank_layout(L, I)
    bank = torch.zeros(n_experts * stride, dtype=torch.uint8, device=device)
    view = bank.view(n_experts, stride)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    for e0 in range(0, n_experts, chunk):
        n = min(chunk, n_experts - e0)
        for (po, so, rows, cols) in ((offs["p1"], offs["s1"], I, L), (offs["p2"], offs["s2"], L, I),
                                     (offs["p3"], offs["s3"], I, L)):
            w = torch.randn((n * rows, cols), generator=gen, device=device) * 0.02
            p, sc = quant_mxfp4_torch(w)
            view[e0:e0 + n, po:po + rows * cols // 2] = p.view(n, -1)
            view[e0:e0 + n, so:so + rows * cols // 32] = sc.view(n, -1)
            del w, p, sc
    return bank, offs, stride


FP32_ACTS = False   # --fp32-acts: full fp32 activations instead of bf16 ones


def make_inputs(M, seed, device):
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    x = torch.randn((M, L_DIM), generator=gen, device=device)
    if not FP32_ACTS:
        x = x.to(torch.bfloat16).float()
    gate = torch.randn((N_ROUTED, L_DIM), generator=gen, device=device) * 0.02
    bias = torch.randn((N_ROUTED,), generator=gen, device=device) * 0.01
    return x.contiguous(), gate.contiguous(), bias.contiguous()


# --------------------------------------------------------- config 4: the model slice ----
# an 8-layer K3-shaped slice (6 KDA + 2 MLA in the 3:1 pattern, d_model
# 7168, the config-2 MoE in every layer: 384 routed experts top-8 + 1 shared, FFN 2048
# SwiGLU, MXFP4), MLA 64 heads / q_lora 1536 / kv_lora 512 / rope 64, KDA 32 heads x 128
# (config 3), vocab 163840, random init; a 64-node draft tree (branching 4, depth 4) over a
# 32k-position random-filled compressed cache, B sequences, greedy acceptance.
C4 = {"hidden_size": 7168, "num_hidden_layers": 8, "vocab_size": 163840, "rms_norm_eps": 1e-5,
      "kda_num_heads": 32, "kda_head_dim": 128, "short_conv_kernel_size": 4, "gate_lower_bound": -5.0,
      "num_attention_heads": 64, "q_lora_rank": 1536, "kv_lora_rank": 512, "qk_nope_head_dim": 128,
      "qk_rope_head_dim": 64, "v_head_dim": 128, "mla_use_output_gate": True, "num_experts": 384,
      "num_experts_per_token": 8, "num_shared_experts": 1, "routed_expert_hidden_size": 7168,
      "moe_intermediate_size": 2048, "routed_scaling_factor": 1.0, "moe_renormalize": True,
      "latent_moe_use_norm": False, "first_k_dense_replace": 0, "intermediate_size": 2048,
      "attn_res_block_size": 2, "situ_beta": 4.0, "situ_linear_beta": 25.0, "full_attn_layers": [4, 8],
      "moe_form": "plain", "act": "swiglu"}
C4_CTX = 32768
C4_TREE, C4_BRANCH, C4_DEPTH = 64, 4, 4


def tree_topology(nodes=C4_TREE, branch=C4_BRANCH, depth=C4_DEPTH, weights=(0.5, 0.25, 0.15, 0.10)):
    """A draft tree's shape as a suffix drafter grows it: best-first by path probability
    (child c of a node carries weights[c] of its parent's), at most `branch` children and
    `depth` levels below the root, `nodes` nodes, parents before children. Returns
    (parent, chain) where chain is the most probable root-to-depth path (node indices)."""
    import heapq
    parent, prob, dep = [-1], [1.0], [0]
    heap, tick = [], 0
    for c in range(branch):
        heapq.heappush(heap, (-weights[c], tick, 0, c))
        tick += 1
    first_child = {}
    while len(parent) < nodes and heap:
        negp, _, par, c = heapq.heappop(heap)
        i = len(parent)
        parent.append(par)
        prob.append(-negp)
        dep.append(dep[par] + 1)
        if c == 0:
            first_child[par] = i
        if dep[i] < depth:
            for cc in range(branch):
                heapq.heappush(heap, (negp * weights[cc], tick, i, cc))
                tick += 1
    chain, n = [0], 0
    while n in first_child:
        n = first_child[n]
        chain.append(n)
    return parent, chain


def make_c4_model(k3, dev, B, seed, kv_cap, max_T=C4_TREE, rank=0, world=1, cfg=None, rank_banks=False,
                  gather_ranks=0):
    """The config-4 slice on the device with random weights: bf16 projections N(0, 0.02),
    unit norms, AttnRes folds N(0, 0.02), router N(0, 0.02) with bias N(0, 0.01), the KDA
    decay parameters of the reference's tiny-model recipe, MXFP4 experts N(0, 0.02).
    world > 1: this rank keeps routed experts rank * 384/world .. of every layer's bank (the
    bank drawn whole, then sliced, so the experts are those of the one-GPU model) and the
    shared expert as a bank of its own; returns (model, shared banks), else (model, None)."""
    # cfg: another configuration of the same layer shapes (config 5's deep stack); rank_banks:
    # each rank draws its own routed experts (rank-seeded) and every rank the same shared
    # expert, instead of slicing one full bank (a 93-layer stack's full banks fit no GPU);
    # gather_ranks = G (with world 1): one GPU holds all G ranks' draws as one bank, the
    # unsharded twin of a G-rank model
    import torch
    c = cfg if cfg is not None else C4
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    E, V = c["hidden_size"], c["vocab_size"]
    H, D, K = c["kda_num_heads"], c["kda_head_dim"], c["short_conv_kernel_size"]
    P = H * D
    Hm, ql, kvl = c["num_attention_heads"], c["q_lora_rank"], c["kv_lora_rank"]
    nope, rope, vh = c["qk_nope_head_dim"], c["qk_rope_head_dim"], c["v_head_dim"]
    n, I_ = c["num_experts"], c["moe_intermediate_size"]

    def bf(*shape):
        return (torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16).view(torch.int16)

    def f32(*shape, std=0.02):
        return torch.randn(shape, generator=g, device=dev) * std

    def ones(k):
        return torch.ones(k, device=dev)

    layers, banks, shared = [], [], []
    for L in range(c["num_hidden_layers"]):
        mla = (L + 1) in c["full_attn_layers"]
        d = {"kind": "mla" if mla else "kda", "in_norm": ones(E), "post_norm": ones(E),
             "attn_res_fold": f32(E), "mlp_res_fold": f32(E), "gate_W": f32(n, E),
             "gate_bias": f32(n, std=0.01)}
        if mla:
            d.update(q_a=bf(ql, E), q_a_norm=ones(ql), q_b=bf(Hm * (nope + rope), ql), kv_a=bf(kvl + rope, E),
                     kv_a_norm=ones(kvl), kv_b=f32(Hm * (nope + vh), kvl), o=bf(E, Hm * vh), g=bf(Hm * vh, E))
        else:
            d.update(q=bf(P, E), k=bf(P, E), v=bf(P, E), g=bf(P, E), o=bf(E, P), f_a=bf(D, E), f_b=bf(P, D),
                     b=bf(H, E), q_conv=f32(P, K, std=0.4), k_conv=f32(P, K, std=0.4), v_conv=f32(P, K, std=0.4),
                     A_log=torch.linspace(-0.4, 1.2, H, device=dev), dt_bias=f32(P, std=0.5), o_norm=ones(D))
        layers.append(d)
        ns = c["num_shared_experts"]
        if gather_ranks:
            nl = n // gather_ranks
            stride = k3.ExpertBank.layout(E, I_).stride
            bank = torch.empty((n + ns) * stride, dtype=torch.uint8, device=dev)
            view = bank.view(n + ns, stride)
            for r in range(gather_ranks):
                view[r * nl:(r + 1) * nl] = make_bank_device(nl, E, I_, seed + 1000 + L + 7919 * r, dev)[0].view(nl, stride)
            view[n:n + ns] = make_bank_device(ns, E, I_, seed + 500000 + L, dev)[0].view(ns, stride)
            kb = k3.ExpertBank(bank, n + ns, E, I_)
            kb.scan()
            banks.append(kb)
            continue
        if rank_banks:
            nl = n // world
            kb = k3.ExpertBank(make_bank_device(nl + (ns if world == 1 else 0), E, I_, seed + 1000 + L + 7919 * rank,
                                                dev)[0], nl + (ns if world == 1 else 0), E, I_)
            if world > 1:
                sb = k3.ExpertBank(make_bank_device(ns, E, I_, seed + 500000 + L, dev)[0], ns, E, I_)
                sb.scan()
                shared.append(sb)
            kb.scan()
            banks.append(kb)
            continue
        bank, _, stride = make_bank_device(n + ns, E, I_, seed + 1000 + L, dev)
        if world > 1:
            nl = n // world
            view = bank.view(n + ns, stride)
            kb = k3.ExpertBank(view[rank * nl:(rank + 1) * nl].reshape(-1).clone(), nl, E, I_)
            sb = k3.ExpertBank(view[n:n + ns].reshape(-1).clone(), ns, E, I_)
            sb.scan()
            shared.append(sb)
            del view, bank
        else:
            kb = k3.ExpertBank(bank, n + ns, E, I_)
        kb.scan()
        banks.append(kb)
    top = {"embed": bf(V, E), "lm_head": bf(V, E), "norm": ones(E), "out_res_fold": f32(E)}
    torch.cuda.empty_cache()   # the bank draws' temporaries, before the model's one large arena
    model = k3.Model(dict(c), layers, top, banks, B=B, max_T=max_T, kv_cap=kv_cap, device=dev)
    return model, (shared if world > 1 else None)


def c4_fill_state(model, seed, ctx):
    """A long conversation's state: KDA states N(0, 0.1) (config 3), ShortConv histories
    N(0, 1), ctx random bf16 N(0, 1) cache rows per sequence in every MLA layer."""
    import torch
    g = torch.Generator(device=model.device)
    g.manual_seed(seed)
    for L in range(model.cfg["num_hidden_layers"]):
        if (L + 1) in model.cfg["full_attn_layers"]:
            lat, rope = model.mla_cache(L)
            lat[:, :ctx].copy_(torch.randn(lat[:, :ctx].shape, generator=g, device=model.device)
                               .to(torch.bfloat16).view(torch.int16))
            rope[:, :ctx].copy_(torch.randn(rope[:, :ctx].shape, generator=g, device=model.device)
                                .to(torch.bfloat16).view(torch.int16))
        else:
            st, hi = model.kda_state(L)
            st.copy_(torch.randn(st.shape, generator=g, device=model.device) * 0.1)
            hi.copy_(torch.randn(hi.shape, generator=g, device=model.device))
    model.set_cached([ctx] * model.B)


def c4_snapshot(model, host=False):
    """The KDA states and histories of every layer (host=True: in pinned host memory, for a
    stack whose states would not fit twice on the device)."""
    snap = []
    for L in range(model.cfg["num_hidden_layers"]):
        if (L + 1) not in model.cfg["full_attn_layers"]:
            st, hi = model.kda_state(L)
            if host:
                snap.append((st.cpu().pin_memory(), hi.cpu().pin_memory()))
            else:
                snap.append((st.clone(), hi.clone()))
    return snap


def c4_restore(model, snap, ctx):
    i = 0
    for L in range(model.cfg["num_hidden_layers"]):
        if (L + 1) not in model.cfg["full_attn_layers"]:
            st, hi = model.kda_state(L)
            st.copy_(snap[i][0])
            hi.copy_(snap[i][1])
            i += 1
    model.set_cached([ctx] * model.B)


def c4_trees(cont, parent, chain, steps, V, seed):
    """Per step and sequence the tree's ids: node 0 the pending id, the most probable branch
    the model's own next ids (cont, from an untimed serial run), every other node a random id
    that differs from its siblings on the branch -- the reference's GATE-4 way of forcing
    drafts (tests/unit/k3_model.c:359-462), since a random-weight model gives an n-gram
    drafter nothing to match. Assumes full acceptance: step s starts at cont[s*(depth+1)-1]."""
    rng = np.random.default_rng(seed)
    B = len(cont)
    T = len(parent)
    depth = len(chain) - 1
    tok = rng.integers(0, V, size=(steps, B, T)).astype(np.int32)
    on_chain = {node: j for j, node in enumerate(chain)}
    for s in range(steps):
        base = s * (depth + 1)
        for b in range(B):
            for j, node in enumerate(chain):
                tok[s, b, node] = cont[b][base + j]
            for i in range(1, T):
                p = parent[i]
                if p in on_chain and i not in on_chain:
                    nxt = on_chain[p] + 1
                    if nxt < len(chain) and tok[s, b, i] == tok[s, b, chain[nxt]]:
                        tok[s, b, i] = (tok[s, b, i] + 1) % V
    return tok


def run_c4(args, k3, dev, local, rank=0, world=1):
    """The headline: tree verification steps on the config-4 slice at B sequences per GPU. A
    step is one verify sweep of every sequence's 64-node tree through the 8 layers and the
    lm_head fused with the argmax (k3gpu_model_verify_greedy), the on-device greedy tree walk
    (k3gpu_accept_tree_greedy on those argmaxes),
    the read of the accepted paths and the commit (k3gpu_model_commit: KDA log replay, MLA
    rows gathered, cached advanced). Accepted tok/s counts every id a step emits (accepted
    drafts plus the bonus id), over all sequences of all ranks. world > 1: the same slice
    with every layer's 384 routed experts split 384/world per GPU (config 5's sharding), the
    token rows exchanged through peer memory inside the model's MoE steps
    (k3gpu_moe_layer_ep); each rank verifies its own B sequences (weak scaling), times are
    the max over ranks, and one sweep is checked against the unsharded model on rank 0."""
    import torch
    dist = None
    if world > 1:
        import torch.distributed as dist
    B, steps, warm = args.c4_B, args.steps, args.warmup
    kv_cap = C4_CTX + (steps + warm + 2) * (C4_DEPTH + 1) + C4_TREE + 8
    t_build = time.perf_counter()
    model, shared = make_c4_model(k3, dev, B, args.seed, kv_cap, rank=rank, world=world)
    exchange = None
    if world > 1:
        exchange = load_ep().EpExchange(k3, B * C4_TREE, C4["hidden_size"], C4["num_experts_per_token"],
                                        C4["num_experts"] // world)
        model.set_ep(exchange, shared)
    build_s = time.perf_counter() - t_build
    parent, chain = tree_topology()
    parent_dev = torch.tensor(parent, dtype=torch.int32, device=dev)
    V = C4["vocab_size"]
    seed_r = args.seed + 7919 * rank          # this rank's own sequences
    c4_fill_state(model, seed_r + 1, C4_CTX)
    snap = c4_snapshot(model)
    # the model's own greedy continuation from a random pending id (untimed, one position per
    # sweep), so the trees' most probable branch can carry it
    depth = len(chain) - 1
    n_cont = (steps + warm + 2) * (depth + 1) + 1
    rng = np.random.default_rng(seed_r + 2)
    x0 = torch.tensor(rng.integers(0, V, size=(B, 1)), dtype=torch.int32, device=dev)
    x = x0
    cont = [[int(x[b, 0])] for b in range(B)]
    for _ in range(n_cont):
        arg, _ = model.verify(x, logits=False)
        model.commit([1] * B)
        x = arg[:, :1].contiguous()
        for b in range(B):
            cont[b].append(int(x[b, 0]))
    c4_restore(model, snap, C4_CTX)
    tok = c4_trees(cont, parent, chain, warm + steps, V, seed_r + 3)
    tok_dev = torch.from_numpy(tok).to(dev)
    stream = torch.cuda.current_stream()
    n_path_host = torch.empty((B,), dtype=torch.int32).pin_memory()
    path_host = torch.empty((B, C4_TREE), dtype=torch.int32).pin_memory()

    def step(s, ids):
        arg, _ = model.verify(ids, parent=parent, logits=False)   # lm_head fused with the argmax
        emit, n_emit, path, _ = k3.accept_tree_greedy(None, ids, parent_dev, arg=arg)
        n_path_host.copy_(n_emit, non_blocking=True)
        path_host.copy_(path, non_blocking=True)
        stream.synchronize()
        keep = n_path_host.tolist()
        model.commit(keep, path_host.tolist())
        return sum(keep), emit

    def sync_all():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def max_over_ranks(v):
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v):
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        return float(t.item())

    for s in range(warm):
        step(s, tok_dev[s])
    if args.profile_c4:   # one step inside an NVTX range, for an ncu launch list
        sync_all()
        torch.cuda.nvtx.range_push("c4_step")
        step(warm, tok_dev[warm])
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        if exchange:
            exchange.close()
        model.close()
        return None
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    accepted = 0
    sync_all()
    l0 = k3.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(warm, warm + steps):
        a, _ = step(s, tok_dev[s])
        accepted += a
    e1.record(stream)
    sync_all()
    launches = k3.launch_count() - l0
    dev_ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    accepted = sum_over_ranks(accepted)
    status = int(max_over_ranks(k3.device_status(dev.index)))
    owners_ok = min(model.ep_owners_ok()) if exchange else 1
    owners_ok = -max_over_ranks(-owners_ok)

    # end to end through the public calls with host buffers: each step's tree ids from pinned
    # host memory, the emitted ids and their count back to the host
    c4_restore(model, snap, C4_CTX)
    tok_host = torch.from_numpy(tok).pin_memory()
    ids_dev = torch.empty((B, C4_TREE), dtype=torch.int32, device=dev)
    emit_host = torch.empty((B, C4_TREE), dtype=torch.int32).pin_memory()
    for s in range(warm):
        ids_dev.copy_(tok_host[s], non_blocking=True)
        step(s, ids_dev)
    acc_e2e = 0
    sync_all()
    e0.record(stream)
    for s in range(warm, warm + steps):
        ids_dev.copy_(tok_host[s], non_blocking=True)
        a, emit = step(s, ids_dev)
        emit_host.copy_(emit, non_blocking=True)
        acc_e2e += a
    e1.record(stream)
    sync_all()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    acc_e2e = sum_over_ranks(acc_e2e)
    clk = clocks.stop() if clocks else None

    # the phases of one step (verify, accept + path read, commit) and the dominant kernel:
    # the gate/up expert stream of the last layer's (local) expert call, its bytes from that
    # call's unique experts on this rank
    c4_restore(model, snap, C4_CTX)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    ph_steps, moe_ph = [], []
    k3.moe_phase_timing(True)
    idx_last = None
    emitted = []          # every sequence's emitted ids, step by step (the stream's fingerprint)
    for s in range(warm):
        ev[0].record(stream)
        arg, _ = model.verify(tok_dev[s], parent=parent, logits=False)
        ev[1].record(stream)
        emit, n_emit, path, _ = k3.accept_tree_greedy(None, tok_dev[s], parent_dev, arg=arg)
        keep = n_emit.tolist()
        ph_path = path.tolist()
        emit_np = emit.cpu().numpy()
        emitted += [emit_np[b, :keep[b]] for b in range(B)]
        ev[2].record(stream)
        moe_ph.append(k3.moe_phase_ms())
        idx_last = model.last_routing(C4_TREE).clone()
        model.commit(keep, ph_path)
        ev[3].record(stream)
        torch.cuda.synchronize()
        ph_steps.append([ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), ev[2].elapsed_time(ev[3])])
    k3.moe_phase_timing(False)
    ph = np.median(np.array(ph_steps), axis=0).tolist()
    mph = np.median(np.array(moe_ph), axis=0).tolist()
    R = B * C4_TREE
    E, I_, n_exp, ns = C4["hidden_size"], C4["moe_intermediate_size"], C4["num_experts"], C4["num_shared_experts"]
    w13 = 2 * I_ * (E // 2 + E // 32)
    if dist:
        # this rank's experts in the last layer's call: those some rank's tokens chose
        alls = [torch.empty_like(idx_last) for _ in range(world)]
        dist.all_gather(alls, idx_last)
        g_idx = torch.cat(alls).cpu().numpy()
        nl = n_exp // world
        mine = g_idx[(g_idx >= rank * nl) & (g_idx < (rank + 1) * nl)]
        u = len(np.unique(mine))
        rows = int(((g_idx // nl) == rank).any(axis=1).sum())
        gateup_bytes = u * w13 + rows * E * 4 + int(mine.size) * I_ * 4
    else:
        il = idx_last.cpu().numpy()
        u = len(np.unique(il[il >= 0])) + ns
        pairs = R * (TOPK + ns)
        gateup_bytes = u * w13 + R * E * 4 + pairs * I_ * 4
    hbm, peak_kind = peaks()
    achieved = gateup_bytes / (mph[2] * 1e-3) / 1e9 if mph[2] > 0 else 0.0
    achieved = -max_over_ranks(-achieved)        # the slowest rank's stream
    traffic = None
    tp = os.path.join(ROOT, "profiles", "moe_gateup_traffic.json")
    if os.path.exists(tp) and world == 1:
        try:
            ratio = float(json.load(open(tp))["traffic_over_algorithmic"])
            traffic = int(ratio * gateup_bytes)
        except (OSError, ValueError, KeyError, TypeError):
            traffic = None
    parity = c4_ep_parity(args, k3, dev, model, snap, tok_dev[warm], parent, rank, world, dist) if dist else None
    if exchange:
        exchange.close()
    model.close()
    del model
    torch.cuda.empty_cache()
    full = steps * B * (depth + 1) * world
    return {
        "value": round(accepted / (dev_ms * steps * 1e-3), 2), "ms_per_step": round(dev_ms, 3),
        "accepted_per_step": round(accepted / steps, 2), "accepted_fraction_of_planted": round(accepted / full, 4),
        "e2e": {"value": round(acc_e2e / (e2e_ms * steps * 1e-3), 2), "unit": "accepted tok/s",
                "h2d_bytes_per_step": int(B * C4_TREE * 4 * world),
                "d2h_bytes_per_step": int((B * 4 + 2 * B * C4_TREE * 4) * world), "ms_per_step": round(e2e_ms, 3)},
        "verify_step_ms": round(ph[0], 3), "accept_ms": round(ph[1], 3), "commit_ms": round(ph[2], 3),
        "moe_phase_ms_last_layer": {"router": round(mph[0], 4), "plan": round(mph[1], 4),
                                    "gateup": round(mph[2], 4), "down": round(mph[3], 4),
                                    "combine": round(mph[4], 4)},
        "roofline": {"bound": "hbm", "kernel": "moe_tc_kernel<0> (gate/up, last layer's expert call)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "traffic": traffic, "peak_source": peak_kind, "algorithmic_bytes_per_launch": int(gateup_bytes),
                     "units": f"{u} experts x {w13} B + rows" + (" (rank 0's; min over ranks)" if dist else "")},
        "gpu_launches": int(launches), "device_status": status, "clocks": clk, "build_s": round(build_s, 1),
        "fnv_accepted_ids": {"hash": fnv1a64(np.concatenate(emitted).astype(np.int32)),
                             "over": f"{warm} untimed steps x {B} sequences of rank {rank}: emitted ids, int32"},
        "ep": None if not dist else {"transport": "peer memory inside the model's MoE steps (k3gpu_moe_layer_ep)",
                                     "experts_per_gpu": n_exp // world, "owners_ok": bool(owners_ok >= 1),
                                     "parity": parity},
        "config": c4_config(B, R, world),
    }


C5_SEQS, C5_K, C5_CTX, C5_EXPERTS_PER_GPU = 64, 8, 8192, 48


def roofline_bound(flops, nbytes, tflops_peak, gbs_peak):
    """(tensor_bound, intensity, ridge): a call whose algorithmic flops per algorithmic byte
    exceed the ridge of the measured peaks (TFLOP/s over GB/s, in flop/B) is bounded by the
    tensor pipe, else by HBM."""
    intensity = flops / max(nbytes, 1)
    ridge = tflops_peak * 1e12 / (gbs_peak * 1e9)
    return intensity > ridge, intensity, ridge


def c5_cfg(n_layers, world):
    """Config 5's stack: config-2 layers (d 7168, FFN 2048 SwiGLU experts top-8 + 1 shared) in
    the 3:1 KDA:MLA pattern (every fourth layer MLA) with the slice's attention shapes, 48
    routed experts per GPU (384 at 8 GPUs)."""
    c = dict(C4)
    c["num_hidden_layers"] = n_layers
    c["full_attn_layers"] = [L for L in range(4, n_layers + 1, 4)]
    c["num_experts"] = C5_EXPERTS_PER_GPU * world
    return c


def c5_ep_parity(args, k3, dev, rank, world, dist, n_layers=4):
    """Before the stack is built: one chain sweep of a 4-layer stack of config 5's shapes,
    expert parallel over the ranks exactly as the stack runs (48 rank-drawn experts per GPU,
    the rows through peer memory), against the same 4 layers unsharded on rank 0 (every
    rank's experts drawn again by their seeds into one bank): argmax equal at every position
    of rank 0's sequences, logits within rel-L2 1e-3. A failed check ends the run."""
    import torch
    cfg = c5_cfg(n_layers, world)
    B, T = C5_SEQS // world, C5_K + 1
    seed = args.seed + 77
    model, shared = make_c4_model(k3, dev, B, seed, C5_CTX + 16, max_T=T, rank=rank, world=world, cfg=cfg,
                                  rank_banks=True)
    exchange = load_ep().EpExchange(k3, B * T, cfg["hidden_size"], cfg["num_experts_per_token"],
                                    C5_EXPERTS_PER_GPU)
    model.set_ep(exchange, shared)
    c4_fill_state(model, seed + 1 + 7919 * rank, C5_CTX)
    rng = np.random.default_rng(seed + 2 + 7919 * rank)
    ids = torch.tensor(rng.integers(0, cfg["vocab_size"], size=(B, T)), dtype=torch.int32, device=dev)
    arg, lg = model.verify(ids)
    torch.cuda.synchronize()
    arg_ep, lg_ep = arg.cpu(), lg.float().cpu()
    status = k3.device_status(dev.index)
    owners = min(model.ep_owners_ok())
    exchange.close()
    model.close()
    del model, shared
    torch.cuda.empty_cache()
    verdict = torch.zeros(4, dtype=torch.float64, device=dev)
    if rank == 0:
        full, _ = make_c4_model(k3, dev, B, seed, C5_CTX + 16, max_T=T, cfg=cfg, gather_ranks=world)
        c4_fill_state(full, seed + 1, C5_CTX)
        a1, l1 = full.verify(ids)
        torch.cuda.synchronize()
        verdict[0] = float((a1.cpu() != arg_ep).sum())
        verdict[1] = float((l1.float().cpu() - lg_ep).norm() / l1.float().cpu().norm())
        full.close()
        del full
        torch.cuda.empty_cache()
    verdict[2] = float(status)
    verdict[3] = float(1 - owners)
    dist.all_reduce(verdict, op=dist.ReduceOp.MAX)
    v = verdict.tolist()
    out = {"argmax_mismatches": int(v[0]), "logits_rel_l2": float(f"{v[1]:.3g}"), "status_max": int(v[2]),
           "owners_ok": v[3] == 0, "positions": B * T,
           "reference": f"the same {n_layers} layers unsharded on one GPU (all ranks' experts), rank 0's state and ids"}
    if v[0] != 0 or not v[1] < 1e-3 or v[2] != 0 or v[3] != 0:
        raise SystemExit(f"expert-parallel stack failed its check, no line printed: {out}")
    return out


def run_c5(args, k3, dev, local, rank=0, world=1):
    """Config 5: the full-depth stack (args.c5_layers layers; 93 fit one B200 beside the 8k
    caches at 48 experts per GPU), 64 sequences over all ranks each verifying a chain of its
    pending id and k = 8 drafts against an 8k-position cache: 576 tokens per step. A step is
    the greedy sweep (k3gpu_model_verify_greedy), the on-device chain acceptance from its
    argmaxes (k3gpu_accept_greedy), the read of the accepted counts and the commit. The drafts
    are forced as in config 4: each chain is the model's own greedy continuation (an untimed
    serial run), so every step accepts all 8 drafts plus the bonus id. world > 1: each rank
    holds 48 routed experts of every layer (rank-seeded) and verifies 64/world sequences;
    the token rows cross through peer memory inside every layer's MoE step."""
    import torch
    dist = None
    if world > 1:
        import torch.distributed as dist
    if C5_SEQS % world:
        raise SystemExit(f"--gpus must divide {C5_SEQS}")
    B, steps, warm, T = C5_SEQS // world, args.steps, args.warmup, C5_K + 1
    parity = c5_ep_parity(args, k3, dev, rank, world, dist) if dist and not args.profile_c4 else None
    cfg = c5_cfg(args.c5_layers, world)
    kv_cap = C5_CTX + (steps + warm + 2) * T + 8
    t_build = time.perf_counter()
    model, shared = make_c4_model(k3, dev, B, args.seed, kv_cap, max_T=T, rank=rank, world=world, cfg=cfg,
                                  rank_banks=True)
    exchange = None
    if world > 1:
        exchange = load_ep().EpExchange(k3, B * T, cfg["hidden_size"], cfg["num_experts_per_token"],
                                        C5_EXPERTS_PER_GPU)
        model.set_ep(exchange, shared)
    build_s = time.perf_counter() - t_build
    V = cfg["vocab_size"]
    seed_r = args.seed + 7919 * rank
    c4_fill_state(model, seed_r + 1, C5_CTX)
    snap = c4_snapshot(model, host=True)
    rng = np.random.default_rng(seed_r + 2)
    pending = torch.tensor(rng.integers(0, V, size=(B,)), dtype=torch.int32, device=dev)
    # The drafts are the model's own greedy continuation. A deep random stack turns the
    # last-bit differences between a one-position sweep and a nine-position one into
    # different argmaxes, so the continuation is taken from the nine-position verify itself:
    # its fixed point (Jacobi: drafts := the sweep's own argmaxes, shifted; after i rounds
    # the first i drafts are final), committed whole before the next step's chain is formed.
    # The timed steps replay these sweeps bit for bit and accept every draft.
    chains = torch.empty((warm + steps, B, T), dtype=torch.int32, device=dev)
    jacobi_rounds = []
    for s in range(warm + steps):
        ids = torch.cat([pending[:, None], torch.zeros((B, T - 1), dtype=torch.int32, device=dev)], dim=1)
        for r in range(T + 1):
            arg, _ = model.verify(ids, logits=False)
            moved = torch.tensor([float((ids[:, 1:] != arg[:, :-1]).any())], device=dev)
            if dist:
                dist.all_reduce(moved, op=dist.ReduceOp.MAX)
            if moved.item() == 0:
                break
            ids = torch.cat([ids[:, :1], arg[:, :-1]], dim=1).contiguous()
        jacobi_rounds.append(r + 1)
        chains[s] = ids
        model.commit([T] * B)
        pending = arg[:, -1].clone()
    c4_restore(model, snap, C5_CTX)
    stream = torch.cuda.current_stream()
    n_host = torch.empty((B,), dtype=torch.int32).pin_memory()

    def step(ids):
        arg, _ = model.verify(ids, logits=False)
        emit, n_emit, _ = k3.accept_greedy(None, ids[:, 1:].contiguous(), arg=arg)
        n_host.copy_(n_emit, non_blocking=True)
        stream.synchronize()
        keep = n_host.tolist()
        model.commit(keep)
        return sum(keep), emit

    def sync_all():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def max_over_ranks(v):
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v):
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        return float(t.item())

    for s in range(warm):
        step(chains[s])
    if args.profile_c4:   # one step inside an NVTX range, for an ncu launch list
        sync_all()
        torch.cuda.nvtx.range_push("c5_step")
        step(chains[warm])
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        if exchange:
            exchange.close()
        model.close()
        return None
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    accepted = 0
    sync_all()
    l0 = k3.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(warm, warm + steps):
        a, _ = step(chains[s])
        accepted += a
    e1.record(stream)
    sync_all()
    launches = k3.launch_count() - l0
    dev_ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    accepted = sum_over_ranks(accepted)
    status = int(max_over_ranks(k3.device_status(dev.index)))
    owners_ok = min(model.ep_owners_ok()) if exchange else 1
    owners_ok = -max_over_ranks(-owners_ok)
    # end to end: each step's chain ids from pinned host memory, the emitted ids back
    c4_restore(model, snap, C5_CTX)
    chains_host = chains.cpu().pin_memory()
    ids_dev = torch.empty((B, T), dtype=torch.int32, device=dev)
    emit_host = torch.empty((B, T), dtype=torch.int32).pin_memory()
    for s in range(warm):
        ids_dev.copy_(chains_host[s], non_blocking=True)
        step(ids_dev)
    acc_e2e = 0
    sync_all()
    e0.record(stream)
    for s in range(warm, warm + steps):
        ids_dev.copy_(chains_host[s], non_blocking=True)
        a, emit = step(ids_dev)
        emit_host.copy_(emit, non_blocking=True)
        acc_e2e += a
    e1.record(stream)
    sync_all()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    acc_e2e = sum_over_ranks(acc_e2e)
    clk = clocks.stop() if clocks else None
    # the last layer's local expert phases over a few untimed steps, and the ids they emit
    c4_restore(model, snap, C5_CTX)
    k3.moe_phase_timing(True)
    moe_ph, emitted = [], []
    idx_last = None
    for s in range(warm):
        arg, _ = model.verify(chains[s], logits=False)
        emit, n_emit, _ = k3.accept_greedy(None, chains[s][:, 1:].contiguous(), arg=arg)
        keep = n_emit.tolist()
        moe_ph.append(k3.moe_phase_ms())
        idx_last = model.last_routing(T).clone()
        e_np = emit.cpu().numpy()
        emitted += [e_np[b, :keep[b]] for b in range(B)]
        model.commit(keep)
    k3.moe_phase_timing(False)
    mph = np.median(np.array(moe_ph), axis=0).tolist()
    E, I_ = cfg["hidden_size"], cfg["moe_intermediate_size"]
    w13 = 2 * I_ * (E // 2 + E // 32)
    if dist:
        alls = [torch.empty_like(idx_last) for _ in range(world)]
        dist.all_gather(alls, idx_last)
        g_idx = torch.cat(alls).cpu().numpy()
        nl = C5_EXPERTS_PER_GPU
        mine = g_idx[(g_idx >= rank * nl) & (g_idx < (rank + 1) * nl)]
        u = len(np.unique(mine))
        rows = int(((g_idx // nl) == rank).any(axis=1).sum())
        gateup_bytes = u * w13 + rows * E * 4 + int(mine.size) * I_ * 4
        pairs = int(mine.size) + B * T                       # local routed pairs + the shared expert's
    else:
        il = idx_last.cpu().numpy()
        u = len(np.unique(il[il >= 0])) + cfg["num_shared_experts"]
        gateup_bytes = u * w13 + B * T * E * 4 + B * T * (TOPK + 1) * I_ * 4
        pairs = B * T * (TOPK + 1)
    # the gate/up call's algorithmic flops: 2 x (gate + up rows) x hidden per (token, expert)
    gateup_flops = 2.0 * pairs * 2 * I_ * E
    hbm, peak_kind = peaks()
    tf_peak = peaks_tensor()
    t_s = mph[2] * 1e-3 if mph[2] > 0 else float("inf")
    achieved = -max_over_ranks(-(gateup_bytes / t_s / 1e9))
    achieved_tf = -max_over_ranks(-(gateup_flops / t_s / 1e12))
    # which roof bounds the call: its intensity against the ridge of the measured peaks (at
    # 96 tokens an expert it is past the ridge, a contraction; at 12, a weight stream)
    tensor_bound, intensity, ridge = roofline_bound(gateup_flops, gateup_bytes, tf_peak, hbm)
    traffic = None
    tp = os.path.join(ROOT, "profiles", "moe_gateup_traffic.json")
    if os.path.exists(tp) and world == 1:
        try:
            traffic = int(float(json.load(open(tp))["traffic_over_algorithmic"]) * gateup_bytes)
        except (OSError, ValueError, KeyError, TypeError):
            traffic = None
    if exchange:
        exchange.close()
    model.close()
    del model
    torch.cuda.empty_cache()
    full = steps * B * T * world
    return {
        "value": round(accepted / (dev_ms * steps * 1e-3), 2), "ms_per_step": round(dev_ms, 3),
        "accepted_per_step": round(accepted / steps, 2), "accepted_fraction_of_planted": round(accepted / full, 4),
        "e2e": {"value": round(acc_e2e / (e2e_ms * steps * 1e-3), 2), "unit": "accepted tok/s",
                "h2d_bytes_per_step": int(B * T * 4 * world), "d2h_bytes_per_step": int((B * 4 + B * T * 4) * world),
                "ms_per_step": round(e2e_ms, 3)},
        "moe_phase_ms_last_layer": {"router": round(mph[0], 4), "plan": round(mph[1], 4), "gateup": round(mph[2], 4),
                                    "down": round(mph[3], 4), "combine": round(mph[4], 4)},
        "roofline": {"bound": "tensor" if tensor_bound else "hbm",
                     "kernel": "moe_tc_kernel<0> (gate/up, last layer's local expert call)",
                     "achieved": round(achieved_tf if tensor_bound else achieved, 1),
                     "peak": tf_peak if tensor_bound else hbm, "unit": "TFLOP/s" if tensor_bound else "GB/s",
                     "frac": round(achieved_tf / tf_peak if tensor_bound else achieved / hbm, 4),
                     "traffic": traffic, "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": int(gateup_bytes), "algorithmic_flops_per_launch": gateup_flops,
                     "intensity_flop_per_byte": round(intensity, 1), "ridge_flop_per_byte": round(ridge, 1),
                     "hbm": {"achieved_gbs": round(achieved, 1), "frac": round(achieved / hbm, 4)},
                     "tensor": {"achieved_tflops": round(achieved_tf, 1), "frac": round(achieved_tf / tf_peak, 4),
                                "note": "algorithmic flops; the kernel issues twice as many (fp32 rows as f16 hi "
                                        "and lo pieces)"},
                     "units": f"{u} experts x {w13} B + rows, {pairs} (token, expert) pairs"
                              + (" (slowest rank)" if dist else "")},
        "fnv_accepted_ids": {"hash": fnv1a64(np.concatenate(emitted).astype(np.int32)),
                             "over": f"{warm} untimed steps x {B} sequences of rank {rank}: emitted ids, int32"},
        "gpu_launches": int(launches), "device_status": status, "clocks": clk, "build_s": round(build_s, 1),
        "planting_sweeps_per_step": round(float(np.mean(jacobi_rounds)), 2),
        "ep": None if not dist else {"transport": "peer memory inside every layer's MoE step (k3gpu_moe_layer_ep)",
                                     "experts_per_gpu": C5_EXPERTS_PER_GPU, "owners_ok": bool(owners_ok >= 1),
                                     "parity": parity},
        "config": c5_config(args.c5_layers, world),
    }


def c5_config(n_layers, world):
    n_mla = n_layers // 4
    return {"workload": f"K3 full-depth stack (benchmark config 5): {n_layers} layers ({n_layers - n_mla} KDA + "
                        f"{n_mla} MLA, 3:1), {C5_SEQS} sequences each verifying a k={C5_K} chain "
                        f"({C5_SEQS * (C5_K + 1)} tokens per step) over an {C5_CTX}-position cache, greedy acceptance",
            "parallelism": f"ep{world}" if world > 1 else "single", "layers": n_layers,
            "layers_note": f"{n_layers} layers of {C5_EXPERTS_PER_GPU} routed experts per GPU with the 8k caches "
                           "fit one B200 (~165 GB); the stack is the same at every GPU count",
            "d_model": C4["hidden_size"], "vocab": C4["vocab_size"],
            "moe": f"{C5_EXPERTS_PER_GPU * world} routed top-8 ({C5_EXPERTS_PER_GPU} per GPU) + 1 shared, FFN 2048 "
                   "SwiGLU, MXFP4 (E2M1 + E8M0/32) N(0,0.02)",
            "kda": "32 heads x 128", "mla": "64 heads, q_lora 1536, kv_lora 512, nope 128, rope 64, v 128",
            "sequences_per_gpu": C5_SEQS // world, "tokens_verified_per_step": C5_SEQS * (C5_K + 1),
            "context": C5_CTX,
            "drafts": "forced: every chain is the model's own greedy continuation, the fixed point of an "
                      "untimed Jacobi run of the same nine-position verify (the reference's GATE-4 method)",
            "weights": "random init: bf16 projections N(0,0.02), MXFP4 experts N(0,0.02)",
            "l2": "weights streamed per step (~130 GB) exceed the 126 MB L2; no flush needed"}


def c4_ep_parity(args, k3, dev, model, snap, ids, parent, rank, world, dist):
    """One tree sweep of the expert-parallel model against the unsharded model on rank 0
    (the same weights, rank 0's state and tree): argmax equal at every node, logits within
    rel-L2 1e-3. A failed check ends the run without a line."""
    import torch
    c4_restore(model, snap, C4_CTX)
    arg, lg = model.verify(ids, parent=parent)
    torch.cuda.synchronize()
    arg_ep, lg_ep = arg.cpu(), lg.float().cpu()
    model.commit([0] * model.B, [[0] * C4_TREE for _ in range(model.B)])
    verdict = torch.zeros(3, dtype=torch.float64, device=dev)
    if rank == 0:
        full, _ = make_c4_model(k3, dev, model.B, args.seed, model.kv_cap)
        c4_fill_state(full, args.seed + 1, C4_CTX)
        a1, l1 = full.verify(ids, parent=parent)
        torch.cuda.synchronize()
        verdict[0] = float((a1.cpu() != arg_ep).sum())
        verdict[1] = float((l1.float().cpu() - lg_ep).norm() / l1.float().cpu().norm())
        full.close()
        del full
        torch.cuda.empty_cache()
    verdict[2] = float(k3.device_status(dev.index))
    dist.all_reduce(verdict, op=dist.ReduceOp.MAX)
    v = verdict.tolist()
    out = {"argmax_mismatches": int(v[0]), "logits_rel_l2": float(f"{v[1]:.3g}"), "status_max": int(v[2]),
           "reference": "the unsharded slice on one GPU, rank 0's state and tree"}
    # the north star's logits bound (rel-L2 1e-3): the expert sum runs per owner, then across
    # owners, and eight random layers carry the fp32 reordering to the logits
    if v[0] != 0 or not v[1] < 1e-3 or v[2] != 0:
        raise SystemExit(f"expert-parallel model failed its check, no line printed: {out}")
    return out


def c4_config(B, R=None, world=1):
    R = R if R is not None else B * C4_TREE
    E, V = C4["hidden_size"], C4["vocab_size"]
    ep = "" if world == 1 else (f", expert parallel over {world} GPUs ({C4['num_experts'] // world} experts per GPU, "
                                f"config 5's sharding), B sequences per GPU")
    return {"workload": f"K3 8-layer slice tree verify (benchmark config 4): B={B} sequences x "
                        f"{C4_TREE}-node draft tree (branching {C4_BRANCH}, depth {C4_DEPTH}) over a "
                        f"{C4_CTX}-position cache, greedy acceptance{ep}",
            "parallelism": f"ep{world}" if world > 1 else "single",
            "layers": "6 KDA + 2 MLA (3:1), every layer MoE", "d_model": E, "vocab": V,
            "moe": "384 routed top-8 + 1 shared, FFN 2048 SwiGLU, MXFP4 (E2M1 + E8M0/32) N(0,0.02)",
            "kda": "32 heads x 128", "mla": "64 heads, q_lora 1536, kv_lora 512, nope 128, rope 64, v 128",
            "B": B, "tree_nodes": C4_TREE, "tokens_verified_per_step": R, "context": C4_CTX,
            "drafts": "forced: each tree's most probable branch (depth 4) is the model's own greedy "
                      "continuation from an untimed serial run, the other 59 nodes random ids (the "
                      "reference's GATE-4 method; a random-weight model gives the n-gram drafter nothing "
                      "to match)",
            "weights": "random init: bf16 projections N(0,0.02), MXFP4 experts N(0,0.02)",
            "l2": "weights streamed per step (~75 GB) exceed the 126 MB L2; no flush needed"}


def unique_experts_bytes(idx_np, stride_bytes_per_expert):
    u = len(np.unique(idx_np[idx_np >= 0]))
    return u, u * stride_bytes_per_expert


# ------------------------------------------------------------------------ clocks ---
def sm_max_mhz(gpu_index=0):
    """The GPU's maximum SM clock (nvidia-smi clocks.max.sm), 1965 MHz when it cannot be read."""
    try:
        r = subprocess.run(["nvidia-smi", "-i", str(gpu_index), "--query-gpu=clocks.max.sm",
                            "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=20)
        return float(r.stdout.strip().splitlines()[0])
    except (OSError, ValueError, IndexError, subprocess.SubprocessError):
        return 1965.0


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        return self.summarize(self.lines)

    @staticmethod
    def summarize(lines):
        """Median SM clock under load, the max clock, and every throttle reason seen Active
        in the samples (csv,noheader,nounits lines of FIELDS); malformed lines are skipped."""
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                clk, cmax = float(f[1]), float(f[2])
            except ValueError:
                continue
            sm.append(clk)
            smax = cmax
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU baseline ---
def cpu_reference_run(x_np, gate_np, bias_np, bank_np, offs, stride, T, nthreads, n_routed=None):
    """The reference's kernels over T tokens on the host; returns (seconds, out, idx)."""
    n_routed = N_ROUTED if n_routed is None else n_routed
    from oracle import oracle as O
    lib = O.ref_bench()
    if lib is None:
        return None
    lay = np.array([offs["p1"], offs["s1"], offs["p2"], offs["s2"], offs["p3"], offs["s3"], stride],
                   np.int64)
    out = np.zeros((T, L_DIM), np.float32)
    idx = np.zeros((T, TOPK), np.int32)
    wt = np.zeros((T, TOPK), np.float32)
    t0 = time.perf_counter()
    rc = lib.ref_moe_layer(out, idx, wt, np.ascontiguousarray(x_np[:T]), gate_np,
                           bias_np.ctypes.data, bank_np, lay, T, L_DIM, I_DIM, n_routed, N_SHARED,
                           TOPK, 1, 4.0, 25.0, nthreads)
    dt = time.perf_counter() - t0
    if rc != 0:
        return None
    return dt, out, idx


def kda_prefill_cpu_baseline(T_sample=256, H=32, D=128, seed=5):
    """The reference reads a prompt with k3_kda_step, one position after another for every
    head (src/core/k3_ops.c:303-360): that chain over a bounded sample on one host thread
    (the reference's library is built here without OpenMP), as positions per second; None
    when the reference library was not built."""
    from oracle import oracle as O
    lib = O.ref_timed()
    if lib is None:
        return None
    rng = np.random.default_rng(seed)
    S = rng.standard_normal((H, D, D)).astype(np.float32) * np.float32(0.1)
    q, k, v = (rng.standard_normal((T_sample, H, D)).astype(np.float32) for _ in range(3))
    al = rng.uniform(0.9, 0.999, (T_sample, H, D)).astype(np.float32)
    be = rng.uniform(0.1, 0.9, (T_sample, H)).astype(np.float32)
    o = np.zeros(D, np.float32)
    t0 = time.perf_counter()
    for t in range(T_sample):
        for h in range(H):
            lib.k3_kda_step(S[h], o, q[t, h], k[t, h], v[t, h], al[t, h], float(be[t, h]), D, D)
    dt = time.perf_counter() - t0
    return {"value": round(T_sample / dt, 1), "unit": "positions/s", "cores": 1, "kind": "reference",
            "isa": O.ISA_TEXT[O.ref_bench_isa()],
            "sample": f"{T_sample} positions x {H} heads x {D}: k3_kda_step chained, one thread"}


def matmul_bf16_cpu_baseline(T, n_in, n_out, rows=256, seed=6):
    """The reference's bf16 projection (k3_matmul_bf16_batch_ld, include/k3/k3.h:454) on one
    host thread over a sample of `rows` output rows, scaled by rows to the full n_out (the
    cost is linear in them): microseconds for the whole call; None when the reference
    library was not built."""
    from oracle import oracle as O
    lib = O.ref_timed()
    if lib is None:
        return None
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((T, n_in)).astype(np.float32)
    W = ((rng.standard_normal((rows, n_in)).astype(np.float32) * np.float32(0.02)).view(np.uint32) >> 16) \
        .astype(np.uint16)
    Y = np.zeros((T, rows), np.float32)
    t0 = time.perf_counter()
    lib.k3_matmul_bf16_batch_ld(Y, rows, X, n_in, W.ctypes.data, n_in, rows, T)
    dt = time.perf_counter() - t0
    return {"value": round(dt * 1e6 * n_out / rows, 1), "unit": "us per call", "cores": 1, "kind": "reference",
            "isa": O.ISA_TEXT[O.ref_bench_isa()],
            "sample": f"{rows} of {n_out} output rows at T={T}, in={n_in}, scaled by rows; one thread"}


def fnv1a64(a) -> str:
    """FNV-1a (64-bit) over an array's bytes, the fingerprint the reference's benchmarks
    print beside each output (benchmarks/bench_router.c:65-88): equal hashes mean
    bit-identical outputs, so a GPU row and a CPU row over the same inputs compare at a
    glance. Used on integer outputs (routing indices, accepted ids), which the path must
    reproduce bit for bit."""
    h = 0xcbf29ce484222325
    for byte in np.ascontiguousarray(a).tobytes():
        h = ((h ^ byte) * 0x100000001b3) & 0xFFFFFFFFFFFFFFFF
    return f"{h:016x}"


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ----------------------------------------------------------------------- arms ------
def run_reference(args):
    """--impl reference: the reference engine's own CPU path for the headline workload
    (config 4, c4_reference_sample) on the host cores, one bounded sample per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch
    from oracle import oracle as O
    if O.ref_bench() is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libk3ref_bench.so was not built (reference sources absent when built)"}))
        return 0
    if not torch.cuda.is_available():
        print(json.dumps({"impl": "reference", "unavailable": "the 9 GB expert bank is drawn on the GPU box"}))
        return 0
    if args.workload == "c5":
        return run_reference_c5(args)
    bank, offs, stride = make_bank_device(N_ROUTED + N_SHARED, L_DIM, I_DIM, args.seed, "cuda")
    bank_np = bank.cpu().numpy()
    del bank
    torch.cuda.empty_cache()
    nth = host_threads()
    for i in range(min(args.warmup, 1)):
        c4_reference_sample(args, bank_np, offs, stride, nth, args.seed + 100 + i)
    samples = []
    for i in range(args.steps):
        r = c4_reference_sample(args, bank_np, offs, stride, nth, args.seed + i)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": "a reference layer sample failed (out of memory)"}))
            return 0
        samples.append(r)
    steps_s = [r["step_s"] for r in samples]
    step = statistics.median(steps_s)
    val = (C4_DEPTH + 1) / step
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "accepted tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * step, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 / MXFP4 weights x fp32 activations, double accumulate (reference CPU)",
        "data": "synthetic (seeded random weights, random 32k cache, forced drafts)",
        "config": c4_config(args.c4_B, None, args.gpus),
        "cpu_baseline": {"value": round(val, 4), "unit": "accepted tok/s", "cores": nth, "kind": "reference",
                         "isa": O.ISA_TEXT[O.ref_bench_isa()] + ", no OpenMP", "sample": c4_sample_text(nth)},
        "e2e": {"value": round(val, 4), "unit": "accepted tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "all_step_s": [round(x, 3) for x in steps_s],
        "layer_s_median": {k: round(statistics.median([r[k] for r in samples]), 4)
                           for k in ("kda_s", "mla_s", "moe_s", "lm_head_s")},
        "note": "one sequence at a time (the reference engine serves one sequence and drafts chains); "
                "the GPU arm verifies B sequences' 64-node trees per step",
    }
    print(json.dumps(line))
    return 0


def run_reference_c5(args):
    """--impl reference for config 5: the reference's per-sequence chain through the stack
    (c5_reference_sample), one bounded sample per step, on the host cores."""
    from oracle import oracle as O
    bank_np, offs, stride = c5_bank_np(args)
    nth = host_threads()
    for i in range(min(args.warmup, 1)):
        c5_reference_sample(args, bank_np, offs, stride, nth, args.seed + 100 + i)
    samples = []
    for i in range(args.steps):
        r = c5_reference_sample(args, bank_np, offs, stride, nth, args.seed + i)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": "a reference layer sample failed"}))
            return 0
        samples.append(r)
    steps_s = [r["step_s"] for r in samples]
    step = statistics.median(steps_s)
    val = (C5_K + 1) / step
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "accepted tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * step, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 / MXFP4 weights x fp32 activations, double accumulate (reference CPU)",
        "data": "synthetic (seeded random weights, random 8k caches, forced drafts)",
        "config": c5_config(args.c5_layers, args.gpus),
        "cpu_baseline": {"value": round(val, 4), "unit": "accepted tok/s", "cores": nth, "kind": "reference",
                         "isa": O.ISA_TEXT[O.ref_bench_isa()] + ", no OpenMP", "sample": c5_sample_text(args, nth)},
        "e2e": {"value": round(val, 4), "unit": "accepted tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "all_step_s": [round(x, 3) for x in steps_s],
        "layer_s_median": {k: round(statistics.median([r[k] for r in samples]), 4)
                           for k in ("kda_s", "mla_s", "moe_s", "lm_head_s")},
        "note": "one sequence at a time (the reference engine serves one sequence); the GPU arm verifies "
                f"{C5_SEQS} sequences' chains per step",
    }
    print(json.dumps(line))
    return 0


def make_bank_cpu(seed):
    raise SystemExit("the reference arm builds its weights on the GPU box; no CUDA device here")


def workload_config(args, M):
    return {"workload": f"K3 MoE layer verify (benchmark config 2): B={args.B} sequences x (1+k={1 + args.k}) "
                        f"= {M} tokens/step/GPU",
            "d_model": L_DIM, "experts": N_ROUTED, "shared": N_SHARED, "topk": TOPK,
            "ffn": I_DIM, "act": "SwiGLU", "weights": "MXFP4 (E2M1 + E8M0/32), N(0,0.02)",
            "activations": "bf16 N(0,1) (fp32 containers)", "B": args.B, "k": args.k,
            "tokens_per_step": M * args.gpus,
            "parallelism": f"ep{args.gpus}" if args.gpus > 1 else "single",
            "l2": "weights streamed per step (GBs) exceed the 126 MB L2; no flush needed"}


def load_ep():
    import importlib.util
    spec = importlib.util.spec_from_file_location("k3b200_ep", os.path.join(ROOT, "kimi-k3-for-me_b200", "ep.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_ep(args, k3, rank, world, dev):
    """--gpus N: the layer with its 384 routed experts sharded 384/N per GPU (expert
    parallel), each rank verifying its own B*(1+k) tokens (weak scaling). The token rows
    travel through peer memory (the library's k3gpu_ep_* kernels over NVLink; --ep-transport
    nccl uses NCCL all-to-all instead). Times are device events per rank, the max over ranks."""
    import torch
    import torch.distributed as dist
    ep = load_ep()
    M = args.B * (1 + args.k)
    if N_ROUTED % world:
        raise SystemExit(f"{N_ROUTED} experts do not split over {world} GPUs")
    n_local = N_ROUTED // world
    bank_l, offs, stride = make_bank_device(n_local, L_DIM, I_DIM, args.seed + 7919 * (rank + 1), dev)
    bank_s, _, _ = make_bank_device(N_SHARED, L_DIM, I_DIM, args.seed + 104729, dev)
    _, gate, bias = make_inputs(M, args.seed + 1, dev)               # replicated gate
    x = make_inputs(M, args.seed + 101 + rank, dev)[0]                # this rank's tokens
    kb_l = k3.ExpertBank(bank_l, n_local, L_DIM, I_DIM)
    kb_s = k3.ExpertBank(bank_s, N_SHARED, L_DIM, I_DIM)
    n_unsafe = 0
    if not args.no_tc:
        n_unsafe = kb_l.scan() + kb_s.scan()
    stream = torch.cuda.current_stream()
    if args.ep_transport == "p2p":
        layer = ep.P2PMoELayer(k3, kb_l, kb_s, gate, bias, N_ROUTED, TOPK, k3.ACT_SWIGLU, cap=M, stream=stream)
    else:
        layer = ep.EPMoELayer.from_k3(k3, kb_l, kb_s, gate, bias, N_ROUTED, TOPK, k3.ACT_SWIGLU, stream=stream)
    try:
        return _run_ep_timed(args, k3, rank, world, dev, layer, x, n_local, M, n_unsafe, stream)
    finally:
        if hasattr(layer, "close"):
            layer.close()


def ep_parity(args, k3, rank, world, dev, layer, x, res):
    """After the timed steps: the device status word of every rank (no bounded exchange wait
    ran out, no index was skipped), every owner's rows arrived at every rank, and the last
    step's outputs and routing on every rank equal the UNSHARDED single-GPU layer's
    (k3gpu_moe_layer over all 384 experts, rebuilt on rank 0 from the same seeds) on the
    same tokens. A failure ends the run without a line: such a step is not a measurement."""
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    status = k3.device_status(dev.index)
    owners = layer.owners_ok() if hasattr(layer, "owners_ok") else [1] * world
    xs = [torch.empty_like(x) for _ in range(world)]
    outs = [torch.empty_like(res["out"]) for _ in range(world)]
    idxs = [torch.empty_like(res["idx"]) for _ in range(world)]
    dist.all_gather(xs, x)
    dist.all_gather(outs, res["out"])
    dist.all_gather(idxs, res["idx"])
    verdict = torch.zeros(4, dtype=torch.float64, device=dev)   # status, owners bad, idx bad, rel
    verdict[0] = float(status)
    verdict[1] = float(min(owners) == 0)
    if rank == 0:
        n_local = N_ROUTED // world
        parts = [make_bank_device(n_local, L_DIM, I_DIM, args.seed + 7919 * (r + 1), dev)[0] for r in range(world)]
        parts.append(make_bank_device(N_SHARED, L_DIM, I_DIM, args.seed + 104729, dev)[0])
        full = torch.cat(parts)
        del parts
        kb = k3.ExpertBank(full, N_ROUTED + N_SHARED, L_DIM, I_DIM)
        if not args.no_tc:
            kb.scan()
        _, gate, bias = make_inputs(x.shape[0], args.seed + 1, dev)
        ref, ridx, _ = k3.moe_layer(torch.cat(xs), gate, bias, kb, TOPK, N_ROUTED, N_SHARED, k3.ACT_SWIGLU)
        got = torch.cat(outs)
        verdict[2] = float(not torch.equal(torch.cat(idxs), ridx))
        verdict[3] = float((got - ref).norm() / ref.norm())
        del full, kb
        torch.cuda.empty_cache()
    dist.all_reduce(verdict, op=dist.ReduceOp.MAX)
    v = verdict.tolist()
    parity = {"status_max_over_ranks": int(v[0]), "owners_ok": v[1] == 0, "idx_equal": v[2] == 0,
              "rel_l2": float(f"{v[3]:.3g}"), "reference": "k3gpu_moe_layer, all experts on one GPU"}
    if v[0] != 0 or v[1] != 0 or v[2] != 0 or not v[3] < 1e-5:
        raise SystemExit(f"expert-parallel step failed its check, no line printed: {parity}")
    return parity


def _run_ep_timed(args, k3, rank, world, dev, layer, x, n_local, M, n_unsafe, stream):
    import torch
    import torch.distributed as dist

    def timed(fn, steps):
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.barrier()
        return float(ms.item())

    res = {}

    def step():
        res["out"], res["idx"], res["wt"] = layer(x)

    for _ in range(args.warmup):
        step()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    dev_ms = timed(step, args.steps)

    x_host = x.cpu().pin_memory()
    out_host = torch.empty((M, L_DIM), dtype=torch.float32).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        o, _, _ = layer(x_dev)
        out_host.copy_(o, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_ms = timed(e2e_step, args.steps)
    clk = clocks.stop() if clocks else None

    # the local routed expert call is the last library call of a step: its phases
    k3.moe_phase_timing(True)
    phases = []
    for _ in range(max(3, min(args.steps, 10))):
        step()
        phases.append(k3.moe_phase_ms())
    k3.moe_phase_timing(False)
    ph = np.median(np.array(phases), axis=0).tolist()
    torch.cuda.synchronize()
    # bytes of the local gate/up stream: the local experts some rank sent rows to
    idx_all = [torch.empty_like(res["idx"]) for _ in range(world)]
    dist.all_gather(idx_all, res["idx"])
    g = torch.cat(idx_all).cpu().numpy()
    mine = g[(g >= rank * n_local) & (g < (rank + 1) * n_local)]
    u = len(np.unique(mine))
    rows = int(((g // n_local) == rank).any(axis=1).sum())
    w13 = 2 * I_DIM * (L_DIM // 2 + L_DIM // 32)
    gateup_bytes = u * w13 + rows * L_DIM * 4 + int(mine.size) * I_DIM * 4
    hbm, peak_kind = peaks()
    achieved = gateup_bytes / (ph[2] * 1e-3) / 1e9 if ph[2] > 0 else 0.0
    ach = torch.tensor([achieved], device=dev)
    dist.all_reduce(ach, op=dist.ReduceOp.MIN)
    parity = ep_parity(args, k3, rank, world, dev, layer, x, res)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(world * M / (dev_ms * 1e-3), 3), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "MXFP4 weights x fp32 activations, fp32 accumulate", "data": "synthetic (seeded)",
            "config": workload_config(args, M),
            "e2e": {"value": round(world * M / (e2e_ms * 1e-3), 3), "unit": "tok/s",
                    "h2d_bytes_per_step": int(x.numel() * 4 * world),
                    "d2h_bytes_per_step": int(M * L_DIM * 4 * world), "ms_per_step": round(e2e_ms, 4)},
            "roofline": {"bound": "hbm", "kernel": "moe_tc_kernel<0> (local gate/up)",
                         "achieved": round(float(ach.item()), 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(float(ach.item()) / hbm, 4), "traffic": None,
                         "peak_source": peak_kind, "note": "min over ranks, rank 0's bytes model"},
            "phase_ms_rank0_local_experts": {"plan": round(ph[1], 4), "gateup": round(ph[2], 4),
                                             "down": round(ph[3], 4), "combine": round(ph[4], 4)},
            # router 2 + shared experts 6 + local experts 6 (+2 each for mma.sync leftovers),
            # + 8 exchange kernels on the peer-memory transport
            "gpu_launches": (14 + (4 if n_unsafe else 0) + (8 if args.ep_transport == "p2p" else 0)) * args.steps,
            "ep_transport": "peer memory (k3gpu_ep_*, NVLink)" if args.ep_transport == "p2p" else "NCCL all_to_all",
            "ep_parity": parity,
            "clocks": clk,
            "cpu_baseline": None,
        }
        print(json.dumps(line))
    return 0


def measure_rows(k3, dev, hbm, tflops_peak, only=None):
    """The other rows of the verify path at their benchmark shapes, device-timed (CUDA events, 3
    warm-up and 10 timed calls, synthetic seeded inputs), with the bound each is graded
    against. A row that fails reports its error instead of a number."""
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(4242)
    rows = {}

    def timed(fn, n=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n * 1000.0        # us

    def hbm_row(us, nbytes, shape):
        gbs = nbytes / (us * 1e-6) / 1e9
        return {"us": round(us, 2), "bytes": int(nbytes), "gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 4),
                "bound": "hbm", "shape": shape}

    # c3 KDA verify + commit: 8 sequences x (1+k) for k = 4, 8, 16, 32 heads x 128, and a
    # rollback to an accepted length drawn U[0, k] per sequence
    for kk_ in (4, 8, 16):
        if only is not None and only != "kda_c3":
            break
        try:
            B, T, H, D = 8, 1 + kk_, 32, 128
            st = torch.randn((B, H, D, D), generator=g, device=dev) * 0.1
            q = torch.nn.functional.normalize(torch.randn((B, T, H, D), generator=g, device=dev), dim=-1)
            kk = torch.nn.functional.normalize(torch.randn((B, T, H, D), generator=g, device=dev), dim=-1)
            v = torch.randn((B, T, H, D), generator=g, device=dev)
            al = 0.9 + 0.099 * torch.rand((B, T, H, D), generator=g, device=dev)
            be = torch.sigmoid(torch.randn((B, T, H), generator=g, device=dev))
            qs = 1.0 / D ** 0.5
            us = timed(lambda: k3.kda_verify(st, q, kk, v, al, be, qs))
            nbytes = st.numel() * 4 + 4 * q.numel() * 4 + be.numel() * 4 + q.numel() * 4
            rows[f"kda_verify_c3_k{kk_}"] = hbm_row(us, nbytes, f"B=8 T={T} H=32 D=128")
            try:   # the reference's k3_kda_step chain over the same B*T positions x 32 heads
                cb = kda_prefill_cpu_baseline(T_sample=B * T, H=H, D=D)
                if cb is not None:
                    cb = dict(cb, value=round(B * T / cb["value"] * 1e6, 1), unit="us per call")
                rows[f"kda_verify_c3_k{kk_}"]["cpu_baseline"] = cb
            except Exception as ex:  # noqa: BLE001 -- the baseline must not cost the row
                rows[f"kda_verify_c3_k{kk_}"]["cpu_baseline"] = {"error": str(ex)[:120]}
            keep = np.random.default_rng(kk_).integers(0, kk_ + 1, size=B).astype(np.int32)
            n = torch.from_numpy(keep).to(dev)
            sc = st.clone()
            us = timed(lambda: k3.kda_commit(sc, kk, v, al, be, n))
            rows[f"kda_commit_c3_k{kk_}"] = hbm_row(
                us, 2 * st.numel() * 4 + 3 * q.numel() * 4 + be.numel() * 4,
                f"B=8 T={T} H=32 D=128, keep U[0,{kk_}] per sequence: {keep.tolist()}")
        except Exception as ex:  # noqa: BLE001
            rows[f"kda_c3_k{kk_}"] = {"error": str(ex)[:200]}

    # KDA prompt read-in (config 3's prefill): one 8192-position prompt, 32 heads x 128,
    # chunked (one launch) against the sequential kernels (verify + commit per 64 positions)
    if only is None or only == "kda_prefill":
        try:
            B, T, H, D = 1, 8192, 32, 128
            st = torch.randn((B, H, D, D), generator=g, device=dev) * 0.1
            q = torch.nn.functional.normalize(torch.randn((B, T, H, D), generator=g, device=dev), dim=-1)
            kk = torch.nn.functional.normalize(torch.randn((B, T, H, D), generator=g, device=dev), dim=-1)
            v = torch.randn((B, T, H, D), generator=g, device=dev)
            al = 0.9 + 0.099 * torch.rand((B, T, H, D), generator=g, device=dev)
            be = torch.sigmoid(torch.randn((B, T, H), generator=g, device=dev))
            qs = 1.0 / D ** 0.5
            sc = st.clone()
            us = timed(lambda: k3.kda_prefill(sc, q, kk, v, al, be, qs), n=5)
            blocks = [tuple(a[:, t0:t0 + 64].contiguous() for a in (q, kk, v, al, be)) for t0 in range(0, T, 64)]
            n64 = torch.full((B,), 64, dtype=torch.int32, device=dev)
            ss = st.clone()

            def sequential():
                for bq, bk, bv, ba, bb in blocks:
                    k3.kda_verify(ss, bq, bk, bv, ba, bb, qs)
                    k3.kda_commit(ss, bk, bv, ba, bb, n64)
            us_seq = timed(sequential, n=3)
            nbytes = 5 * q.numel() * 4 + be.numel() * 4 + 2 * st.numel() * 4
            row = hbm_row(us, nbytes, "B=1 T=8192 H=32 D=128 (one prompt), 32-position chunks")
            row.update({"positions_per_s": round(B * T / (us * 1e-6), 1), "sequential_us": round(us_seq, 2),
                        "speedup_vs_sequential": round(us_seq / us, 2), "compute": "fp32 CUDA cores"})
            try:
                row["cpu_baseline"] = kda_prefill_cpu_baseline(H=H, D=D)
            except Exception as ex:  # noqa: BLE001 -- the baseline must not cost the row
                row["cpu_baseline"] = {"error": str(ex)[:120]}
            rows["kda_prefill_8k"] = row
        except Exception as ex:  # noqa: BLE001
            rows["kda_prefill"] = {"error": str(ex)[:200]}

    # c4 MLA absorbed: 64-node tree (branching 4) over a 32k bf16 latent cache, 64 heads
    if only is None or only == "mla_absorbed_c4":
        try:
            B, T, H, qn, qr, vh, kvl, ctx = 1, 64, 64, 128, 64, 128, 512, 32768
            cap = ctx + T
            qnope = torch.randn((B, T, H, qn), generator=g, device=dev)
            qrope = torch.randn((B, T, H, qr), generator=g, device=dev)
            kvb = torch.randn((H * (qn + vh), kvl), generator=g, device=dev) * 0.05
            lat = torch.randn((B, cap, kvl), generator=g, device=dev).to(torch.bfloat16).view(torch.int16)
            rope = torch.randn((B, cap, qr), generator=g, device=dev).to(torch.bfloat16).view(torch.int16)
            cached = torch.tensor([ctx], dtype=torch.int32, device=dev)
            parent = [-1] + [(i - 1) // 4 for i in range(1, T)]
            masks = []
            for i in range(T):                          # ancestor bitmask of node i (itself included)
                m, j = 0, i
                while j >= 0:
                    m |= 1 << j
                    j = parent[j]
                masks.append(m - (1 << 64) if m >= (1 << 63) else m)
            mask = torch.tensor(masks, dtype=torch.int64, device=dev)
            ws = k3.workspace(k3.lib.k3gpu_mla_workspace(B, T, H, kvl, cap), dev)
            us = timed(lambda: k3.mla_absorbed(qnope, qrope, kvb, lat, rope, cached, mask, vh, cap,
                                                1.0 / (qn + qr) ** 0.5, ws=ws), n=10)
            flop = 2.0 * B * T * H * ctx * ((kvl + qr) + kvl)
            tf = flop / (us * 1e-6) / 1e12
            # the tcgen05 kernel issues 3.06x the algorithmic MMA work: hi and lo bf16 pieces of
            # the queries and of P, and the score product once per half of the latent output
            mma_factor = (4.0 * (kvl + qr) + 2.0 * kvl) / ((kvl + qr) + kvl)
            rows["mla_absorbed_c4"] = {"us": round(us, 1), "tflops": round(tf, 2), "frac_tensor": round(tf / tflops_peak, 4),
                                       "bound": "tensor", "shape": "64-node tree, 32k cache, H=64, kv_lora 512, rope 64",
                                       "mma_work_factor": round(mma_factor, 3),
                                       "issued_frac_tensor": round(tf * mma_factor / tflops_peak, 4),
                                       "note": "tcgen05 flash-decoding (q_abs, attend, merge kernels together)"}
        except Exception as ex:  # noqa: BLE001
            rows["mla_absorbed_c4"] = {"error": str(ex)[:200]}

    # trunk projection: T = 72 positions through a 7168 x 7168 bf16 matrix (tcgen05)
    if only is None or only == "trunk_matmul_bf16":
        try:
            T, n_in, n_out = 72, 7168, 7168
            X = torch.randn((T, n_in), generator=g, device=dev)
            W = (torch.randn((n_out, n_in), generator=g, device=dev) * 0.02).to(torch.bfloat16)
            Y = torch.empty((T, n_out), device=dev)
            ws = k3.workspace(k3.lib.k3gpu_matmul_bf16_workspace(T, n_in, n_out), dev)
            us = timed(lambda: k3.matmul_bf16(X, W, out=Y, ws=ws))
            rows["trunk_matmul_bf16"] = hbm_row(us, n_out * n_in * 2 + T * (n_in + n_out) * 4, "T=72, 7168 -> 7168")
            try:
                rows["trunk_matmul_bf16"]["cpu_baseline"] = matmul_bf16_cpu_baseline(T, n_in, n_out)
            except Exception as ex:  # noqa: BLE001 -- the baseline must not cost the row
                rows["trunk_matmul_bf16"]["cpu_baseline"] = {"error": str(ex)[:120]}
        except Exception as ex:  # noqa: BLE001
            rows["trunk_matmul_bf16"] = {"error": str(ex)[:200]}

    # lm_head: T = 72 positions through the c4 vocabulary (163840 x 7168 bf16, 2.35 GB)
    if only is None or only == "lm_head_bf16_c4":
        try:
            T, n_in, n_out = 72, 7168, 163840
            X = torch.randn((T, n_in), generator=g, device=dev)
            W = (torch.randn((n_out, n_in), generator=g, device=dev) * 0.02).to(torch.bfloat16)
            Y = torch.empty((T, n_out), device=dev)
            ws = k3.workspace(k3.lib.k3gpu_matmul_bf16_workspace(T, n_in, n_out), dev)
            us = timed(lambda: k3.matmul_bf16(X, W, out=Y, ws=ws))
            rows["lm_head_bf16_c4"] = hbm_row(us, n_out * n_in * 2 + T * (n_in + n_out) * 4, "T=72, 7168 -> 163840")
            try:
                rows["lm_head_bf16_c4"]["cpu_baseline"] = matmul_bf16_cpu_baseline(T, n_in, n_out)
            except Exception as ex:  # noqa: BLE001
                rows["lm_head_bf16_c4"]["cpu_baseline"] = {"error": str(ex)[:120]}
            del W, Y
        except Exception as ex:  # noqa: BLE001
            rows["lm_head_bf16_c4"] = {"error": str(ex)[:200]}

    # a tree batch's projection: T = 1024 positions (c4: 16 sequences x 64 nodes) through a
    # 7168 -> 4096 bf16 matrix; a real GEMM, graded as tensor work (hi and lo products)
    if only is None or only == "trunk_matmul_bf16_t1024":
        try:
            T, n_in, n_out = 1024, 7168, 4096
            X = torch.randn((T, n_in), generator=g, device=dev)
            W = (torch.randn((n_out, n_in), generator=g, device=dev) * 0.02).to(torch.bfloat16)
            Y = torch.empty((T, n_out), device=dev)
            ws = k3.workspace(k3.lib.k3gpu_matmul_bf16_workspace(T, n_in, n_out), dev)
            us = timed(lambda: k3.matmul_bf16(X, W, out=Y, ws=ws))
            tf = 4.0 * T * n_in * n_out / (us * 1e-6) / 1e12
            rows["trunk_matmul_bf16_t1024"] = {"us": round(us, 2), "tflops": round(tf, 1),
                                               "frac_tensor": round(tf / tflops_peak, 4), "bound": "tensor",
                                               "flops": "4*T*in*out (the hi and lo products)",
                                               "shape": "T=1024, 7168 -> 4096"}
            del W, Y
        except Exception as ex:  # noqa: BLE001
            rows["trunk_matmul_bf16_t1024"] = {"error": str(ex)[:200]}

    # the router over 384 experts x 7168: a verify step of config 2 (72 tokens) and the c4
    # sweep (1024 tokens); each score one in-order double chain, graded against FP64 issue
    # (64 FMA per clock per SM at the clock this run saw)
    if only is None or only == "router":
        try:
            n, hidden, topk = 384, 7168, 8
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            rr = {}
            for T in (72, 1024):
                x = torch.randn((T, hidden), generator=g, device=dev)
                W = torch.randn((n, hidden), generator=g, device=dev) * 0.02
                bias = torch.randn((n,), generator=g, device=dev) * 0.01
                ws = k3.workspace(k3.lib.k3gpu_router_workspace(T, n), dev)
                us = timed(lambda: k3.router(x, W, bias, topk, ws=ws))
                mhz = sm_max_mhz(torch.cuda.current_device())
                floor_us = T * n * hidden / (64.0 * sms * mhz)
                rr[f"T{T}"] = {"us": round(us, 2), "dfma_per_s": round(T * n * hidden / (us * 1e-6), 0),
                               "fp64_floor_us": round(floor_us, 2), "frac_fp64": round(floor_us / us, 4),
                               "sm_mhz": mhz}
            rows["router"] = dict(rr, bound="fp64 issue (64 FMA/clock/SM at the max SM clock); shared-memory "
                                            "operand delivery in practice",
                                  shape="384 experts x 7168, top-8")
        except Exception as ex:  # noqa: BLE001
            rows["router"] = {"error": str(ex)[:200]}

    # AttnRes at the config-5 sweep (576 positions x 7168): a stack 24 sources deep (the
    # 93-layer stack's average) and 48 deep (its last layers); every source read once
    if only is None or only == "attn_res_c5":
        try:
            T, n = 576, 7168
            ar = {}
            for nsrc in (24, 48):
                br = torch.randn((T, nsrc - 1, n), generator=g, device=dev)
                cur = torch.randn((T, n), generator=g, device=dev)
                fold = torch.randn((n,), generator=g, device=dev) * 0.05
                nb = torch.full((T,), nsrc - 1, dtype=torch.int32, device=dev)
                us = timed(lambda: k3.attn_res(br, cur, fold, nb, 1e-5))
                ar[f"sources{nsrc}"] = hbm_row(us, (nsrc * T * n + T * n + n + T) * 4,
                                               f"T={T} n={n}, {nsrc} sources")
                del br, cur
            rows["attn_res_c5"] = ar
        except Exception as ex:  # noqa: BLE001
            rows["attn_res_c5"] = {"error": str(ex)[:200]}

    # greedy accept over the K3 vocabulary: 8 sequences x 9 positions x 163840
    if only is None or only == "accept_greedy_vocab":
        try:
            B, T, V = 8, 9, 163840
            lg = torch.randn((B, T, V), generator=g, device=dev)
            d = lg[:, :T - 1].argmax(dim=2).to(torch.int32)
            us = timed(lambda: k3.accept_greedy(lg, d))
            rows["accept_greedy_vocab"] = hbm_row(us, lg.numel() * 4, "B=8 T=9 vocab=163840")
        except Exception as ex:  # noqa: BLE001
            rows["accept_greedy_vocab"] = {"error": str(ex)[:200]}
    return rows


def measure_c2(args, k3, dev, kb, bank, offs, stride, M, seed, n_unsafe, cpu_tokens=0):
    """One config-2 point: the MoE layer over M = B(1+k) verify tokens, device-timed, end to
    end with host buffers, the gate/up stream's roofline and (cpu_tokens > 0) the reference's
    kernels on a sample of the same step."""
    import torch
    x, gate, bias = make_inputs(M, seed, dev)
    ws = k3.workspace(k3.lib.k3gpu_moe_workspace(M, TOPK, N_SHARED, L_DIM, I_DIM, N_ROUTED), dev)
    out = torch.empty((M, L_DIM), dtype=torch.float32, device=dev)
    idx = torch.empty((M, TOPK), dtype=torch.int32, device=dev)
    wt = torch.empty((M, TOPK), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()

    def step():
        k3.moe_layer(x, gate, bias, kb, TOPK, N_ROUTED, N_SHARED, k3.ACT_SWIGLU, ws=ws, out=out,
                     idx=idx, wt=wt, stream=stream)

    steps = max(args.steps // 2, 5)
    for _ in range(3):
        step()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    l0 = k3.launch_count()
    ev0.record(stream)
    for _ in range(steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    launches = (k3.launch_count() - l0) // steps
    dev_ms = ev0.elapsed_time(ev1) / steps
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((M, L_DIM), dtype=torch.float32).pin_memory()
    idx_host = torch.empty((M, TOPK), dtype=torch.int32).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        k3.moe_layer(x_dev, gate, bias, kb, TOPK, N_ROUTED, N_SHARED, k3.ACT_SWIGLU, ws=ws,
                     out=out, idx=idx, wt=wt, stream=stream)
        out_host.copy_(out, non_blocking=True)
        idx_host.copy_(idx, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(steps):
        e2e_step()
    ev1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = ev0.elapsed_time(ev1) / steps
    k3.moe_phase_timing(True)
    phases = []
    for _ in range(5):
        step()
        phases.append(k3.moe_phase_ms())
    k3.moe_phase_timing(False)
    ph = np.median(np.array(phases), axis=0).tolist()
    idx_np = idx.cpu().numpy()
    u = len(np.unique(idx_np)) + N_SHARED
    pairs = M * (TOPK + N_SHARED)
    w13 = 2 * I_DIM * (L_DIM // 2 + L_DIM // 32)
    w2 = L_DIM * (I_DIM // 2 + I_DIM // 32)
    gateup_bytes = u * w13 + M * L_DIM * 4 + pairs * I_DIM * 4
    down_bytes = u * w2 + pairs * I_DIM * 4 + pairs * L_DIM * 4
    hbm, peak_kind = peaks()
    achieved = gateup_bytes / (ph[2] * 1e-3) / 1e9
    expert_gbs = (gateup_bytes + down_bytes) / ((ph[2] + ph[3]) * 1e-3) / 1e9
    row = {"M": M, "tokens_per_expert": round(M * TOPK / N_ROUTED, 2), "tok_s": round(M / (dev_ms * 1e-3), 1),
           "ms": round(dev_ms, 4), "e2e_tok_s": round(M / (e2e_ms * 1e-3), 1), "e2e_ms": round(e2e_ms, 4),
           "gateup": {"ms": round(ph[2], 4), "bytes": int(gateup_bytes), "gbs": round(achieved, 1),
                      "frac_hbm": round(achieved / hbm, 4)},
           "expert_stream": {"gbs": round(expert_gbs, 1), "frac_hbm": round(expert_gbs / hbm, 4),
                             "unique_experts": u},
           "phase_ms": {"router": round(ph[0], 4), "plan": round(ph[1], 4), "gateup": round(ph[2], 4),
                        "down": round(ph[3], 4), "combine": round(ph[4], 4)},
           "gpu_launches_per_step": int(launches), "fnv_routing": fnv1a64(idx_np)}
    if cpu_tokens > 0:
        Ts = min(M, cpu_tokens)
        bank_np = bank.cpu().numpy()
        r = cpu_reference_run(x.cpu().numpy(), gate.cpu().numpy(), bias.cpu().numpy(), bank_np,
                              offs, stride, Ts, host_threads())
        del bank_np
        if r is not None:
            from oracle import oracle as O
            dt, ref_out, ref_idx = r
            got = out.cpu().numpy()[:Ts]
            row["cpu_baseline"] = {
                "value": round(Ts / dt, 3), "unit": "tok/s", "cores": host_threads(), "kind": "reference",
                "isa": O.ISA_TEXT[O.ref_bench_isa()] + ", no OpenMP: pthreads over (token, slot) items",
                "sample": f"{Ts} of {M} tokens of the same step through the reference's k3_router + "
                          f"k3_matmul_mxfp4 expert loop ({dt:.2f} s)",
                "routing_bitexact": bool(np.array_equal(ref_idx, idx_np[:Ts])),
                "fnv_routing": fnv1a64(ref_idx.astype(np.int32)), "fnv_routing_gpu_same_tokens": fnv1a64(idx_np[:Ts]),
                "out_rel_l2_vs_gpu": float(np.linalg.norm(got - ref_out) / max(np.linalg.norm(ref_out), 1e-30))}
    return row


C2_SWEEP = [(1, 4), (1, 8), (1, 16), (8, 4), (8, 8), (8, 16), (64, 4), (64, 8), (64, 16)]


def c2_rows(args, k3, dev):
    """BASELINE config 2 at every (B, k): M = B(1+k) in {5, 9, 17, 40, 72, 136, 320, 576, 1088}."""
    import torch
    bank, offs, stride = make_bank_device(N_ROUTED + N_SHARED, L_DIM, I_DIM, args.seed, dev)
    kb = k3.ExpertBank(bank, N_ROUTED + N_SHARED, L_DIM, I_DIM)
    n_unsafe = kb.scan() if not args.no_tc else None
    out = {}
    for B, k in C2_SWEEP:
        M = B * (1 + k)
        try:
            cpu = args.cpu_tokens if (not args.no_cpu and (B, k) == (8, 8)) else 0
            out[f"B{B}_k{k}"] = measure_c2(args, k3, dev, kb, bank, offs, stride, M, args.seed + 1, n_unsafe, cpu)
        except Exception as ex:  # noqa: BLE001 -- one failed point must not cost the others
            out[f"B{B}_k{k}"] = {"M": M, "error": str(ex)[:200]}
    out["expert_kernels"] = "mma.sync" if args.no_tc else f"tcgen05 ({n_unsafe} experts on mma.sync)"
    del kb, bank
    torch.cuda.empty_cache()
    return out


def run_b200(args):
    import torch
    k3 = load_pkg()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        try:
            if args.workload == "c5":
                c5 = run_c5(args, k3, dev, local, rank, world)
                if rank == 0:
                    print(json.dumps(c5_line(args, c5, world, None, None)))
                return 0
            if args.ep_workload == "c2":
                return run_ep(args, k3, rank, world, dev)
            c4 = run_c4(args, k3, dev, local, rank, world)
            if rank == 0 and c4 is not None:
                print(json.dumps(c4_line(args, c4, world, None, None)))
            return 0
        finally:
            dist.destroy_process_group()

    hbm, peak_kind = peaks()
    if args.workload == "c5":
        c5 = run_c5(args, k3, dev, local)   # first: the stack takes ~160 of the 178 GiB
        if c5 is None:                      # --profile-c4: one profiled step
            return 0
        rows = {}
        if not args.no_rows:
            c4 = run_c4(args, k3, dev, local)
            rows["c4_slice_tree_verify"] = {k: c4[k] for k in ("value", "ms_per_step", "accepted_per_step",
                                                               "accepted_fraction_of_planted", "e2e", "roofline",
                                                               "verify_step_ms", "accept_ms", "commit_ms",
                                                               "moe_phase_ms_last_layer", "fnv_accepted_ids")}
            rows["c4_slice_tree_verify"]["config"] = c4["config"]
            rows["moe_layer_c2"] = c2_rows(args, k3, dev)
            rows.update(measure_rows(k3, dev, hbm, peaks_tensor()))
        cpu = None if args.no_cpu else c5_cpu_baseline(args)
        print(json.dumps(c5_line(args, c5, 1, cpu, rows)))
        return 0
    rows = {}
    if not args.no_rows and not args.profile_c4:
        rows["moe_layer_c2"] = c2_rows(args, k3, dev)
        rows.update(measure_rows(k3, dev, hbm, peaks_tensor()))
    c4 = run_c4(args, k3, dev, local)
    if c4 is None:        # --profile-c4
        return 0
    cpu = None if args.no_cpu else c4_cpu_baseline(args)
    print(json.dumps(c4_line(args, c4, 1, cpu, rows)))
    return 0


def c4_line(args, c4, world, cpu, rows):
    line = {
        "metric": METRIC, "value": c4["value"], "unit": "accepted tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": c4["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "MXFP4 experts and bf16 projections x fp32 activations, fp32 accumulate",
        "data": "synthetic (seeded random weights, random 32k cache, forced drafts)",
        "config": c4["config"], "e2e": c4["e2e"], "roofline": c4["roofline"],
        "verify_step_ms": c4["verify_step_ms"], "accept_ms": c4["accept_ms"], "commit_ms": c4["commit_ms"],
        "accepted_per_step": c4["accepted_per_step"],
        "accepted_fraction_of_planted": c4["accepted_fraction_of_planted"],
        "fnv_accepted_ids": c4["fnv_accepted_ids"],
        "moe_phase_ms_last_layer": c4["moe_phase_ms_last_layer"],
        "gpu_launches": c4["gpu_launches"], "device_status": c4["device_status"],
        "clocks": c4["clocks"], "cpu_baseline": cpu, "build_s": c4["build_s"], "ep": c4["ep"], "rows": rows,
    }
    return line


def c5_line(args, c5, world, cpu, rows):
    line = {
        "metric": METRIC, "value": c5["value"], "unit": "accepted tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": c5["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "MXFP4 experts and bf16 projections x fp32 activations, fp32 accumulate",
        "data": "synthetic (seeded random weights, random 8k caches, forced drafts)",
        "config": c5["config"], "e2e": c5["e2e"], "roofline": c5["roofline"],
        "accepted_per_step": c5["accepted_per_step"],
        "accepted_fraction_of_planted": c5["accepted_fraction_of_planted"],
        "fnv_accepted_ids": c5["fnv_accepted_ids"], "moe_phase_ms_last_layer": c5["moe_phase_ms_last_layer"],
        "gpu_launches": c5["gpu_launches"], "device_status": c5["device_status"], "clocks": c5["clocks"],
        "cpu_baseline": cpu, "build_s": c5["build_s"], "planting_sweeps_per_step": c5["planting_sweeps_per_step"],
        "ep": c5["ep"], "rows": rows,
    }
    return line


def c4_reference_sample(args, bank_np=None, offs=None, stride=None, nth=None, seed=0):
    """The reference engine verifying the same accepted branch on the host: one sequence's
    sweep of the 5-position chain (the pending id and the 4 drafts that are accepted -- the
    reference drafts chains only) through its own kernels, timed layer by layer on a bounded
    sample and summed over the slice: 6 x (KDA layer + MoE) + 2 x (MLA layer over the 32k
    cache + MoE) + the lm_head over 5 positions (a 4096-row sample scaled to 163840 rows).
    The KDA and MLA layers are k3_kda_layer_log and k3_mla_cached (latent, absorbed) at K3
    dimensions (oracle/ref_slice_bench.c), serial as the reference runs without OpenMP; the
    MoE is its k3_router + k3_matmul_mxfp4 expert loop over all host threads
    (oracle/ref_moe_bench.c) on the config's 385-expert bank. Returns a dict with the step
    seconds and the accepted tok/s it implies (5 ids per step), or None when the reference
    library was not built."""
    from oracle import oracle as O
    lib = O.ref_bench()
    if lib is None:
        return None
    for f in ("ref_c4_kda", "ref_c4_mla", "ref_c4_lm_rows"):
        getattr(lib, f).restype = C.c_double
        getattr(lib, f).argtypes = [C.c_int, C.c_int, C.c_uint] if f == "ref_c4_mla" else [C.c_int, C.c_uint]
    T = C4_DEPTH + 1
    lm_rows = 4096
    t_kda = lib.ref_c4_kda(T, seed + 1)
    t_mla = lib.ref_c4_mla(T, C4_CTX, seed + 2)
    t_lm = lib.ref_c4_lm_rows(T, lm_rows, seed + 3) * C4["vocab_size"] / lm_rows
    t_moe = None
    if bank_np is not None:
        rng = np.random.default_rng(seed + 4)
        x = rng.standard_normal((T, L_DIM), dtype=np.float32)
        gate = rng.standard_normal((N_ROUTED, L_DIM), dtype=np.float32) * np.float32(0.02)
        bias = rng.standard_normal(N_ROUTED, dtype=np.float32) * np.float32(0.01)
        r = cpu_reference_run(x, gate, bias, bank_np, offs, stride, T, nth)
        t_moe = r[0] if r is not None else None
    if min(t_kda, t_mla, t_lm) < 0 or t_moe is None:
        return None
    n_kda, n_mla = 6, 2
    step = n_kda * (t_kda + t_moe) + n_mla * (t_mla + t_moe) + t_lm
    return {"step_s": step, "value": T / step, "kda_s": t_kda, "mla_s": t_mla, "moe_s": t_moe, "lm_head_s": t_lm}


def c4_sample_text(nth):
    return (f"one sequence verifying the accepted 5-position branch: the reference's k3_kda_layer_log and "
            f"k3_mla_cached (latent, absorbed, 32768 cached positions) at K3 dims timed once each (serial, no "
            f"OpenMP), its k3_router + k3_matmul_mxfp4 MoE over 5 tokens on {nth} host threads, the lm_head "
            f"over a 4096-row sample scaled to 163840, summed as 6 x (KDA + MoE) + 2 x (MLA + MoE) + lm_head")


def c4_cpu_baseline(args):
    """The reference on the host beside our run (rank 0, N = 1): one bounded sample."""
    import torch
    from oracle import oracle as O
    bank, offs, stride = make_bank_device(N_ROUTED + N_SHARED, L_DIM, I_DIM, args.seed, "cuda")
    bank_np = bank.cpu().numpy()
    del bank
    torch.cuda.empty_cache()
    nth = host_threads()
    r = c4_reference_sample(args, bank_np, offs, stride, nth, args.seed)
    del bank_np
    if r is None:
        return None
    return {"value": round(r["value"], 4), "unit": "accepted tok/s", "cores": nth, "kind": "reference",
            "isa": O.ISA_TEXT[O.ref_bench_isa()] + ", no OpenMP",
            "sample": c4_sample_text(nth), "step_s": round(r["step_s"], 3),
            "layer_s": {k: round(r[k], 4) for k in ("kda_s", "mla_s", "moe_s", "lm_head_s")}}


def c5_reference_sample(args, bank_np, offs, stride, nth, seed=0):
    """The reference engine verifying one sequence's k = 8 chain (its pending id and 8 drafts,
    all accepted) through the config-5 stack on the host: its k3_kda_layer_log and
    k3_mla_cached (latent, absorbed, 8192 cached positions) at K3 dimensions timed once each
    (serial, as the reference runs without OpenMP), its k3_router + k3_matmul_mxfp4 MoE over
    the 9 tokens on all host threads with a 48-routed-expert bank, the lm_head over a
    4096-row sample scaled to 163840 rows; summed over the layers as the stack has them.
    Returns the step seconds and the accepted tok/s they imply (9 ids a step)."""
    from oracle import oracle as O
    lib = O.ref_bench()
    if lib is None:
        return None
    for f in ("ref_c4_kda", "ref_c4_mla", "ref_c4_lm_rows"):
        getattr(lib, f).restype = C.c_double
        getattr(lib, f).argtypes = [C.c_int, C.c_int, C.c_uint] if f == "ref_c4_mla" else [C.c_int, C.c_uint]
    T, n_layers = C5_K + 1, args.c5_layers
    n_mla = n_layers // 4
    lm_rows = 4096
    t_kda = lib.ref_c4_kda(T, seed + 1)
    t_mla = lib.ref_c4_mla(T, C5_CTX, seed + 2)
    t_lm = lib.ref_c4_lm_rows(T, lm_rows, seed + 3) * C4["vocab_size"] / lm_rows
    rng = np.random.default_rng(seed + 4)
    x = rng.standard_normal((T, L_DIM), dtype=np.float32)
    gate = rng.standard_normal((C5_EXPERTS_PER_GPU, L_DIM), dtype=np.float32) * np.float32(0.02)
    bias = rng.standard_normal(C5_EXPERTS_PER_GPU, dtype=np.float32) * np.float32(0.01)
    r = cpu_reference_run(x, gate, bias, bank_np, offs, stride, T, nth, n_routed=C5_EXPERTS_PER_GPU)
    if r is None or min(t_kda, t_mla, t_lm) < 0:
        return None
    t_moe = r[0]
    step = (n_layers - n_mla) * (t_kda + t_moe) + n_mla * (t_mla + t_moe) + t_lm
    return {"step_s": step, "value": T / step, "kda_s": t_kda, "mla_s": t_mla, "moe_s": t_moe, "lm_head_s": t_lm}


def c5_sample_text(args, nth):
    n_mla = args.c5_layers // 4
    return (f"one sequence verifying its 9-position chain (pending id + 8 accepted drafts): the reference's "
            f"k3_kda_layer_log and k3_mla_cached (latent, absorbed, {C5_CTX} cached positions) at K3 dims timed "
            f"once each (serial, no OpenMP), its k3_router + k3_matmul_mxfp4 MoE over 9 tokens on {nth} host "
            f"threads with {C5_EXPERTS_PER_GPU} routed experts, the lm_head over a 4096-row sample scaled to "
            f"163840, summed as {args.c5_layers - n_mla} x (KDA + MoE) + {n_mla} x (MLA + MoE) + lm_head")


def c5_bank_np(args):
    import torch
    bank, offs, stride = make_bank_device(C5_EXPERTS_PER_GPU + N_SHARED, L_DIM, I_DIM, args.seed, "cuda")
    bank_np = bank.cpu().numpy()
    del bank
    torch.cuda.empty_cache()
    return bank_np, offs, stride


def c5_cpu_baseline(args):
    """The reference on the host beside our run (rank 0, N = 1): one bounded sample."""
    from oracle import oracle as O
    bank_np, offs, stride = c5_bank_np(args)
    nth = host_threads()
    r = c5_reference_sample(args, bank_np, offs, stride, nth, args.seed)
    if r is None:
        return None
    return {"value": round(r["value"], 4), "unit": "accepted tok/s", "cores": nth, "kind": "reference",
            "isa": O.ISA_TEXT[O.ref_bench_isa()] + ", no OpenMP", "sample": c5_sample_text(args, nth),
            "step_s": round(r["step_s"], 3),
            "layer_s": {k: round(r[k], 4) for k in ("kda_s", "mla_s", "moe_s", "lm_head_s")}}


def main():
    global N_ROUTED
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--B", type=int, default=8, help="sequences per GPU (config-2 layer runs)")
    ap.add_argument("--c4-B", type=int, default=16, help="sequences of the config-4 slice (headline)")
    ap.add_argument("--k", type=int, default=8, help="drafts per sequence")
    ap.add_argument("--seed", type=int, default=2024)
    ap.add_argument("--cpu-tokens", type=int, default=72, help="tokens in the CPU baseline sample")
    ap.add_argument("--ref-tokens", type=int, default=0, help="tokens per reference-arm step (0 = all)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-rows", action="store_true", help="skip the other rows' kernel timings")
    ap.add_argument("--no-tc", action="store_true", help="skip the bank scan: mma.sync expert kernels only")
    ap.add_argument("--workload", default="c5", choices=["c4", "c5"],
                    help="the headline: config 5's full-depth expert-parallel stack (default; config 4's slice "
                         "tree verification is a row beside it at one GPU) or config 4 alone")
    ap.add_argument("--c5-layers", type=int, default=93,
                    help="layers of the config-5 stack (93, the K3 depth, fit one B200 at 48 experts per GPU)")
    ap.add_argument("--ep-workload", default="c4", choices=["c4", "c2"],
                    help="--gpus N > 1: the config-4 slice expert parallel (default) or one config-2 layer")
    ap.add_argument("--ep-transport", default="p2p", choices=["p2p", "nccl"],
                    help="--gpus N > 1: token rows through peer memory (default) or NCCL all-to-all")
    ap.add_argument("--only-row", default=None,
                    choices=["kda_c3", "kda_prefill", "mla_absorbed_c4", "trunk_matmul_bf16", "lm_head_bf16_c4",
                             "trunk_matmul_bf16_t1024", "router", "attn_res_c5", "accept_greedy_vocab"],
                    help="time one of the other rows alone and print it (for profiling captures)")
    ap.add_argument("--only-c2", type=int, nargs=2, metavar=("B", "K"), default=None,
                    help="time the config-2 layer at one (B, k) point alone and print its row (small cases "
                         "for captures with --n-routed)")
    ap.add_argument("--fp32-acts", action="store_true",
                    help="with --only-c2: full fp32 activations (the model's post-norm rows) instead of bf16")
    ap.add_argument("--profile-c4", action="store_true",
                    help="build the headline workload, run the warm-up steps, then one step inside the NVTX range "
                         "'c4_step' (--workload c4) or 'c5_step' (c5) and exit (for an ncu launch list with "
                         "--nvtx-include c5_step/)")
    ap.add_argument("--n-routed", type=int, default=N_ROUTED,
                    help="routed experts (smaller values give small cases for ncu captures)")
    args = ap.parse_args()
    N_ROUTED = args.n_routed
    if args.workload == "c5" and "torch" not in sys.modules:
        # the stack fills ~160 of the 178 GiB: the expert draws' temporaries must not strand
        # reserved segments that the model's one large arena then cannot use
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.only_c2:
        import torch
        k3 = load_pkg()
        dev = torch.device("cuda", 0)
        bank, offs, stride = make_bank_device(N_ROUTED + N_SHARED, L_DIM, I_DIM, args.seed, dev)
        kb = k3.ExpertBank(bank, N_ROUTED + N_SHARED, L_DIM, I_DIM)
        n_unsafe = kb.scan() if not args.no_tc else None
        B, k = args.only_c2
        global FP32_ACTS
        FP32_ACTS = args.fp32_acts
        print(json.dumps(measure_c2(args, k3, dev, kb, bank, offs, stride, B * (1 + k), args.seed + 1, n_unsafe)))
        return 0
    if args.only_row:
        k3 = load_pkg()
        hbm, _ = peaks()
        print(json.dumps(measure_rows(k3, "cuda", hbm, peaks_tensor(), only=args.only_row)))
        return 0
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
