"""Expert-parallel MoE layer: the routed experts sharded over the ranks of a process group.

One process per GPU. The reference runs every expert of a layer on one host
(src/core/k3_ops.c:2058-2132, k3_moe_prefill); here the routed experts of a layer are
split into `world` contiguous shards of n_routed / world experts, and a layer step over
each rank's own tokens is

  1. route locally (the gate is replicated): idx, wt [T][topk] with global expert ids;
  2. dispatch: every token goes once to each rank that owns one of its experts (rows
     deduplicated per destination), carrying, per top-k slot, the local expert id on that
     rank (or -1) and the routing weight -- one all-to-all of packed rows after an
     all-to-all of the row counts;
  3. the owner runs k3gpu_moe_experts on what it received: its experts, weighted, summed
     over the token's slots it owns;
  4. combine: the partial sums go back with the reverse all-to-all, and the source adds
     them per token to the shared experts' output (shared experts are replicated and run
     on the rank's own tokens).

The sum over a token's experts is therefore taken per owning rank and then across ranks,
not in top-k order as on one GPU: the results agree to fp32 rounding, not bit for bit.
The backend is whatever the process group is (NCCL on GPUs, gloo in the CPU tests); the
row counts make one device-to-host copy per step (the all-to-all split sizes).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def plan_dispatch(idx: torch.Tensor, wt: torch.Tensor, n_local: int, world: int):
    """Send plan for one step. idx/wt [T][K] (global expert ids, -1 = dropped slot).

    Returns (send_tok [S], send_counts [world], meta_idx [S][K] int32, meta_wt [S][K]):
    row s goes to rank d (rows ordered by destination, then token), carries token
    send_tok[s] and, per slot k, the local expert id on d (-1 when slot k is not d's)
    and the weight (0 there)."""
    T, K = idx.shape
    idx64 = idx.to(torch.int64)
    valid = idx64 >= 0
    dest = torch.where(valid, idx64 // n_local, torch.full_like(idx64, -1))
    ranks = torch.arange(world, device=idx.device, dtype=torch.int64)
    hit = dest.unsqueeze(1) == ranks.view(1, world, 1)            # [T][world][K]
    present = hit.any(dim=2)                                        # [T][world]
    d_s, t_s = present.t().nonzero(as_tuple=True)                   # sorted by d, then t
    send_counts = present.sum(dim=0).to(torch.int64)                # [world]
    sel = hit[t_s, d_s]                                             # [S][K]
    local = idx64 - dest * n_local
    meta_idx = torch.where(sel, local[t_s], torch.full_like(local[t_s], -1)).to(torch.int32)
    meta_wt = torch.where(sel, wt[t_s], torch.zeros_like(wt[t_s]))
    return t_s, send_counts, meta_idx, meta_wt


def _pack(rows: torch.Tensor, meta_idx: torch.Tensor, meta_wt: torch.Tensor) -> torch.Tensor:
    """[S][L + 2K] fp32: the row, the K local ids (int32 bits) and the K weights."""
    return torch.cat([rows, meta_idx.view(torch.float32), meta_wt], dim=1)


def _unpack(buf: torch.Tensor, L: int, K: int):
    rows = buf[:, :L].contiguous()
    meta_idx = buf[:, L:L + K].contiguous().view(torch.int32)
    meta_wt = buf[:, L + K:L + 2 * K].contiguous()
    return rows, meta_idx, meta_wt


class EPMoELayer:
    """One MoE layer with its routed experts sharded across `group`.

    route_fn(x) -> (idx, wt); experts_fn(z, idx, wt) -> [R][L], the weighted sum over each
    row's slots of this rank's experts (local ids, -1 dropped); shared_fn(x) -> [T][L] or
    None. The GPU constructor `from_k3` binds these to the library's C ABI; tests bind
    them to a CPU stand-in."""

    def __init__(self, route_fn: Callable, experts_fn: Callable, shared_fn: Optional[Callable],
                 n_routed: int, topk: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_routed % self.world:
            raise ValueError(f"{n_routed} routed experts do not split over {self.world} ranks")
        self.n_local = n_routed // self.world
        self.topk = topk
        self.route_fn, self.experts_fn, self.shared_fn = route_fn, experts_fn, shared_fn

    @classmethod
    def from_k3(cls, k3, bank_local, shared_bank, gate_W, bias, n_routed, topk, act,
                b1=4.0, b2=25.0, renorm=1, routed_scale=1.0, group=None, stream=None):
        """bank_local: this rank's n_routed/world routed experts (an ExpertBank, no shared
        experts); shared_bank: the shared experts (ExpertBank) or None."""
        world = dist.get_world_size(group)
        n_local = n_routed // world

        def route(x):
            return k3.router(x, gate_W, bias, topk, renorm, routed_scale, stream=stream)

        def experts(z, idx, wt):
            return k3.moe_experts(z, idx, wt, bank_local, topk, n_local, 0, act, b1, b2, stream=stream)

        shared = None
        if shared_bank is not None:
            ns = shared_bank.n_experts

            def shared(x):
                T = x.shape[0]
                idx = torch.arange(ns, device=x.device, dtype=torch.int32).repeat(T, 1)
                wt = torch.ones((T, ns), device=x.device, dtype=torch.float32)
                return k3.moe_experts(x, idx, wt, shared_bank, ns, ns, 0, act, b1, b2, stream=stream)

        return cls(route, experts, shared, n_routed, topk, group)

    def forward(self, x: torch.Tensor):
        """x [T][L] fp32 -> (out [T][L], idx, wt)."""
        T, L = x.shape
        K = self.topk
        idx, wt = self.route_fn(x)
        send_tok, send_counts, meta_idx, meta_wt = plan_dispatch(idx, wt, self.n_local, self.world)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        # split sizes are host lists: the one device-to-host copy of the step
        counts = torch.stack([send_counts, recv_counts]).cpu()
        s_split, r_split = counts[0].tolist(), counts[1].tolist()
        send = _pack(x[send_tok], meta_idx, meta_wt)
        recv = torch.empty((sum(r_split), L + 2 * K), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(recv, send, r_split, s_split, group=self.group)
        out = self.shared_fn(x) if self.shared_fn is not None else torch.zeros_like(x)
        z, ridx, rwt = _unpack(recv, L, K)
        part = self.experts_fn(z, ridx, rwt) if z.shape[0] else torch.empty((0, L), dtype=x.dtype, device=x.device)
        back = torch.empty((sum(s_split), L), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(back, part.contiguous(), s_split, r_split, group=self.group)
        out.index_add_(0, send_tok, back)
        return out, idx, wt

    __call__ = forward
