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

Two transports. `EPMoELayer` exchanges through the process group (NCCL on GPUs, gloo in
the CPU tests): all-to-all of the row counts, one device-to-host copy of them (the split
sizes), all-to-all of the packed rows and back. `P2PMoELayer` is the B200 path: every rank
maps every other rank's exchange arena (CUDA IPC over NVLink / NVSwitch) and the library's
k3gpu_ep_* kernels store rows straight into the owners' arenas and signal with
system-scope flags (bounded waits), so a step has no collective and no host round trip;
the process group is used once, to share the IPC handles.
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


class EpExchange:
    """The peer-memory exchange of one rank: its arena (k3gpu_ep_arena_alloc), every other
    rank's arena mapped by CUDA IPC (the process group carries the handles once), and the
    K3GpuEpGroup the k3gpu_ep_* and k3gpu_moe_layer_ep calls take. cap: the most token rows
    a rank sends in one exchange step."""

    def __init__(self, k3, cap, L, K, n_local, group=None):
        import ctypes as C
        self.k3, self.C = k3, C
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.group = group
        if self.world > k3.EP_MAX_WORLD:
            raise ValueError(f"at most {k3.EP_MAX_WORLD} ranks")
        lib = k3.lib
        nbytes = lib.k3gpu_ep_arena_bytes(self.world, cap, L, K)
        arena = C.c_void_p()
        k3.check(lib.k3gpu_ep_arena_alloc(C.byref(arena), nbytes), "k3gpu_ep_arena_alloc")
        self.arena = arena
        h = (C.c_uint8 * k3.EP_HANDLE_BYTES)()
        k3.check(lib.k3gpu_ep_ipc_handle(arena, h), "k3gpu_ep_ipc_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h), group=group)
        g = k3.K3GpuEpGroup()
        g.world, g.rank, g.cap, g.L, g.K, g.n_local = self.world, self.rank, cap, L, K, n_local
        self.peers = []
        for r in range(self.world):
            if r == self.rank:
                g.arena[r] = arena.value
                continue
            hb = (C.c_uint8 * k3.EP_HANDLE_BYTES).from_buffer_copy(handles[r])
            peer = C.c_void_p()
            k3.check(lib.k3gpu_ep_ipc_open(hb, C.byref(peer)), "k3gpu_ep_ipc_open")
            g.arena[r] = peer.value
            self.peers.append(peer)
        self.desc = g
        # every rank's arena exists and is mapped before the first dispatch writes into it
        dist.barrier(group=group)

    def close(self):
        """Unmap the peers' arenas and free this rank's, after a barrier (no rank still
        writes into it)."""
        import torch
        lib = self.k3.lib
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self.peers:
            lib.k3gpu_ep_ipc_close(p)
        self.peers = []
        if self.arena is not None:
            lib.k3gpu_ep_arena_free(self.arena)
            self.arena = None


class P2PMoELayer:
    """The routed experts sharded across `group`, token rows exchanged through peer memory
    by the library's k3gpu_ep_* kernels (no collective on the data path).

    cap: the most token rows one rank sends in a step (its token count bound)."""

    def __init__(self, k3, bank_local, shared_bank, gate_W, bias, n_routed, topk, act, cap, b1=4.0, b2=25.0,
                 renorm=1, routed_scale=1.0, group=None, stream=None):
        import ctypes as C
        self.k3, self.C = k3, C
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_routed % self.world:
            raise ValueError(f"{n_routed} routed experts do not split over {self.world} ranks")
        if self.world > k3.EP_MAX_WORLD:
            raise ValueError(f"at most {k3.EP_MAX_WORLD} ranks")
        self.n_local = n_routed // self.world
        self.topk, self.act, self.b1, self.b2 = topk, act, b1, b2
        self.renorm, self.routed_scale = renorm, routed_scale
        self.bank_local, self.shared_bank = bank_local, shared_bank
        self.gate_W, self.bias, self.stream = gate_W, bias, stream
        self.cap, self.L = cap, bank_local.L
        lib = k3.lib
        nbytes = lib.k3gpu_ep_arena_bytes(self.world, cap, self.L, topk)
        arena = C.c_void_p()
        k3.check(lib.k3gpu_ep_arena_alloc(C.byref(arena), nbytes), "k3gpu_ep_arena_alloc")
        self.arena = arena
        h = (C.c_uint8 * k3.EP_HANDLE_BYTES)()
        k3.check(lib.k3gpu_ep_ipc_handle(arena, h), "k3gpu_ep_ipc_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h), group=group)
        g = k3.K3GpuEpGroup()
        g.world, g.rank, g.cap, g.L, g.K, g.n_local = self.world, self.rank, cap, self.L, topk, self.n_local
        self.peers = []
        for r in range(self.world):
            if r == self.rank:
                g.arena[r] = arena.value
                continue
            hb = (C.c_uint8 * k3.EP_HANDLE_BYTES).from_buffer_copy(handles[r])
            peer = C.c_void_p()
            k3.check(lib.k3gpu_ep_ipc_open(hb, C.byref(peer)), "k3gpu_ep_ipc_open")
            g.arena[r] = peer.value
            self.peers.append(peer)
        self.group_desc = g
        xr, ir, wr = C.c_void_p(), C.c_void_p(), C.c_void_p()
        k3.check(lib.k3gpu_ep_recv_views(C.byref(g), C.byref(xr), C.byref(ir), C.byref(wr)), "k3gpu_ep_recv_views")
        self.views = (xr, ir, wr)
        dev = gate_W.device
        self.pos = torch.empty(self.world * cap, dtype=torch.int32, device=dev)
        self.ok = torch.empty(self.world, dtype=torch.int32, device=dev)
        self.part = torch.empty((self.world * cap, self.L), dtype=torch.float32, device=dev)
        self.ws = k3.workspace(lib.k3gpu_moe_workspace(self.world * cap, topk, 0, self.L, bank_local.I,
                                                       self.n_local), dev)
        self.seq = 0
        # every rank's arena exists and is mapped before the first dispatch writes into it
        dist.barrier(group=group)

    def forward(self, x: torch.Tensor):
        """x [T][L] fp32 (T <= cap) -> (out [T][L], idx, wt)."""
        k3, C, lib = self.k3, self.C, self.k3.lib
        T = x.shape[0]
        if T > self.cap:
            raise ValueError(f"{T} tokens exceed the exchange capacity {self.cap}")
        self.seq += 1
        seq = self.seq
        g = C.byref(self.group_desc)
        sp = k3.stream_ptr(self.stream)
        idx, wt = k3.router(x, self.gate_W, self.bias, self.topk, self.renorm, self.routed_scale, stream=self.stream)
        k3.check(lib.k3gpu_ep_dispatch(g, k3.ptr(x), k3.ptr(idx), k3.ptr(wt), T, seq, k3.ptr(self.pos), sp),
                 "k3gpu_ep_dispatch")
        # the shared experts on this rank's own tokens while the rows travel
        if self.shared_bank is not None:
            ns = self.shared_bank.n_experts
            sidx = torch.arange(ns, device=x.device, dtype=torch.int32).repeat(T, 1)
            swt = torch.ones((T, ns), device=x.device, dtype=torch.float32)
            out = k3.moe_experts(x, sidx, swt, self.shared_bank, ns, ns, 0, self.act, self.b1, self.b2,
                                 stream=self.stream)
        else:
            out = torch.zeros_like(x)
        k3.check(lib.k3gpu_ep_receive(g, seq, sp), "k3gpu_ep_receive")
        xr, ir, wr = self.views
        k3.moe_experts_ptrs(self.part, xr, ir, wr, self.world * self.cap, self.bank_local, self.topk, self.n_local,
                            0, self.act, self.b1, self.b2, ws=self.ws, stream=self.stream)
        k3.check(lib.k3gpu_ep_return(g, k3.ptr(self.part), seq, sp), "k3gpu_ep_return")
        k3.check(lib.k3gpu_ep_combine(g, k3.ptr(out), k3.ptr(self.pos), T, seq, k3.ptr(self.ok), sp),
                 "k3gpu_ep_combine")
        return out, idx, wt

    __call__ = forward

    def owners_ok(self):
        """Per owner rank, whether its rows of the last step arrived (host list; waits for
        the step). A 0 means that owner's bounded wait ran out and its contribution is
        missing from the output (k3gpu_device_status also holds the timeout bit)."""
        return self.ok.tolist()

    def close(self):
        """Unmap the peers' arenas and free this rank's (after a barrier, so no rank still
        writes into it)."""
        lib = self.k3.lib
        torch.cuda.synchronize()
        dist.barrier()
        for p in self.peers:
            lib.k3gpu_ep_ipc_close(p)
        self.peers = []
        if self.arena is not None:
            lib.k3gpu_ep_arena_free(self.arena)
            self.arena = None
