"""A conversation's carried state to and from a K3ST file (host side): the engine's
--save-state / --load-state (src/cli/k3_run.c:162-407) for this library's state.

The file holds, per KDA slot, kper floats in the layout this library keeps on the device
for one sequence ([H][D][D] recurrent state, then the ShortConv history [3][P][K-1]), and
per MLA layer the cache rows as fp32. This library caches MLA rows as bf16, so saving
widens them (exact) and loading narrows the file's fp32 rows back to bf16 by rounding to
nearest even: exact for a file this library wrote; a file the reference engine wrote
holds fp32 rows, and `inexact` reports how many values the rounding changed.

Arrays may be numpy arrays or (CPU or CUDA) torch tensors; bf16 rows are bit patterns
(uint16, or int16 as torch carries them). `k3` is the package module.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np


def _host(a, dtype=None):
    if hasattr(a, "detach"):                      # a torch tensor
        a = a.detach().cpu().numpy()
    a = np.ascontiguousarray(a)
    return a.view(dtype) if dtype is not None and a.dtype != dtype and a.dtype.itemsize == np.dtype(dtype).itemsize \
        else a


def _widen(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _narrow(x):
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def save_state(k3, path, layout, seq, cached, kda_slots, mla_lat, mla_rope, kv_cap, pcached=None, passes=None):
    """Write the state after `cached` positions of `seq` (cached or cached + 1 ids).
    kda_slots: one array of layout.kper floats per slot (n_bound, or the loop's nv);
    mla_lat / mla_rope: one bf16 array [kv_cap][kvpp] / [kv_cap][ropepp] per MLA layer."""
    ks = np.concatenate([_host(s, np.float32).reshape(-1).astype(np.float32) for s in kda_slots]) \
        if kda_slots else np.zeros(1, np.float32)
    nm = layout.n_mla
    kvc = np.zeros((max(nm, 1), kv_cap, layout.kvpp), np.float32)       # [n_mla][kv_cap][kvpp], as read
    ropec = np.zeros((max(nm, 1), kv_cap, layout.ropepp), np.float32)
    for i in range(nm):
        kvc[i] = _widen(_host(mla_lat[i], np.uint16).reshape(kv_cap, layout.kvpp))
        ropec[i] = _widen(_host(mla_rope[i], np.uint16).reshape(kv_cap, layout.ropepp))
    s = np.asarray(seq, np.int32)
    pc = np.asarray(pcached, np.int32) if pcached is not None else None
    ps = np.asarray(passes, np.int32) if passes is not None else None
    st = k3.lib.k3_state_save(os.fsencode(path), C.byref(layout), s.ctypes.data, len(s), cached, ks.ctypes.data,
                              kvc.ctypes.data, ropec.ctypes.data, kv_cap, pc.ctypes.data if pc is not None else None,
                              ps.ctypes.data if ps is not None else None)
    k3.check(st, "k3_state_save")


def load_state(k3, path, layout, seq_cap, kv_cap):
    """Read a state written for `layout` (refused otherwise, as the engine refuses it).
    Returns {"seq", "cached", "kda_slots" (float32 [kper] each), "mla_lat", "mla_rope"
    (bf16 bits [kv_cap][kvpp] / [kv_cap][ropepp]), "inexact", "pcached", "passes"}."""
    slots = layout.loop_nv if layout.loop_count else layout.n_bound
    seq = np.zeros(seq_cap, np.int32)
    ks = np.zeros(max(slots * layout.kper, 1), np.float32)
    nm = layout.n_mla
    kvc = np.zeros((max(nm, 1), kv_cap, layout.kvpp), np.float32)
    ropec = np.zeros((max(nm, 1), kv_cap, layout.ropepp), np.float32)
    pc = np.zeros(max(layout.loop_count + 1, 1), np.int32)
    ps = np.zeros(seq_cap, np.int32)
    cached, nseq = C.c_int(0), C.c_int(0)
    st = k3.lib.k3_state_load(os.fsencode(path), C.byref(layout), seq.ctypes.data, seq_cap, ks.ctypes.data,
                              kvc.ctypes.data, ropec.ctypes.data, kv_cap, pc.ctypes.data, ps.ctypes.data,
                              C.byref(cached), C.byref(nseq))
    k3.check(st, "k3_state_load")
    n = cached.value
    out = {"seq": seq[:nseq.value].tolist(), "cached": n,
           "kda_slots": [ks[i * layout.kper:(i + 1) * layout.kper].copy() for i in range(slots)],
           "mla_lat": [], "mla_rope": [], "inexact": 0,
           "pcached": pc[:layout.loop_count + 1].tolist() if layout.loop_count else None,
           "passes": ps[:nseq.value].tolist() if layout.loop_count else None}
    for i in range(nm):
        for key, arr in (("mla_lat", kvc), ("mla_rope", ropec)):
            x = np.ascontiguousarray(arr[i])
            b = _narrow(x)
            out["inexact"] += int(np.count_nonzero(_widen(b)[:n] != x[:n]))
            out[key].append(b)
    return out
