"""The C-ABI library without a GPU: it loads, exports every function include/k3gpu.h
declares, rejects bad arguments before touching CUDA, and its host-side pieces (bank
layout, n-gram drafter) agree with the oracle. No compute call reaches a device here."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

from oracle import oracle as O
from tests import k3lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "k3gpu.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"\b(k3gpu_\w+|k3_\w+)\s*\(", src)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    m = k3lib.load()
    out = subprocess.run(["nm", "-D", "--defined-only", m.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (\w+)$", out, flags=re.M))
    want = declared_functions()
    assert len(want) >= 20
    missing = [n for n in want if n not in exported]
    assert not missing, f"declared but not exported: {missing}"


def test_bank_layout_matches_oracle_layout():
    m = k3lib.load()
    for L, I in ((7168, 2048), (512, 256), (64, 64), (3584, 3072)):
        d = m.ExpertBank.layout(L, I)
        lay = O.bank_layout(L, I)
        assert [d.p1, d.s1, d.p2, d.s2, d.p3, d.s3, d.stride] == lay.tolist()
        assert d.L == L and d.I == I
        for off in (d.p1, d.p2, d.p3, d.stride):
            assert off % 16 == 0


def test_argument_checks_need_no_device():
    m = k3lib.load()
    lib = m.lib
    assert lib.k3gpu_router(None, None, None, None, None, 1, 8, 8, 2, 1, 1.0, None, 0, None) == m.K3GPU_EINVAL
    bank = m.K3GpuExpertBank()
    assert lib.k3gpu_moe_experts(None, None, None, None, C.byref(bank), 1, 2, 8, 0, 0, 4.0, 25.0,
                                 None, 1e-5, None, 0, None) == m.K3GPU_EINVAL
    assert lib.k3gpu_kda_verify(None, None, None, None, None, None, None, 1, 1, 1, 128, 1.0, None) == m.K3GPU_EINVAL
    # a bad head dim is refused even with (fake, never dereferenced) pointers
    p = C.c_void_p(16)
    assert lib.k3gpu_kda_verify(p, p, p, p, p, p, p, 1, 4, 2, 100, 1.0, None) == m.K3GPU_EINVAL
    assert lib.k3gpu_accept_sample(p, p, p, p, None, 1, 4, 10, 0.0, 1, 0, None) == m.K3GPU_EINVAL
    assert lib.k3gpu_mla_absorbed(*([p] * 8), 1, 65, 4, 16, 8, 16, 512, 128, 128, 1.0, p, 0, None) == m.K3GPU_EINVAL
    # the later entry points refuse before any CUDA call too
    assert lib.k3gpu_kda_prefill(None, None, p, p, p, p, p, 1, 8, 2, 128, 1.0, None) == m.K3GPU_EINVAL
    assert lib.k3gpu_kda_prefill(p, None, p, p, p, p, p, 1, 8, 2, 48, 1.0, None) == m.K3GPU_EINVAL   # D
    assert lib.k3gpu_kda_prefill(p, None, p, p, p, p, p, 1, 0, 2, 128, 1.0, None) == m.K3GPU_EINVAL  # T
    assert lib.k3gpu_accept_tree_greedy(None, p, p, p, p, p, p, 1, 4, 16, None) == m.K3GPU_EINVAL
    assert lib.k3gpu_matmul_bf16_batch(None, 8, p, 8, p, 8, 8, 1, None, 0, None) == m.K3GPU_EINVAL
    assert lib.k3gpu_ep_dispatch(None, p, p, p, 1, 1, p, None) == m.K3GPU_EINVAL
    assert lib.k3gpu_ep_arena_bytes(0, 16, 64, 8) == 0
    big_t = 524288 // 384 + 1                           # K3GPU_ROUTER_NOALLOC_MAX_SCORES
    assert lib.k3gpu_router_noalloc(p, p, p, p, p, big_t, 7168, 384, 8, 1, 1.0, None) == m.K3GPU_ECAPACITY
    assert lib.k3gpu_router_workspace(16, 384) >= 16 * 384 * 4
    assert lib.k3gpu_moe_workspace(72, 8, 1, 7168, 2048, 384) > 72 * 9 * 7168 * 4
    assert m.lib.k3gpu_strerror(m.K3GPU_ECAPACITY).decode().startswith("capacity")


@pytest.mark.parametrize("seed", range(40))
def test_host_drafter_matches_oracle(seed):
    m = k3lib.load()
    rng = np.random.default_rng(seed)
    # small alphabets make repeated n-grams (and disagreeing histories) common
    seq = rng.integers(0, 3 + seed % 5, size=int(rng.integers(1, 60))).astype(np.int32).tolist()
    for (nmax, nmin, cap) in ((4, 3, 8), (3, 3, 16), (4, 3, 2)):
        out = np.zeros(cap, np.int32)
        nd = O.orc().orc_spec_draft(np.asarray(seq, np.int32), len(seq), cap, nmax, nmin, out)
        assert m.spec_draft(seq, cap, nmax, nmin) == out[:nd].tolist()


def test_ep_arena_holds_every_region():
    """The expert-parallel exchange arena (k3gpu_ep_arena_bytes), host arithmetic only: a
    4 KiB header, then per source rank `cap` received rows [L] fp32, their expert ids and
    weights [K], and the returned partial rows [L] fp32, each region 256-byte aligned;
    refused sizes give 0."""
    m = k3lib.load()
    a256 = lambda n: (n + 255) // 256 * 256   # noqa: E731
    for world, cap, L, K in ((2, 64, 7168, 8), (8, 72, 7168, 8), (1, 1, 32, 1), (3, 17, 100, 3)):
        want = 4096 + 2 * a256(world * cap * L * 4) + 2 * a256(world * cap * K * 4)
        assert m.lib.k3gpu_ep_arena_bytes(world, cap, L, K) == want
    assert m.lib.k3gpu_ep_arena_bytes(9, 64, 7168, 8) == 0          # above K3GPU_EP_MAX_WORLD
    assert m.lib.k3gpu_ep_arena_bytes(2, 0, 7168, 8) == 0


def test_shim_exports_the_reference_names():
    """libk3shim.so carries the reference's own host-pointer names over the GPU kernels (the
    op-suite build the same without k3_router), resolving to the library's C ABI."""
    m = k3lib.load()
    pkg = os.path.dirname(m.LIB_PATH)
    for lib, names in (("libk3shim.so", ["k3_router", "k3_rmsnorm", "k3_attn_res", "k3_kda_step",
                                          "k3_mxfp4_dequant"]),
                       ("libk3shim_ops.so", ["k3_rmsnorm", "k3_attn_res", "k3_kda_step", "k3_mxfp4_dequant"])):
        out = subprocess.run(["nm", "-D", "--defined-only", os.path.join(pkg, lib)], capture_output=True, text=True,
                             check=True).stdout
        exported = set(re.findall(r" T (\w+)$", out, flags=re.M))
        assert set(names) <= exported, (lib, sorted(exported))
        if lib == "libk3shim_ops.so":
            assert "k3_router" not in exported
        C.CDLL(os.path.join(pkg, lib))      # loads, its dependency on libk3gpu.so resolves
