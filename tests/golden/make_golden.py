"""Generate the golden fixtures under tests/golden/ (run here, where the reference exists).

Two sources, both the reference's own:

1. ``ops_fixtures.npz`` / ``mxfp4_fixture.npz`` -- the reference's checked-in golden
   vectors (``tests/fixtures/ops/*.json`` emitted by its torch oracle, and
   ``tests/fixtures/mxfp4.json`` holding released-checkpoint MXFP4 bytes), converted to
   compact numpy arrays so that the tests run without the reference tree.

2. ``ref_*.npz`` -- outputs of the reference engine's own C kernels
   (``oracle/_ref/libk3ref.so``, compiled from the reference's ``src/core/k3_ops.c`` by
   ``oracle/Makefile``) on seeded inputs. Only the seeds, the shapes and the OUTPUTS are
   stored; the tests regenerate the inputs from the seeds with numpy's PCG64 (stable
   across numpy versions), so large inputs never enter the repository.

Usage: python tests/golden/make_golden.py [--ref <path of the reference checkout>]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_dir():
    """K3_REFERENCE, else a checkout named `reference` beside this repository."""
    return os.environ.get("K3_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402
from tests.golden import inputs as GI  # noqa: E402


def arr(d, key, dtype=np.float32):
    v = d[key]
    return np.asarray(v["data"], dtype=dtype).reshape(v["shape"])


def convert_fixtures(ref: str) -> None:
    ops = os.path.join(ref, "tests", "fixtures", "ops")
    out = {}
    for name in ("router", "kda_recur1", "kda_recur8", "kda_decay", "shortconv", "situ_glu",
                 "rmsnorm", "attnres", "mla", "moe", "kda_layer1", "kda_layer8"):
        d = json.load(open(os.path.join(ops, name + ".json")))
        for k, v in d.items():
            if isinstance(v, dict) and "data" in v:
                out[f"{name}/{k}"] = arr(d, k)
            elif isinstance(v, (int, float)):
                out[f"{name}/{k}"] = np.asarray(v)
            elif isinstance(v, list) and v and isinstance(v[0], (int, float)):
                out[f"{name}/{k}"] = np.asarray(v)
    np.savez_compressed(os.path.join(HERE, "ops_fixtures.npz"), **out)

    d = json.load(open(os.path.join(ref, "tests", "fixtures", "mxfp4.json")))
    np.savez_compressed(
        os.path.join(HERE, "mxfp4_fixture.npz"),
        packed=arr(d, "packed", np.float32).astype(np.uint8),
        scales=arr(d, "scales", np.float32).astype(np.uint8),
        expected=arr(d, "expected"),
        swapped_first64=np.asarray(d["expected_swapped_nibbles"]["first64"], np.float32),
        rows=np.asarray(d["rows"]), logical_width=np.asarray(d["logical_width"]))


def gen_router(lib) -> None:
    """k3_router on benchmark config-2 shapes (384 x 7168, top-8) and a near-tie stress."""
    res = {}
    for case in GI.ROUTER_CASES:
        x, W, bias = GI.router_inputs(case)
        idx, w = O.router(x, W, bias, case["topk"], lib=lib)
        res[case["name"] + "/idx"] = idx
        res[case["name"] + "/w"] = w
    np.savez_compressed(os.path.join(HERE, "ref_router.npz"), **res)


def gen_mxfp4(lib) -> None:
    """k3_matmul_mxfp4 (reference) on a seeded expert matrix at K3 width."""
    res = {}
    for case in GI.MXFP4_CASES:
        packed, scales, x = GI.mxfp4_inputs(case)
        R, K = case["rows"], case["in"]
        y = np.zeros(R, np.float32)
        lib.k3_matmul_mxfp4(y, x, packed, scales, K, R, 32)
        res[case["name"] + "/y"] = y
    np.savez_compressed(os.path.join(HERE, "ref_mxfp4.npz"), **res)


def gen_kda(lib) -> None:
    """k3_kda_step (reference) chained over a verify chunk, then commits of every length:
    the bit-exact pins for the KDA verify and commit kernels."""
    res = {}
    for case in GI.KDA_CASES:
        st0, q, k, v, al, be = GI.kda_inputs(case)
        T, H, D = q.shape
        qs = np.float32(1.0) / np.sqrt(np.float32(D))
        o = np.zeros((T, H, D), np.float32)
        for h in range(H):
            S = st0[h].copy()
            for t in range(T):
                ot = np.zeros(D, np.float32)
                qh = (q[t, h] * qs).astype(np.float32)
                lib.k3_kda_step(S, ot, qh, np.ascontiguousarray(k[t, h]),
                                np.ascontiguousarray(v[t, h]), np.ascontiguousarray(al[t, h]),
                                float(be[t, h]), D, D)
                o[t, h] = ot
        res[case["name"] + "/o"] = o
        zq = np.zeros(D, np.float32)
        for n in case["commits"]:
            S = st0.copy()
            for h in range(H):
                Sh = np.ascontiguousarray(S[h])
                for t in range(n):
                    lib.k3_kda_step(Sh, np.zeros(D, np.float32), zq,
                                    np.ascontiguousarray(k[t, h]), np.ascontiguousarray(v[t, h]),
                                    np.ascontiguousarray(al[t, h]), float(be[t, h]), D, D)
                S[h] = Sh
            res[case["name"] + f"/state_n{n}"] = S
    np.savez_compressed(os.path.join(HERE, "ref_kda.npz"), **res)


# -- the reference's k3_moe with an in-memory MXFP4 expert source (its own test pattern,
#    tests/unit/test_ops.c:784 mem_get), on a small LatentMoE --------------------------
class K3Cfg(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_layers", C.c_int), ("vocab", C.c_int),
                ("rms_eps", C.c_float), ("kda_heads", C.c_int), ("kda_head_dim", C.c_int),
                ("conv_k", C.c_int), ("gate_lb", C.c_float), ("n_heads", C.c_int),
                ("q_lora", C.c_int), ("kv_lora", C.c_int), ("qk_nope", C.c_int),
                ("qk_rope", C.c_int), ("v_head", C.c_int), ("mla_out_gate", C.c_int),
                ("n_experts", C.c_int), ("topk", C.c_int), ("n_shared", C.c_int),
                ("latent", C.c_int), ("moe_inter", C.c_int), ("routed_scale", C.c_float),
                ("moe_renorm", C.c_int), ("latent_norm", C.c_int), ("first_dense", C.c_int),
                ("dense_inter", C.c_int), ("attn_res_block", C.c_int),
                ("attn_res_extra", C.c_int), ("situ_b1", C.c_float), ("situ_b2", C.c_float),
                ("n_full_attn", C.c_int), ("full_attn", C.POINTER(C.c_int))]


class K3ExpertQ(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("p1", "s1", "p3", "s3", "p2", "s2")]


class K3ExpertSrc(C.Structure):
    pass


GETF = C.CFUNCTYPE(C.c_int, C.POINTER(K3ExpertSrc), C.c_int, C.c_int, C.POINTER(K3ExpertQ))
K3ExpertSrc._fields_ = [("get", GETF), ("getmany", C.c_void_p), ("resident", C.c_void_p),
                        ("ctx", C.c_void_p)]


class K3MoeW(C.Structure):
    _fields_ = [("gate", C.c_void_p), ("bias", C.c_void_p), ("w1", C.c_void_p),
                ("w3", C.c_void_p), ("w2", C.c_void_p), ("latent_norm", C.c_void_p),
                ("down", C.c_void_p), ("up", C.c_void_p), ("sh1", C.c_void_p),
                ("sh3", C.c_void_p), ("sh2", C.c_void_p), ("wdt", C.c_int),
                ("src", C.POINTER(K3ExpertSrc)), ("layer", C.c_int), ("cache_only", C.c_int)]


def gen_moe(lib) -> None:
    p = GI.latent_moe_inputs()
    cfg = K3Cfg()
    cfg.hidden, cfg.rms_eps = p["E"], 1e-5
    cfg.n_experts, cfg.topk, cfg.n_shared = p["n_experts"], p["topk"], p["n_shared"]
    cfg.latent, cfg.moe_inter = p["L"], p["I"]
    cfg.routed_scale, cfg.moe_renorm, cfg.latent_norm = 1.0, 1, 1
    cfg.situ_b1, cfg.situ_b2 = 4.0, 25.0
    bank, lay = p["bank"], p["lay"]
    base = bank.ctypes.data

    def get(_self, _layer, e, out):
        r = base + int(e) * int(lay[6])
        q = out.contents
        q.p1, q.s1 = r + int(lay[0]), r + int(lay[1])
        q.p2, q.s2 = r + int(lay[2]), r + int(lay[3])
        q.p3, q.s3 = r + int(lay[4]), r + int(lay[5])
        return 0

    getf = GETF(get)
    src = K3ExpertSrc(getf, None, None, None)
    keep = {k: np.ascontiguousarray(v, np.float32) for k, v in p.items()
            if k in ("gate", "bias", "latent_norm", "down", "up", "sh1", "sh3", "sh2", "x")}
    w = K3MoeW()
    for k in ("gate", "bias", "latent_norm", "down", "up", "sh1", "sh3", "sh2"):
        setattr(w, k, keep[k].ctypes.data)
    w.wdt, w.src = 0, C.pointer(src)
    lib.k3_moe_scratch.restype = C.c_size_t
    lib.k3_moe_scratch.argtypes = [C.POINTER(K3Cfg), C.c_int]
    T = p["x"].shape[0]
    scr = np.zeros(lib.k3_moe_scratch(C.byref(cfg), T), np.float32)
    out = np.zeros((T, p["E"]), np.float32)
    idx = np.zeros(64, np.int32)
    wt = np.zeros(64, np.float32)
    lib.k3_moe.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(K3MoeW), C.POINTER(K3Cfg), C.c_int,
                           C.c_void_p, C.c_void_p, C.c_void_p]
    lib.k3_moe.restype = None
    lib.k3_moe(out.ctypes.data, keep["x"].ctypes.data, C.byref(w), C.byref(cfg), T,
               idx.ctypes.data, wt.ctypes.data, scr.ctypes.data)
    np.savez_compressed(os.path.join(HERE, "ref_moe.npz"), out=out)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=reference_dir(),
                    help="the reference checkout (default: K3_REFERENCE, else `reference` beside this repository)")
    a = ap.parse_args()
    O.build()
    lib = O.ref()
    if lib is None:
        raise SystemExit("oracle/_ref/libk3ref.so was not built (reference tree missing?)")
    convert_fixtures(a.ref)
    gen_router(lib)
    gen_mxfp4(lib)
    gen_kda(lib)
    gen_moe(lib)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f"{f:24s} {os.path.getsize(os.path.join(HERE, f)):>9d} bytes")


if __name__ == "__main__":
    main()
