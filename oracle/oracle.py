"""ctypes bindings for the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Loads ``liborc.so`` (this repository's C restatement of the path, ``k3_oracle.c``) and,
when present, ``_ref/libk3ref.so`` (the reference engine's own ``src/core/k3_ops.c``,
compiled by ``oracle/Makefile``) and ``_ref/libk3ref_bench.so`` (the timed CPU baseline).
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs import this
module. The product path never does.

Also holds the numpy compositions the tests use to pin the C restatement against the
reference's whole-module fixtures (``mla.json``, ``moe.json``, ``kda_layer8.json``): each
composes orc_* kernels in the order the reference's module does, citing it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_orc = None
_ref = None
_ref4 = None
_refb = None

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")


def build() -> None:
    """Compile liborc.so (and _ref/ when the reference tree is present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def orc():
    """The restatement library, built on first use."""
    global _orc
    if _orc is None:
        path = os.path.join(HERE, "liborc.so")
        if not os.path.exists(path):
            build()
        lib = C.CDLL(path)
        I, F = C.c_int, C.c_float
        sig = {
            "orc_rmsnorm": [f32p, f32p, f32p, I, F],
            "orc_situ_glu": [f32p, f32p, I, F, F],
            "orc_swiglu": [f32p, f32p, I],
            "orc_router": [i32p, f32p, f32p, f32p, C.c_void_p, I, I, I, I, F],
            "orc_router_scores": [f32p, f32p, f32p, I, I],
            "orc_mxfp4_dequant": [f32p, u8p, u8p, I, I],
            "orc_matmul_mxfp4": [f32p, f32p, u8p, u8p, I, I],
            "orc_bank_layout": [i64p, I, I],
            "orc_expert": [f32p, f32p, u8p, i64p, I, I, I, F, F],
            "orc_moe_routed": [f32p, f32p, i32p, f32p, u8p, i64p, I, I, I, I, I, I, I, F, F,
                               C.c_void_p, F],
            "orc_kda_step": [f32p, f32p, f32p, f32p, f32p, f32p, F, I, I],
            "orc_kda_verify": [f32p, f32p, f32p, f32p, f32p, f32p, f32p, I, I, I, F],
            "orc_kda_commit": [f32p, f32p, f32p, f32p, f32p, I, I, I],
            "orc_shortconv": [f32p, f32p, f32p, C.c_void_p, I, I, I],
            "orc_l2norm": [f32p, I, F],
            "orc_kda_decay": [f32p, f32p, f32p, f32p, f32p, I, I, F],
            "orc_kda_prologue": [f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p,
                                 C.c_void_p, f32p, f32p, I, I, I, I, F],
            "orc_kda_commit_conv": [f32p, f32p, I, I, I],
            "orc_kda_norm_gate": [f32p, f32p, f32p, I, I, I, F],
            "orc_mla_absorbed": [f32p, f32p, f32p, f32p, f32p, f32p, I, I, I, I, I, I, I,
                                 u64p, F],
            "orc_attn_res": [f32p, f32p, f32p, I, I, F],
            "orc_spec_draft": [i32p, I, I, I, I, i32p],
            "orc_argmax": [f32p, I],
            "orc_accept_greedy": [i32p, C.POINTER(C.c_int), i32p, f32p, i32p, I, I],
            "orc_emit_keep": [i32p, I, I, I, I, I, C.c_void_p, I],
        }
        for name, args in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = None
        lib.orc_accept_tree_greedy.argtypes = [i32p, i32p, f32p, i32p, i32p, I, I]
        lib.orc_accept_tree_greedy.restype = C.c_int
        lib.orc_philox_uniform.argtypes = [C.c_uint64, C.c_uint64, I, I, I]
        lib.orc_philox_uniform.restype = C.c_double
        lib.orc_accept_sample.argtypes = [i32p, f32p, i32p, I, I, F, C.c_uint64, C.c_uint64, I]
        lib.orc_accept_sample.restype = C.c_int
        lib.orc_spec_draft.restype = C.c_int
        lib.orc_argmax.restype = C.c_int
        lib.orc_accept_greedy.restype = C.c_int
        lib.orc_emit_keep.restype = C.c_int
        _orc = lib
    return _orc


def _load_ref(path):
    lib = C.CDLL(path)
    I, F = C.c_int, C.c_float
    lib.k3_router.argtypes = [i32p, f32p, f32p, f32p, C.c_void_p, I, I, I, I, F]
    lib.k3_matmul_mxfp4.argtypes = [f32p, f32p, u8p, u8p, I, I, I]
    lib.k3_mxfp4_dequant.argtypes = [f32p, u8p, u8p, I, I, I]
    lib.k3_kda_step.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, F, I, I]
    lib.k3_situ_glu.argtypes = [f32p, f32p, I, F, F]
    lib.k3_rmsnorm.argtypes = [f32p, f32p, f32p, I, F]
    lib.k3_shortconv.argtypes = [f32p, f32p, f32p, C.c_void_p, I, I, I]
    lib.k3_kda_decay.argtypes = [f32p, f32p, f32p, f32p, f32p, I, I, F]
    lib.k3_matmul_bf16_batch_ld.argtypes = [f32p, I, f32p, I, C.c_void_p, I, I, I]
    for n in ("k3_router", "k3_matmul_mxfp4", "k3_mxfp4_dequant", "k3_kda_step",
              "k3_situ_glu", "k3_rmsnorm", "k3_shortconv", "k3_kda_decay",
              "k3_matmul_bf16_batch_ld"):
        getattr(lib, n).restype = None
    return lib


def ref():
    """The reference engine's own numeric core (the x86-64-v3 build the parity checks use),
    or None when it was not built here."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libk3ref.so")
        if not os.path.exists(path):
            return None
        _ref = _load_ref(path)
    return _ref


def ref_timed():
    """The build of the reference's numeric core that the timed CPU baselines call: the
    x86-64-v4 one (its AVX-512 paths) when ref_bench_isa() picks it, else ref()."""
    global _ref4
    if ref_bench_isa() != "v4":
        return ref()
    if _ref4 is None:
        _ref4 = _load_ref(os.path.join(HERE, "_ref", "v4", "libk3ref4.so"))
    return _ref4


def ref_v4_if_runnable():
    """The x86-64-v4 build of the numeric core when it was built and this host runs it
    (for holding it to the v3 build), else None."""
    global _ref4
    path = os.path.join(HERE, "_ref", "v4", "libk3ref4.so")
    if not (os.path.exists(path) and host_has_x86_64_v4()):
        return None
    if _ref4 is None:
        _ref4 = _load_ref(path)
    return _ref4


V4_FLAGS = ("avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl")


def host_has_x86_64_v4():
    """True when this host's CPU reports the AVX-512 subsets of x86-64-v4 (/proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    have = set(line.split(":", 1)[1].split())
                    return all(x in have for x in V4_FLAGS)
    except OSError:
        pass
    return False


def ref_bench_isa(variant=None):
    """Which build of the timed reference baselines ref_bench() loads: "v4" (the reference's
    AVX-512 paths) when the host has them and _ref/v4 was built, else "v3" (AVX2 + FMA).
    K3_REF_ISA=v3 or v4 forces one (v4 only where the host runs it)."""
    want = variant or os.environ.get("K3_REF_ISA", "")
    v4 = os.path.join(HERE, "_ref", "v4", "libk3ref_bench.so")
    if want == "v3":
        return "v3"
    if os.path.exists(v4) and host_has_x86_64_v4():
        return "v4"
    return "v3"


ISA_TEXT = {"v3": "x86-64-v3 (AVX2 + FMA)", "v4": "x86-64-v4 (AVX-512: the reference's __AVX512F__ paths)"}


def ref_bench_path(variant=None):
    isa = ref_bench_isa(variant)
    return os.path.join(HERE, "_ref", "v4", "libk3ref_bench.so") if isa == "v4" else \
        os.path.join(HERE, "_ref", "libk3ref_bench.so")


def ref_bench():
    """The reference-kernel CPU baseline harness (the build ref_bench_isa() names), or None
    when it was not built here."""
    global _refb
    if _refb is None:
        path = ref_bench_path()
        if not os.path.exists(path):
            return None
        lib = C.CDLL(path)
        I, F = C.c_int, C.c_float
        lib.ref_moe_layer.argtypes = [f32p, i32p, f32p, f32p, f32p, C.c_void_p, u8p, i64p,
                                      I, I, I, I, I, I, I, F, F, I]
        lib.ref_moe_layer.restype = C.c_int
        _refb = lib
    return _refb


# ------------------------------------------------------------------ thin wrappers --

def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def router(x, W, bias, topk, renorm=1, scale=1.0, lib=None):
    """Route every row of x: (idx [T][topk] int32, w [T][topk] float32)."""
    lib = lib or orc()
    x, W = _f(x), _f(W)
    T, E = x.shape
    n = W.shape[0]
    idx = np.zeros((T, topk), np.int32)
    w = np.zeros((T, topk), np.float32)
    b = _f(bias) if bias is not None else None
    fn = lib.orc_router if lib is orc() else lib.k3_router
    for t in range(T):
        it = np.zeros(topk, np.int32)
        wt = np.zeros(topk, np.float32)
        fn(it, wt, np.ascontiguousarray(x[t]), W,
           b.ctypes.data_as(C.c_void_p) if b is not None else None, E, n, topk, renorm,
           float(scale))
        idx[t], w[t] = it, wt
    return idx, w


def bank_layout(L, I):
    lay = np.zeros(7, np.int64)
    orc().orc_bank_layout(lay, L, I)
    return lay


def mxfp4_quant(w: np.ndarray):
    """Quantise [R][C] fp32 to (packed [R][C/2] u8, scales [R][C/32] u8) by the rule of
    the reference's tiny-checkpoint generator (tools/make_tiny_checkpoint.py:88-138):
    scale = 2^(floor(log2 amax) - 2) per 32, nibble = nearest E2M1 magnitude (argmin,
    first index on ties), sign from the element, low nibble = even element."""
    w = np.asarray(w, np.float32)
    R, Cc = w.shape
    g = Cc // 32
    blocks = w.reshape(R, g, 32)
    amax = np.abs(blocks).max(axis=2)
    ex = (np.floor(np.log2(np.maximum(amax, 1e-30))) - 2).astype(np.int32)
    ex = np.clip(ex, -127, 127)
    scales = (ex + 127).astype(np.uint8)
    mult = np.exp2(ex.astype(np.float32)).reshape(R, g, 1)
    xq = blocks / mult
    # nearest of {0, .5, 1, 1.5, 2, 3, 4, 6} with ties to the lower code: the count of
    # midpoints strictly below |xq| (each |xq - lut| the argmin compares is exact in fp32,
    # so this equals the generator's argmin, first index on ties)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    idx = np.searchsorted(mids, np.abs(xq).ravel(), side="left").astype(np.uint8).reshape(xq.shape)
    nib = np.where(xq < 0, idx | 0x8, idx).astype(np.uint8)
    packed = (nib[:, :, 0::2] | (nib[:, :, 1::2] << 4)).reshape(R, Cc // 2)
    return np.ascontiguousarray(packed), np.ascontiguousarray(scales)


def make_bank(rng, n_experts, L, I, std=0.02, w13_std=None):
    """A contiguous MXFP4 expert bank in the reference's per-expert run layout."""
    lay = bank_layout(L, I)
    stride = int(lay[6])
    bank = np.zeros(n_experts * stride, np.uint8)
    for e in range(n_experts):
        base = e * stride
        s13 = w13_std if w13_std is not None else std
        for (po, so, rows, cols, sd) in ((lay[0], lay[1], I, L, s13), (lay[2], lay[3], L, I, std),
                                         (lay[4], lay[5], I, L, s13)):
            w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(sd)
            p, s = mxfp4_quant(w)
            bank[base + po: base + po + p.size] = p.ravel()
            bank[base + so: base + so + s.size] = s.ravel()
    return bank, lay


def moe_routed(z, idx, wt, bank, lay, L, I, topk, n_routed, n_shared, act, b1=4.0, b2=25.0,
               latent_norm=None, eps=1e-5):
    z = _f(z)
    T = z.shape[0]
    acc = np.zeros((T, L), np.float32)
    ln = _f(latent_norm) if latent_norm is not None else None
    orc().orc_moe_routed(acc, z, np.ascontiguousarray(idx, np.int32), _f(wt), bank, lay, T, L,
                         I, topk, n_routed, n_shared, act, float(b1), float(b2),
                         ln.ctypes.data_as(C.c_void_p) if ln is not None else None, float(eps))
    return acc


def kda_verify(state, q, k, v, alpha, beta, qscale):
    T, H, D = q.shape
    o = np.zeros((T, H, D), np.float32)
    orc().orc_kda_verify(o, _f(state), _f(q), _f(k), _f(v), _f(alpha), _f(beta), T, H, D,
                         float(qscale))
    return o


def kda_commit(state, k, v, alpha, beta, n):
    st = _f(state).copy()
    H, D = st.shape[0], st.shape[1]
    orc().orc_kda_commit(st, _f(k), _f(v), _f(alpha), _f(beta), int(n), H, D)
    return st


def mla_absorbed(q_nope, q_rope, kv_b, lat, rope, cached, mask, scale, vh):
    T, H, qn = q_nope.shape
    qr = q_rope.shape[2]
    kvl = lat.shape[1]
    out = np.zeros((T, H, vh), np.float32)
    orc().orc_mla_absorbed(out, _f(q_nope), _f(q_rope), _f(kv_b), _f(lat), _f(rope), T, H, qn,
                           qr, vh, kvl, int(cached),
                           np.ascontiguousarray(mask, np.uint64), float(scale))
    return out


def chain_masks(T):
    """Causal chain: query t sees new rows 0..t."""
    return np.array([(1 << (t + 1)) - 1 for t in range(T)], np.uint64)


def tree_masks(parent):
    """Ancestor masks for a draft tree given parent[i] (-1 for the root): node i sees
    itself and every ancestor."""
    T = len(parent)
    m = np.zeros(T, np.uint64)
    for i in range(T):
        bits, j = 0, i
        while j >= 0:
            bits |= 1 << j
            j = parent[j]
        m[i] = bits
    return m


def rmsnorm(x, w, eps):
    x = _f(x)
    y = np.empty_like(x)
    flat, yf = x.reshape(-1, x.shape[-1]), y.reshape(-1, x.shape[-1])
    for r in range(flat.shape[0]):
        out = np.empty(flat.shape[1], np.float32)
        orc().orc_rmsnorm(out, np.ascontiguousarray(flat[r]), _f(w), flat.shape[1], float(eps))
        yf[r] = out
    return y


def matmul_bf16_ref(X, Wbits):
    """The reference's own k3_matmul_bf16_batch_ld (oracle/_ref) on X [T][in] fp32 and
    W bf16 bits [out][in] uint16, or None when oracle/_ref was not built."""
    lib = ref()
    if lib is None:
        return None
    X = _f(X)
    Wb = np.ascontiguousarray(Wbits, np.uint16)
    T, n_in = X.shape
    n_out = Wb.shape[0]
    Y = np.empty((T, n_out), np.float32)
    lib.k3_matmul_bf16_batch_ld(Y, n_out, X, n_in, Wb.ctypes.data_as(C.c_void_p), n_in, n_out, T)
    return Y


def bf16_bits_to_f32(Wbits):
    return (np.asarray(Wbits, np.uint32) << 16).view(np.float32)


def matmul_d(x, W):
    """y = W x with a double accumulator per output (the reference's fp32 k3_matmul
    contract up to its 16-accumulator partition, k3_ops.c:363-399), rounded to float."""
    return (np.asarray(x, np.float64) @ np.asarray(W, np.float64).T).astype(np.float32)


def mla_forward(x, wts, cfg):
    """The whole gated NoPE MLA of the reference's k3_mla (src/core/k3_ops.c:1115-1615)
    in absorbed form over positions 0..T-1 of one sequence: q_a -> RMSNorm -> q_b;
    kv_a -> RMSNorm on the latent (not the rope slot); the absorbed core (orc_mla_absorbed)
    with the causal chain; sigmoid output gate then o_proj. Used to pin orc_mla_absorbed
    against the reference's mla.json fixture."""
    H, qn, qr, vh, kvl = cfg["n_heads"], cfg["qk_nope"], cfg["qk_rope"], cfg["v_head"], cfg["kv_lora"]
    T = x.shape[0]
    ql = rmsnorm(matmul_d(x, wts["q_a"]), wts["q_a_norm"], cfg["eps"])
    q = matmul_d(ql, wts["q_b"]).reshape(T, H, qn + qr)
    ct = matmul_d(x, wts["kv_a"])
    lat = rmsnorm(ct[:, :kvl], wts["kv_a_norm"], cfg["eps"])
    rope = np.ascontiguousarray(ct[:, kvl:])
    scale = np.float32(1.0) / np.sqrt(np.float32(qn + qr))
    acc = mla_absorbed(np.ascontiguousarray(q[:, :, :qn]), np.ascontiguousarray(q[:, :, qn:]),
                       wts["kv_b"], lat, rope, 0, chain_masks(T), scale, vh)
    acc = acc.reshape(T, H * vh)
    if wts.get("g") is not None:
        g = matmul_d(x, wts["g"])
        acc = acc * (np.float32(1) / (np.float32(1) + np.exp(-g, dtype=np.float32)))
    return matmul_d(acc, wts["o"])


# ---------------------------------------------------------------- drafting policies ---
def eager_draft(seq, T, cap=8):
    """P1 of the reference's drafting study (tools/spec_replay.py:174-184): the most recent
    earlier occurrence of the suffix 4-gram, else 3-gram, else 2-gram, and the ids after it
    up to cap (<= 8) and the end of the history."""
    cap = min(cap, 8)
    for n in (4, 3, 2):
        if T < n + 1:
            continue
        for j in range(T - n - 1, -1, -1):
            if all(seq[j + i] == seq[T - n + i] for i in range(n)):
                return [seq[j + n + i] for i in range(cap) if j + n + i < T]
    return []


def longest_suffix_draft(seq, T, cap=8):
    """P2 of the study (tools/spec_replay.py:319-336, 442-449) by brute force: the longest
    suffix of seq[0..T) that also ends at some e <= T-2, its most recent such end, and
    seq[e + 1 + i % (T - 1 - e)] for i < cap. Returns (draft, L, g); ([], 0, 0) without a
    match."""
    best = (0, -1)
    for L in range(1, T):
        suf = list(seq[T - L:T])
        ends = [e for e in range(L - 1, T - 1) if list(seq[e - L + 1:e + 1]) == suf]
        if not ends:
            break
        best = (L, max(ends))
    L, e = best
    if L == 0:
        return [], 0, 0
    g = (T - 1) - e
    return [seq[e + 1 + (i % g)] for i in range(min(cap, 8))], L, g


def suffix_tree_draft(seq, max_nodes=64, branch=4, max_depth=8, min_len=1):
    """The draft tree of k3_suffix_drafter_tree by brute-force string counting (a tree
    extension of P2 with no counterpart in the reference, whose drafts are chains).

    Root: the pending id seq[-1]; its context is the longest suffix of the history that
    also ends earlier. A context s was followed by id c k(s, c) times (end positions
    p <= T-2 of s with seq[p+1] == c); its children are the `branch` most frequent c (ties:
    the smaller id), each with probability k / sum(k). A context never followed backs off
    to its longest proper suffix with more end positions while that suffix keeps >= min_len
    ids. Best-first by the product of probabilities (ties: the earliest candidate), up to
    max_nodes nodes and depth max_depth. Returns (tok, parent)."""
    seq = list(seq)
    T = len(seq)

    def ends(s):
        m = len(s)
        return [p for p in range(m - 1, T) if seq[p - m + 1:p + 1] == s]

    def follows(s):
        f = {}
        for p in ends(s):
            if p <= T - 2:
                f[seq[p + 1]] = f.get(seq[p + 1], 0) + 1
        return f

    def backoff(s):
        e = len(ends(s))
        for m in range(len(s) - 1, 0, -1):
            if len(ends(s[-m:])) != e:
                return s[-m:]
        return []

    tok, parent = [seq[-1]], [-1]
    L = longest_suffix_draft(seq, T, 1)[1]
    if L == 0 or L < min_len or max_depth < 1 or max_nodes <= 1:
        return tok, parent
    cand = []

    def expand(node, s, pp, depth):
        f = follows(s)
        while not f:
            b = backoff(s)
            if not b or len(b) < min_len:
                return
            s, f = b, follows(b)
        total = sum(f.values())
        for c, k in sorted(f.items(), key=lambda kv: (-kv[1], kv[0]))[:max(1, min(branch, 16))]:
            cand.append((pp * (k / total), node, c, s + [c], depth + 1))

    expand(0, seq[T - L:], 1.0, 0)
    while len(tok) < max_nodes and cand:
        best = 0
        for i in range(1, len(cand)):
            if cand[i][0] > cand[best][0]:
                best = i
        p, par, c, s, depth = cand.pop(best)
        tok.append(c)
        parent.append(par)
        if depth < max_depth:
            expand(len(tok) - 1, s, p, depth)
    return tok, parent


def emit_keep(emit, nout, gen, T, tmax, stops):
    """How many of a step's emitted ids the output keeps (src/cli/k3_run.c:1300-1317)."""
    k = 0
    while k < len(emit) and nout + k < gen and T + k < tmax:
        k += 1
        if emit[k - 1] in stops:
            return k
    return k


def spec_loop(next_id, ids, cached, policy, spec_n, min_len, gen, tmax, kv_cap, stops, tree_nodes=64,
              tree_branch=4, draft_next=None):
    """The engine's incremental speculative loop (src/cli/k3_run.c:2812-3047) over a greedy
    model given as next_id(context ids) -> id. Policies 0 none, 1 the engine's n-gram
    spec_draft, 2 P1, 3 P2, 5 a suffix draft tree (suffix_tree_draft, depth spec_n) with
    greedy tree acceptance (a child is accepted when its parent is and its id is the
    parent's next id, the lowest index first), 6 a draft model given as draft_next(context)
    proposing spec_n ids greedily (the engine's --draft, src/cli/k3_run.c:2862-2905,
    2956-2965; its draft counters: rounds, ids drafted, accepted, fed positions dropped).
    Returns (generated ids, [(nd, m, keep, fed)] per step, the engine's counters, cached,
    ids)."""
    seq = list(ids)
    out, trace = [], []
    st = dict(steps=0, sweeps=0, drafted=0, accepted=0, dropped=0, full=0, partial=0, cut=0,
              draft_rounds=0, draft_drafted=0, draft_accepted=0, draft_dropped=0)
    hist = [0] * 9
    g = 0
    while len(out) < gen or g == 0:
        base = cached
        T = len(seq)
        if g == 0:                                            # :2820-2854
            n = T - base
            emit = [next_id(seq)]
            cached = T
            keep = emit_keep(emit, len(out), gen, T, tmax, stops)
            trace.append((0, 0, keep, n))
        elif policy == 5:
            tok, par = [seq[base]], [-1]
            if T + spec_n + 1 < tmax and base + tree_nodes <= kv_cap:
                tok, par = suffix_tree_draft(seq, tree_nodes, tree_branch, spec_n, min_len)
            n = len(tok)

            def ctx_of(i):
                p = []
                while i >= 0:
                    p.append(tok[i])
                    i = par[i]
                return seq[:base] + p[::-1]
            arg = [next_id(ctx_of(i)) for i in range(n)]
            path = [0]
            while True:
                kids = [c for c in range(n) if par[c] == path[-1] and tok[c] == arg[path[-1]]]
                if not kids:
                    break
                path.append(kids[0])
            m, nd = len(path) - 1, n - 1
            emit = [tok[i] for i in path[1:]] + [arg[path[-1]]]
            keep = emit_keep(emit, len(out), gen, T, tmax, stops)
            cached = base + (keep if nd else 1)
            if nd:
                st["sweeps"] += 1
                st["drafted"] += nd
                st["accepted"] += m
                st["dropped"] += nd + 1 - keep
                st["full" if path[-1] not in par else "partial"] += 1
                st["cut"] += keep < m + 1
                hist[m] += 1
            trace.append((nd, m, keep, n))
        else:
            d = []
            if policy and T + spec_n + 1 < tmax and base + spec_n + 1 <= kv_cap:   # :2859
                if policy == 6:
                    if spec_n > 0:                            # the draft model's greedy chain
                        ctx_d = seq[:base + 1]
                        for _ in range(spec_n):
                            d.append(draft_next(ctx_d))
                            ctx_d = ctx_d + [d[-1]]
                        st["draft_rounds"] += 1
                        st["draft_drafted"] += spec_n
                elif policy == 1:
                    buf = np.zeros(max(spec_n, 1), np.int32)
                    nd = orc().orc_spec_draft(np.asarray(seq, np.int32), T, spec_n, 4, 3, buf)
                    d = buf[:nd].tolist()
                elif policy == 2:
                    d = eager_draft(seq, T, spec_n)
                elif policy == 3:
                    dd, L, _ = longest_suffix_draft(seq, T, spec_n)
                    d = dd if L >= min_len else []
            nd = len(d)
            ctx = seq[:base + 1]
            arg = []
            for i in range(nd + 1):                           # the verify sweep
                arg.append(next_id(ctx))
                if i < nd:
                    ctx = ctx + [d[i]]
            m = 0
            while m < nd and arg[m] == d[m]:
                m += 1
            emit = d[:m] + [arg[m]]
            keep = emit_keep(emit, len(out), gen, T, tmax, stops)
            cached = base + (keep if nd else 1)
            if policy == 6 and nd:                            # :2956-2965
                st["draft_accepted"] += m
                st["draft_dropped"] += nd - min(keep, nd)
            if nd:                                            # :2945-2955
                st["sweeps"] += 1
                st["drafted"] += nd
                st["accepted"] += m
                st["dropped"] += nd + 1 - keep
                st["full" if m == nd else "partial"] += 1
                st["cut"] += keep < m + 1
                hist[m] += 1
            trace.append((nd, m, keep, nd + 1))
        st["steps"] += 1
        g += 1
        seq += emit[:keep]
        out += emit[:keep]
        if keep and emit[keep - 1] in stops:
            break
        if len(seq) >= tmax:
            break
    st["hist"] = hist
    return out, trace, st, cached, seq


def kda_chunked(state, q, k, v, alpha, beta, qscale, chunk=64):
    """The chunked parallel form of the KDA recurrence, in float64: the checker for a
    chunked prefill (the reference runs only the sequential k3_kda_step,
    src/core/k3_ops.c:303-360, and records the chunked form's properties as properties of
    the algorithm, include/k3/k3.h:51-60).

    Per chunk of n positions from state S0 (rows = key channels), with g_t the cumulative
    log decay through position t and ratios r_ts = exp(g_t - g_s) <= 1 for s <= t: the
    delta-rule writes w_t = beta_t (v_t - S'_t^T k_t) solve the unit lower-triangular
    system (I + A) W = diag(beta) (V - (Gamma K) S0), A_ts = beta_t sum_i k_s k_t r_ts (s < t,
    the UT transform; Akk's diagonal is dropped); outputs o_t = S0^T (Gamma_t q_t) +
    sum_{s <= t} (sum_i k_s q_t r_ts) w_s (Aqk keeps its diagonal: the output reads the
    updated state); the next state is Gamma_n S0 + sum_s (Gamma_n / Gamma_s k_s) w_s^T.
    (The delta-rule chunking of Yang et al., "Parallelizing Linear Transformers with the
    Delta Rule over Sequence Length", NeurIPS 2024, with a per-channel decay.)
    Returns (o [T][H][D] f32, state [H][D][D] f32)."""
    T, H, D = q.shape
    S = np.asarray(state, np.float64).reshape(H, D, D).copy()
    o = np.zeros((T, H, D))
    for h in range(H):
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            n = c1 - c0
            Q = np.asarray(q[c0:c1, h], np.float64) * np.float64(np.float32(qscale))
            K = np.asarray(k[c0:c1, h], np.float64)
            V = np.asarray(v[c0:c1, h], np.float64)
            B = np.asarray(beta[c0:c1, h], np.float64)
            g = np.cumsum(np.log(np.maximum(np.asarray(alpha[c0:c1, h], np.float64), 1e-300)), axis=0)
            diff = g[:, None, :] - g[None, :, :]                       # [t][s][i]
            lower = np.tril(np.ones((n, n), bool))
            R = np.exp(np.where(lower[:, :, None], diff, -np.inf))
            Akk = np.tril(np.einsum("si,ti,tsi->ts", K, K, R), -1) * B[:, None]
            Aqk = np.einsum("si,ti,tsi->ts", K, Q, R)
            rhs = B[:, None] * (V - (K * np.exp(g)) @ S[h])
            W = np.zeros((n, D))
            for t in range(n):                                         # forward substitution
                W[t] = rhs[t] - Akk[t, :t] @ W[:t]
            o[c0:c1, h] = (Q * np.exp(g)) @ S[h] + Aqk @ W
            S[h] = np.exp(g[-1])[:, None] * S[h] + (K * np.exp(g[-1][None, :] - g)).T @ W
    return o.astype(np.float32), S.astype(np.float32)


def kda_chunked_factored_f32(state, q, k, v, alpha, beta, qscale, chunk=32, max_range=100.0):
    """The chunked KDA recurrence as a tensor-core kernel would compute it, in float32: the
    decay ratios 2^(g_t - g_s) factored about the chunk's middle position m,
    2^(g_t - g_m) * 2^(g_m - g_s), so the pair sums A = (K 2^(g - g_m)) (K 2^(g_m - g))^T and
    Aq = (Q 2^(g - g_m)) (K 2^(g_m - g))^T become plain products -- valid while no factor
    leaves float range, i.e. while the chunk's total log2 decay per channel stays within
    max_range; a chunk beyond it takes the exact per-pair form. Same algebra as
    kda_chunked otherwise. Returns (o [T][H][D], state [H][D][D]) float32."""
    T, H, D = q.shape
    f = np.float32
    S = np.asarray(state, f).reshape(H, D, D).copy()
    o = np.zeros((T, H, D), f)
    for h in range(H):
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            n = c1 - c0
            Q = np.asarray(q[c0:c1, h], f) * f(qscale)
            K = np.asarray(k[c0:c1, h], f)
            V = np.asarray(v[c0:c1, h], f)
            B = np.asarray(beta[c0:c1, h], f)
            g = np.cumsum(np.log2(np.maximum(np.asarray(alpha[c0:c1, h], f), f(1.1754944e-38))), axis=0,
                          dtype=f)
            lower = np.tril(np.ones((n, n), bool))
            if float(np.max(g[0] - g[-1])) <= max_range:
                gm = g[n // 2]
                Ka, Kb = K * np.exp2(g - gm), K * np.exp2(gm - g)
                Akk = np.tril(Ka @ Kb.T, -1) * B[:, None]
                Aqk = np.where(lower, (Q * np.exp2(g - gm)) @ Kb.T, f(0))
            else:                                   # the exact per-pair form
                R = np.exp2(np.where(lower[:, :, None], g[:, None, :] - g[None, :, :], -np.inf)).astype(f)
                Akk = np.tril(np.einsum("si,ti,tsi->ts", K, K, R), -1) * B[:, None]
                Aqk = np.einsum("si,ti,tsi->ts", K, Q, R)
            rhs = B[:, None] * (V - (K * np.exp2(g)) @ S[h])
            W = np.zeros((n, D), f)
            for t in range(n):
                W[t] = rhs[t] - Akk[t, :t] @ W[:t]
            o[c0:c1, h] = (Q * np.exp2(g)) @ S[h] + Aqk @ W
            S[h] = np.exp2(g[-1])[:, None] * S[h] + (K * np.exp2(g[-1][None, :] - g)).T @ W
    return o, S
