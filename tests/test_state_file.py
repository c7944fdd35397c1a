"""The conversation state file (k3_state_save / peek / load), CPU only.

The expected bytes are restated here from the reference's writer (src/cli/k3_run.c:
183-196 structs, :362-405 k3_state_save): a 96-byte header {"K3ST", int32 2, int32
fp[12], int32 n_bound, n_mla, cached, nseq, int64 kper, kvpp, ropepp}, the 24-byte loop
record {int32 a, b, count, nv; double eps}, ids, the loop arrays when count > 0, the KDA
slots, then every MLA layer's cache rows and every MLA layer's rope rows position-major.
The file this library writes must equal them byte for byte, and the loader must refuse
what the reference's loader refuses (:263-325).
"""
import os
import struct
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from k3lib import load  # noqa: E402

FP = [512, 4, 1000, 4, 16, 4, 2, 8, 4, 8, 16, 2]   # k3_state_fp order


@pytest.fixture(scope="module")
def k3():
    return load()


def layout(k3, n_bound=4, n_mla=2, H=4, D=16, K=4, kvl=32, qr=4, loop=(0, -1, -1, 0, -1.0)):
    P = H * D
    s = k3.K3StateLayout()
    for i, v in enumerate(FP):
        s.fp[i] = v
    s.n_bound, s.n_mla = n_bound, n_mla
    s.kper, s.kvpp, s.ropepp = P * D + 3 * P * (K - 1), kvl, qr
    s.loop_count, s.loop_a, s.loop_b, s.loop_nv, s.loop_eps = loop
    return s


def expected_bytes(s, seq, cached, ks, kvc, ropec, pcached=None, passes=None):
    b = b"K3ST" + struct.pack("<i", 2) + struct.pack("<12i", *FP)
    b += struct.pack("<4i", s.n_bound, s.n_mla, cached, len(seq)) + struct.pack("<3q", s.kper, s.kvpp, s.ropepp)
    b += struct.pack("<4id", s.loop_a, s.loop_b, s.loop_count, s.loop_nv, s.loop_eps)
    b += np.asarray(seq, np.int32).tobytes()
    if s.loop_count:
        b += np.asarray(pcached, np.int32).tobytes() + np.asarray(passes, np.int32).tobytes()
    b += ks.astype(np.float32).tobytes()
    for mi in range(s.n_mla):
        b += kvc[mi, :cached].astype(np.float32).tobytes()
    for mi in range(s.n_mla):
        b += ropec[mi, :cached].astype(np.float32).tobytes()
    return b


def save(k3, path, s, seq, cached, ks, kvc, ropec, kv_cap, pcached=None, passes=None):
    C = k3.C
    a = lambda x: None if x is None else np.ascontiguousarray(x).ctypes.data
    seqa = np.asarray(seq, np.int32)
    return k3.lib.k3_state_save(os.fsencode(path), C.byref(s), a(seqa), len(seq), cached, a(ks), a(kvc), a(ropec),
                                kv_cap, a(None if pcached is None else np.asarray(pcached, np.int32)),
                                a(None if passes is None else np.asarray(passes, np.int32)))


def load_state(k3, path, s, seq_cap, slots, kv_cap, loop_count=0):
    C = k3.C
    seq = np.zeros(seq_cap, np.int32)
    ks = np.zeros(slots * s.kper, np.float32)
    kvc = np.zeros((s.n_mla, kv_cap, s.kvpp), np.float32)
    ropec = np.zeros((s.n_mla, kv_cap, s.ropepp), np.float32)
    pc = np.zeros(max(loop_count + 1, 1), np.int32)
    ps = np.zeros(seq_cap, np.int32)
    cached, nseq = C.c_int(0), C.c_int(0)
    st = k3.lib.k3_state_load(os.fsencode(path), C.byref(s), seq.ctypes.data, seq_cap, ks.ctypes.data,
                              kvc.ctypes.data, ropec.ctypes.data, kv_cap, pc.ctypes.data, ps.ctypes.data,
                              C.byref(cached), C.byref(nseq))
    return st, seq[:nseq.value], ks, kvc, ropec, cached.value, pc, ps[:nseq.value]


def case(rng, s, kv_cap, cached, pending=1):
    slots = s.loop_nv if s.loop_count else s.n_bound
    seq = rng.integers(0, 1000, cached + pending).tolist()
    ks = rng.standard_normal(slots * s.kper).astype(np.float32)
    kvc = rng.standard_normal((s.n_mla, kv_cap, s.kvpp)).astype(np.float32)
    ropec = rng.standard_normal((s.n_mla, kv_cap, s.ropepp)).astype(np.float32)
    return seq, ks, kvc, ropec


def test_save_is_the_reference_format_and_round_trips(k3, tmp_path):
    rng = np.random.default_rng(1)
    s = layout(k3)
    kv_cap, cached = 50, 37
    seq, ks, kvc, ropec = case(rng, s, kv_cap, cached)
    p = str(tmp_path / "a.k3st")
    assert save(k3, p, s, seq, cached, ks, kvc, ropec, kv_cap) == 0
    assert open(p, "rb").read() == expected_bytes(s, seq, cached, ks, kvc, ropec)
    # peek, then load into a differently sized cache (the file is position-major per layer)
    C = k3.C
    got = k3.K3StateLayout()
    c, n = C.c_int(0), C.c_int(0)
    assert k3.lib.k3_state_peek(os.fsencode(p), C.byref(got), C.byref(c), C.byref(n)) == 0
    assert (c.value, n.value, got.kper, got.n_mla, list(got.fp)) == (cached, cached + 1, s.kper, 2, FP)
    st, seq2, ks2, kvc2, ropec2, cached2, _, _ = load_state(k3, p, s, 64, s.n_bound, 40)
    assert st == 0 and cached2 == cached and seq2.tolist() == seq
    np.testing.assert_array_equal(ks2, ks)
    np.testing.assert_array_equal(kvc2[:, :cached], kvc[:, :cached])
    np.testing.assert_array_equal(ropec2[:, :cached], ropec[:, :cached])


def test_layer_loop_record(k3, tmp_path):
    rng = np.random.default_rng(2)
    s = layout(k3, loop=(2, 1, 2, 6, 0.25))              # count 2, layers 1-2, 6 slots
    kv_cap, cached = 20, 12
    seq, ks, kvc, ropec = case(rng, s, kv_cap, cached, pending=0)
    pcached, passes = [12, 9, 4], rng.integers(1, 3, cached).tolist()
    p = str(tmp_path / "loop.k3st")
    assert save(k3, p, s, seq, cached, ks, kvc, ropec, kv_cap, pcached, passes) == 0
    assert open(p, "rb").read() == expected_bytes(s, seq, cached, ks, kvc, ropec, pcached, passes)
    st, seq2, ks2, _, _, _, pc, ps = load_state(k3, p, s, 32, 6, kv_cap, loop_count=2)
    assert st == 0 and pc.tolist() == pcached and ps.tolist() == passes
    np.testing.assert_array_equal(ks2, ks)
    # another loop refuses
    other = layout(k3, loop=(2, 1, 3, 6, 0.25))
    assert load_state(k3, p, other, 32, 6, kv_cap, loop_count=2)[0] == k3.K3GPU_EINVAL


def test_version_one_file_reads_as_no_loop(k3, tmp_path):
    rng = np.random.default_rng(3)
    s = layout(k3)
    kv_cap, cached = 10, 5
    seq, ks, kvc, ropec = case(rng, s, kv_cap, cached)
    b = bytearray(expected_bytes(s, seq, cached, ks, kvc, ropec))
    b[4:8] = struct.pack("<i", 1)
    del b[96:120]                                          # no loop record in version 1
    p = str(tmp_path / "v1.k3st")
    open(p, "wb").write(bytes(b))
    st, seq2, ks2, kvc2, _, cached2, _, _ = load_state(k3, p, s, 16, s.n_bound, kv_cap)
    assert st == 0 and seq2.tolist() == seq and cached2 == cached
    np.testing.assert_array_equal(kvc2[:, :cached], kvc[:, :cached])


def test_refusals(k3, tmp_path):
    rng = np.random.default_rng(4)
    s = layout(k3)
    kv_cap, cached = 30, 20
    seq, ks, kvc, ropec = case(rng, s, kv_cap, cached)
    p = str(tmp_path / "r.k3st")
    assert save(k3, p, s, seq, cached, ks, kvc, ropec, kv_cap) == 0
    raw = open(p, "rb").read()
    E, CAP = k3.K3GPU_EINVAL, k3.K3GPU_ECAPACITY

    def variant(name, data):
        q = str(tmp_path / name)
        open(q, "wb").write(data)
        return q

    fp2 = layout(k3)
    fp2.fp[0] = 7168                                        # another architecture
    assert load_state(k3, p, fp2, 64, s.n_bound, kv_cap)[0] == E
    lat = layout(k3, kvl=64)                                # another cache width
    assert load_state(k3, p, lat, 64, s.n_bound, kv_cap)[0] == E
    nb = layout(k3, n_mla=3)
    assert load_state(k3, p, nb, 64, s.n_bound, kv_cap)[0] == E
    assert load_state(k3, p, s, 64, s.n_bound, cached - 1)[0] == CAP     # too many positions
    assert load_state(k3, p, s, cached, s.n_bound, kv_cap)[0] == CAP     # too many ids
    assert load_state(k3, variant("magic", b"K4ST" + raw[4:]), s, 64, s.n_bound, kv_cap)[0] == E
    assert load_state(k3, variant("ver", raw[:4] + struct.pack("<i", 3) + raw[8:]), s, 64, s.n_bound, kv_cap)[0] == E
    bad_n = bytearray(raw)
    bad_n[68:72] = struct.pack("<i", cached + 2)           # more than one pending id
    assert load_state(k3, variant("nseq", bytes(bad_n)), s, 64, s.n_bound, kv_cap)[0] == E
    assert load_state(k3, variant("trunc", raw[:-5]), s, 64, s.n_bound, kv_cap)[0] == E
    # the writer refuses a sequence that is not the cached positions plus at most one id
    assert save(k3, str(tmp_path / "w.k3st"), s, seq + [1, 2], cached, ks, kvc, ropec, kv_cap) == E


def test_untrusted_loop_record_and_sizes(k3, tmp_path):
    """Sizes the loader reads with are bounded whatever the caller expects: a loop count
    outside 0..8 (the counter array holds 9) or a negative slot count is refused, also when
    the caller passes no counter array; the writer refuses a negative slot count."""
    rng = np.random.default_rng(6)
    s = layout(k3, loop=(2, 1, 3, 3, 1e-3))
    kv_cap, cached = 24, 10
    seq, ks, kvc, ropec = case(rng, s, kv_cap, cached)
    p = str(tmp_path / "l.k3st")
    assert save(k3, p, s, seq, cached, ks, kvc, ropec, kv_cap, [1, 2, 3], [0] * len(seq)) == 0
    raw = bytearray(open(p, "rb").read())
    C = k3.C
    for count, nv in ((20, 3), (-3, 3), (2, -5)):
        bad = bytearray(raw)
        bad[104:112] = struct.pack("<2i", count, nv)       # the loop record's count and nv
        q = str(tmp_path / f"bad{count}_{nv}.k3st")
        open(q, "wb").write(bytes(bad))
        e = layout(k3, loop=(count, 1, 3, nv, 1e-3))
        seq_b = np.zeros(64, np.int32)
        ks_b = np.zeros(4 * e.kper, np.float32)
        kvc_b = np.zeros((e.n_mla, kv_cap, e.kvpp), np.float32)
        ropec_b = np.zeros((e.n_mla, kv_cap, e.ropepp), np.float32)
        ci, ni = C.c_int(0), C.c_int(0)
        st = k3.lib.k3_state_load(os.fsencode(q), C.byref(e), seq_b.ctypes.data, 64, ks_b.ctypes.data,
                                  kvc_b.ctypes.data, ropec_b.ctypes.data, kv_cap, None, None, C.byref(ci),
                                  C.byref(ni))
        assert st == k3.K3GPU_EINVAL, (count, nv)
    neg = layout(k3, loop=(2, 1, 3, -1, 1e-3))
    assert save(k3, str(tmp_path / "n.k3st"), neg, seq, cached, ks, kvc, ropec, kv_cap, [1, 2, 3],
                [0] * len(seq)) == k3.K3GPU_EINVAL
