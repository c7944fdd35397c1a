"""A conversation's state to and from a K3ST file (session.save_state / load_state), CPU.

The KDA slots and the bf16 MLA caches (numpy arrays or torch tensors, as on the device)
round-trip exactly; the file is the format k3_state_save writes (the widened cache rows
read back through the raw loader); a file holding fp32 cache rows that bf16 cannot carry
(as the reference engine writes) loads rounded to nearest even with the changed values
counted; a layout that differs is refused.
"""
import importlib.util
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from k3lib import load  # noqa: E402

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def k3():
    return load()


def _session():
    spec = importlib.util.spec_from_file_location("session", os.path.join(os.path.dirname(HERE),
                                                                         "kimi-k3-for-me_b200", "session.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def layout(k3, H=2, D=8, K=4, n_bound=3, n_mla=2, kvl=16, qr=4):
    P = H * D
    s = k3.K3StateLayout()
    for i in range(12):
        s.fp[i] = 100 + i
    s.n_bound, s.n_mla, s.kper, s.kvpp, s.ropepp = n_bound, n_mla, P * D + 3 * P * (K - 1), kvl, qr
    s.loop_count, s.loop_a, s.loop_b, s.loop_nv, s.loop_eps = 0, -1, -1, n_bound, -1.0
    return s


def bf16_bits(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).view(torch.int16)


def test_round_trip_with_torch_tensors(k3, tmp_path):
    S = _session()
    rng = np.random.default_rng(71)
    lay, kv_cap, cached = layout(k3), 40, 25
    seq = rng.integers(0, 1000, cached + 1).tolist()
    slots = [torch.from_numpy(rng.standard_normal(lay.kper).astype(np.float32)) for _ in range(lay.n_bound)]
    lat = [bf16_bits(rng.standard_normal((kv_cap, lay.kvpp))) for _ in range(lay.n_mla)]
    rope = [bf16_bits(rng.standard_normal((kv_cap, lay.ropepp))) for _ in range(lay.n_mla)]
    p = str(tmp_path / "s.k3st")
    S.save_state(k3, p, lay, seq, cached, slots, lat, rope, kv_cap)
    got = S.load_state(k3, p, layout(k3), 64, kv_cap)
    assert got["seq"] == seq and got["cached"] == cached and got["inexact"] == 0
    for a, b in zip(got["kda_slots"], slots):
        np.testing.assert_array_equal(a, b.numpy())
    for i in range(lay.n_mla):          # rows the file holds: the cached ones
        np.testing.assert_array_equal(got["mla_lat"][i][:cached], lat[i].numpy().view(np.uint16)[:cached])
        np.testing.assert_array_equal(got["mla_rope"][i][:cached], rope[i].numpy().view(np.uint16)[:cached])
    other = layout(k3, kvl=32)
    with pytest.raises(k3.K3Error):
        S.load_state(k3, p, other, 64, kv_cap)                       # another cache width


def test_fp32_cache_rows_round_to_bf16_and_are_counted(k3, tmp_path):
    S = _session()
    rng = np.random.default_rng(72)
    lay, kv_cap, cached = layout(k3, n_mla=1), 12, 10
    seq = rng.integers(0, 50, cached).tolist()
    ks = rng.standard_normal(lay.n_bound * lay.kper).astype(np.float32)
    kvc = rng.standard_normal((1, kv_cap, lay.kvpp)).astype(np.float32)      # not bf16-representable
    ropec = bf16_bits(rng.standard_normal((1, kv_cap, lay.ropepp))).numpy().view(np.uint16)
    ropec = (ropec.astype(np.uint32) << 16).view(np.float32)                 # representable
    p = str(tmp_path / "f.k3st")
    st = k3.lib.k3_state_save(os.fsencode(p), k3.C.byref(lay), np.asarray(seq, np.int32).ctypes.data, len(seq),
                              cached, ks.ctypes.data, kvc.ctypes.data, np.ascontiguousarray(ropec).ctypes.data, kv_cap,
                              None, None)
    assert st == 0
    got = S.load_state(k3, p, layout(k3, n_mla=1), 64, kv_cap)
    want = bf16_bits(kvc[0]).numpy().view(np.uint16)
    np.testing.assert_array_equal(got["mla_lat"][0][:cached], want[:cached])
    assert got["inexact"] == cached * lay.kvpp                              # every lat value rounded
