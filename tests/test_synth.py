"""The synthetic checkpoint writer (host, no GPU): its quantiser is the reference writer's
rule (as the oracle restates it), the directory it writes is read by the config reader and
bound whole by the binder and the expert loader, and it is reproducible from its seed."""
import hashlib
import importlib.util
import os

import numpy as np

from oracle import oracle as O
from tests import k3lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _mod(name, rel):
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, rel))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_quantiser_is_the_reference_rule():
    S = _mod("k3synth_q", "kimi-k3-for-me_b200/synth.py")
    rng = np.random.default_rng(5)
    for std in (0.02, 1.2, 30.0):
        w = rng.standard_normal((48, 256), dtype=np.float32) * np.float32(std)
        w[3, :32] = 0.0                                   # an all-zero group
        a, b = S.mxfp4_quant(w), O.mxfp4_quant(w)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_config1_checkpoint_binds_and_reproduces(tmp_path):
    S = _mod("k3synth_b", "kimi-k3-for-me_b200/synth.py")
    cm = _mod("k3cfg_b", "kimi-k3-for-me_b200/config.py")
    bm = _mod("k3bind_b", "kimi-k3-for-me_b200/bind.py")
    k3 = k3lib.load()
    d = S.write_checkpoint(str(tmp_path / "a"), seed=0)
    cfg = cm.read_config(os.path.join(d, "config.json"))
    assert cfg["num_hidden_layers"] == 4 and cfg["full_attn_layers"] == [4]
    idx = k3.SafetensorsIndex(d)
    b = bm.Binder(idx, cfg)
    kinds = [b.layer(L)["kind"] for L in range(4)]
    assert kinds == ["kda", "kda", "kda", "mla"]
    top = b.model()
    assert top["embed"].shape == (1024 * 512,) and top["lm_head"].dtype == np.uint16
    assert not b.converted                                  # every projection stored as bf16
    files = [os.path.join(d, "model.safetensors")]
    bank = k3.bank_read_safetensors(files, 2, 0, 16, 512, 256)
    assert bank.any()
    idx.close()
    # the same (config, seed, recipe) gives the same bytes
    d2 = S.write_checkpoint(str(tmp_path / "b"), seed=0)
    h = [hashlib.sha256(open(os.path.join(x, "model.safetensors"), "rb").read()).hexdigest() for x in (d, d2)]
    assert h[0] == h[1]
