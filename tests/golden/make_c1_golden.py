"""Golden token streams of BASELINE config 1 from the reference engine itself (run here,
where its sources compile): tests/golden/c1_golden.npz.

The checkpoint is the package's synthetic config-1 model (``synth.write_checkpoint``,
seed 0, the reference generator's initialisation recipe), written to a temporary
directory; it is regenerated bit for bit from the same call on the GPU box, so only the
reference's OUTPUTS are stored. The engine is ``oracle/_ref/k3``: the reference's own CLI
compiled from its sources by ``oracle/Makefile`` (``make -C oracle``), run serially with
the latent MLA cache and the absorbed attention (``--kv-latent --mla-absorb``), the
layout this library keeps.

Runs stored (ids, the logits behind every generated id, the spec trace):
  base      the 32-id uniform-random prompt (python random.Random(0), ids < 1024), greedy
            64 ids, ``--incremental --spec 4``; on this random model the n-gram drafter
            never fires (0 sweeps), so it is also the serial stream; the state saved after
            the run (``--save-state``, K3ST) is stored as the reference's final KDA state
            and latent cache.
  craft<k>  for k = 0..4: a prompt built so that the FIRST verify sweep drafts 4 ids and
            the model accepts exactly k of them (k = 4: all). The prompt ends with a 3-gram
            `a` that also opens it, followed there by the model's own next id and then its
            continuation up to the rejection point and a wrong id, so the drafter (n = 4,
            the suffix a + next id) proposes exactly that; the continuation depends on the
            prompt, so the prompt is iterated with serial runs until it reproduces itself.
            Greedy 10 ids with ``--spec 4`` (and checked equal to the serial run).

Usage: python tests/golden/make_c1_golden.py   (needs oracle/_ref/k3: `make -C oracle`)
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import os
import random
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
K3 = os.path.join(ROOT, "oracle", "_ref", "k3")
SPEC = 4
VOCAB = 1024


def load(name, rel):
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, rel))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def base_prompt():
    r = random.Random(0)
    return [r.randrange(VOCAB) for _ in range(32)]


def run_ref(ckpt, ids, gen, spec, work, tag, state=False):
    """One reference run; returns (report, logits [n_generated][vocab])."""
    out = os.path.join(work, tag + ".json")
    lg = os.path.join(work, tag + ".bin")
    cmd = [K3, ckpt, "--ids", ",".join(map(str, ids)), "--gen", str(gen), "--incremental", "--kv-latent",
           "--mla-absorb", "--cache-gb", "1", "--dump-all-logits", lg, "--out", out]
    if spec:
        cmd += ["--spec", str(spec)]
    if state:
        cmd += ["--save-state", os.path.join(work, tag + ".k3st")]
    subprocess.run(cmd, check=True, stdout=subprocess.DEVNULL, cwd=work)
    rep = json.load(open(out))
    logits = np.fromfile(lg, np.float32).reshape(-1, VOCAB)
    assert logits.shape[0] == len(rep["generated_ids"])
    return rep, logits


def crafted(ckpt, accept, work):
    """A prompt whose first sweep drafts SPEC ids of which the model accepts `accept`."""
    rnd = random.Random(1000 + accept)
    for _attempt in range(20):
        a = [rnd.randrange(VOCAB) for _ in range(3)]
        r = [rnd.randrange(VOCAB) for _ in range(8)]
        y = [rnd.randrange(VOCAB) for _ in range(SPEC + 2)]
        for _it in range(8):
            junk = (y[accept + 1] + 1 + rnd.randrange(VOCAB - 1)) % VOCAB
            b = y[:SPEC + 1] if accept == SPEC else (y[:accept + 1] + [junk] + y[accept + 2:])[:SPEC + 1]
            prompt = a + b + r + a
            rep, _ = run_ref(ckpt, prompt, SPEC + 2, 0, work, "serial")
            got = rep["generated_ids"]
            need = accept + 2 if accept < SPEC else SPEC + 1
            if got[:need] == y[:need] and (accept == SPEC or got[accept + 1] != junk):
                return prompt
            y = got
    raise SystemExit(f"no stable crafted prompt for accept={accept}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "c1_golden.npz"))
    a = ap.parse_args()
    if not os.path.exists(K3):
        raise SystemExit(f"{K3} is missing: build it with `make -C oracle`")
    synth = load("k3synth", "kimi-k3-for-me_b200/synth.py")
    k3 = load("k3b200", "kimi-k3-for-me_b200/__init__.py")
    out = {}
    with tempfile.TemporaryDirectory() as work:
        ckpt = synth.write_checkpoint(os.path.join(work, "c1"), seed=0, recipe="reference")
        p = base_prompt()
        rep, logits = run_ref(ckpt, p, 64, SPEC, work, "base", state=True)
        rs, ls = run_ref(ckpt, p, 64, 0, work, "base_serial")
        assert rep["generated_ids"] == rs["generated_ids"] and np.array_equal(logits, ls)
        out["base/prompt"] = np.asarray(p, np.int32)
        out["base/ids"] = np.asarray(rep["generated_ids"], np.int32)
        out["base/logits"] = logits
        out["base/sweeps"] = np.asarray(rep["spec_sweeps"], np.int32)
        # the carried state after the run: KDA slots and the fp32 latent cache rows
        lay = k3.K3StateLayout()
        cached, nseq = C.c_int(0), C.c_int(0)
        path = os.fsencode(os.path.join(work, "base.k3st"))
        k3.check(k3.lib.k3_state_peek(path, C.byref(lay), C.byref(cached), C.byref(nseq)), "peek")
        kv_cap = cached.value
        ks = np.zeros(lay.n_bound * lay.kper, np.float32)
        kvc = np.zeros((lay.n_mla, kv_cap, lay.kvpp), np.float32)
        ropec = np.zeros((lay.n_mla, kv_cap, lay.ropepp), np.float32)
        seq = np.zeros(nseq.value, np.int32)
        c2, n2 = C.c_int(0), C.c_int(0)
        k3.check(k3.lib.k3_state_load(path, C.byref(lay), seq.ctypes.data, len(seq), ks.ctypes.data,
                                      kvc.ctypes.data, ropec.ctypes.data, kv_cap, None, None, C.byref(c2),
                                      C.byref(n2)), "load")
        out["base/state_cached"] = np.asarray(c2.value, np.int32)
        out["base/state_seq"] = seq
        out["base/state_kda"] = ks.reshape(lay.n_bound, lay.kper)
        out["base/state_lat"] = kvc
        out["base/state_rope"] = ropec
        for k in range(SPEC + 1):
            prompt = crafted(ckpt, k, work)
            rep, logits = run_ref(ckpt, prompt, 10, SPEC, work, f"craft{k}")
            rs, ls = run_ref(ckpt, prompt, 10, 0, work, f"craft{k}_serial")
            assert rep["generated_ids"] == rs["generated_ids"], "spec and serial differ"
            assert rep["spec_trace"] and rep["spec_trace"][0] == [SPEC, k, k + 1], rep["spec_trace"]
            out[f"craft{k}/prompt"] = np.asarray(prompt, np.int32)
            out[f"craft{k}/ids"] = np.asarray(rep["generated_ids"], np.int32)
            out[f"craft{k}/trace"] = np.asarray(rep["spec_trace"], np.int32).reshape(-1, 3)
            out[f"craft{k}/logits"] = logits
            print(f"craft{k}: prompt {len(prompt)} ids, trace {rep['spec_trace']}")
    np.savez_compressed(a.out, **out)
    print("wrote", a.out, os.path.getsize(a.out), "bytes")


if __name__ == "__main__":
    main()
