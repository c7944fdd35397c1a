"""Pieces of bench.py's reporting that run without a GPU, CPU only: the clock record
that decides whether a timed run stands (median SM clock under load, the throttle
reasons seen Active -- hw_slowdown and the thermal ones reject a run, sw_power_cap is
kept and noted), and the unique-expert byte count behind the roofline's achieved figure.
"""
import importlib.util
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def line(sm, smax, hw="Not Active", hwt="Not Active", swt="Not Active", cap="Not Active"):
    return f"0, {sm}, {smax}, 812.40, 0x0000000000000000, {hw}, {hwt}, {swt}, {cap}"


def test_clock_summary():
    b = _bench()
    s = b.ClockSampler.summarize([line(1965, 1965), line(1950, 1965), line(1965, 1965)])
    assert s == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 3}
    s = b.ClockSampler.summarize([line(1300, 1965, cap="Active"), line(1320, 1965, cap="Active"),
                                  line(1410, 1965, hw="Active")])
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"] and s["sm_mhz"] == 1320.0
    s = b.ClockSampler.summarize([line(1800, 1965, hwt="Active", swt="Active")])
    assert s["reasons"] == ["hw_thermal_slowdown", "sw_thermal_slowdown"]
    # malformed samples are skipped whole: too few fields, a clock or max clock not a number
    s = b.ClockSampler.summarize(["garbage", line("[N/A]", 1965), line(1500, "[N/A]"), line(1700, 1965)])
    assert s["samples"] == 1 and s["sm_mhz"] == 1700.0
    assert b.ClockSampler.summarize([]) == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def test_unique_expert_bytes():
    b = _bench()
    idx = np.array([[3, 7], [7, 1], [3, 3]], np.int32)
    u, nbytes = b.unique_experts_bytes(idx, 1000)
    assert u == 3 and nbytes == 3000


def test_kda_prefill_cpu_baseline_runs_the_reference_step():
    """The prefill row's CPU baseline times the reference's own k3_kda_step (needs the
    reference library built under oracle/_ref; skipped where it is not)."""
    import pytest
    import sys
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    if O.ref() is None:
        pytest.skip("oracle/_ref not built")
    b = _bench()
    r = b.kda_prefill_cpu_baseline(T_sample=16, H=4, D=128)
    assert r["unit"] == "positions/s" and r["kind"] == "reference" and r["value"] > 0 and r["cores"] == 1


def test_matmul_cpu_baseline_runs_the_reference_projection():
    import pytest
    import sys
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    if O.ref() is None:
        pytest.skip("oracle/_ref not built")
    r = _bench().matmul_bf16_cpu_baseline(8, 256, 4096, rows=32)
    assert r["unit"] == "us per call" and r["kind"] == "reference" and r["value"] > 0


def test_c4_tree_and_forced_drafts():
    """The config-4 draft tree: 64 nodes, parents before children, at most 4 children and 4
    levels, its most probable branch 4 deep; the forced trees carry the continuation on that
    branch, and no sibling of a branch node repeats the branch's id there."""
    b = _bench()
    parent, chain = b.tree_topology()
    assert len(parent) == 64 and parent[0] == -1
    assert all(0 <= parent[i] < i for i in range(1, 64))
    assert max(np.bincount([p for p in parent if p >= 0])) <= 4
    assert len(chain) == 5 and all(parent[chain[j + 1]] == chain[j] for j in range(4))
    depth = [0] * 64
    for i in range(1, 64):
        depth[i] = depth[parent[i]] + 1
    assert max(depth) == 4
    cont = [list(range(100 * b_, 100 * b_ + 40)) for b_ in range(3)]
    tok = b.c4_trees(cont, parent, chain, steps=3, V=1000, seed=0)
    for s in range(3):
        for q in range(3):
            assert [tok[s, q, n] for n in chain] == cont[q][5 * s:5 * s + 5]
            for i in range(1, 64):
                if parent[i] in chain and i not in chain:
                    j = chain.index(parent[i]) + 1
                    if j < 5:
                        assert tok[s, q, i] != tok[s, q, chain[j]]


def test_fnv1a64_known_answers():
    """The output fingerprint is 64-bit FNV-1a over the bytes: the published test vectors of
    the hash (offset basis for the empty input, 'a', 'foobar') and an int32 array's bytes."""
    b = _bench()
    assert b.fnv1a64(np.zeros(0, np.uint8)) == "cbf29ce484222325"
    assert b.fnv1a64(np.frombuffer(b"a", np.uint8)) == "af63dc4c8601ec8c"
    assert b.fnv1a64(np.frombuffer(b"foobar", np.uint8)) == "85944171f73967e8"
    ids = np.array([1, 2, 3], np.int32)
    assert b.fnv1a64(ids) == b.fnv1a64(np.frombuffer(ids.tobytes(), np.uint8))
    assert b.fnv1a64(ids) != b.fnv1a64(ids[::-1])


def test_config5_stack_and_roofline_bound():
    """Config 5's stack: MLA every fourth layer (the 3:1 pattern, one-based), 48 routed
    experts per GPU; the roofline bound chosen by intensity against the measured ridge."""
    b = _bench()
    c = b.c5_cfg(93, 8)
    assert c["num_hidden_layers"] == 93 and c["num_experts"] == 384
    assert c["full_attn_layers"] == list(range(4, 93, 4)) and len(c["full_attn_layers"]) == 23
    assert b.c5_cfg(8, 1)["full_attn_layers"] == [4, 8] and b.c5_cfg(8, 1)["num_experts"] == 48
    cfg = b.c5_config(93, 2)
    assert cfg["layers"] == 93 and cfg["sequences_per_gpu"] == 32 and cfg["tokens_verified_per_step"] == 576
    # config 5 at one GPU: 5184 pairs over 49 experts (past the ridge); at two: a weight stream
    w13 = 2 * 2048 * (7168 // 2 + 7168 // 32)
    t1, i1, r1 = b.roofline_bound(2.0 * 5184 * 2 * 2048 * 7168, 49 * w13, 1654.4, 6543.4)
    t2, i2, _ = b.roofline_bound(2.0 * 2592 * 2 * 2048 * 7168, 48 * w13, 1654.4, 6543.4)
    assert t1 and not t2 and i2 < r1 < i1 and abs(r1 - 252.8) < 0.1


def test_reference_build_choice_follows_the_host_cpu(monkeypatch, tmp_path):
    """The timed reference baselines load the x86-64-v4 build only where it was built and the
    host reports the AVX-512 subsets; K3_REF_ISA=v3 forces the v3 build; every baseline line
    names the ISA it timed."""
    import sys
    sys.path.insert(0, ROOT)
    from oracle import oracle as O
    flags_v4 = "flags\t\t: fpu sse2 avx2 fma avx512f avx512bw avx512cd avx512dq avx512vl\n"
    flags_v3 = "flags\t\t: fpu sse2 avx2 fma\n"
    real_open = open

    def fake_cpuinfo(text):
        def opener(path, *a, **k):
            if path == "/proc/cpuinfo":
                p = tmp_path / "cpuinfo"
                p.write_text(text)
                return real_open(p, *a, **k)
            return real_open(path, *a, **k)
        return opener

    import builtins
    monkeypatch.setattr(builtins, "open", fake_cpuinfo(flags_v3))
    assert not O.host_has_x86_64_v4()
    assert O.ref_bench_isa() == "v3"
    monkeypatch.setattr(builtins, "open", fake_cpuinfo(flags_v4))
    assert O.host_has_x86_64_v4()
    built = os.path.exists(os.path.join(ROOT, "oracle", "_ref", "v4", "libk3ref_bench.so"))
    assert O.ref_bench_isa() == ("v4" if built else "v3")
    monkeypatch.setenv("K3_REF_ISA", "v3")
    assert O.ref_bench_isa() == "v3"
    assert O.ref_bench_path().endswith(os.path.join("_ref", "libk3ref_bench.so"))
    assert set(O.ISA_TEXT) == {"v3", "v4"}
