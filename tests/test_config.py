"""The model configuration reader (config.read_config) and the structures built from it,
CPU only.

The same model described in the released nested shape (text_config with
linear_attn_config; num_heads / head_dim; activation_situ_*) and in the reference
fixtures' flat shape (kda_num_heads / kda_head_dim; situ_*) must read to the same flat
configuration (include/k3/k3_cfg.h:60-200); a config lacking required keys must be
refused with every missing key named, never defaulted; the three optional switches
default on. The layer and MoE configuration structures must carry every field.
"""
import copy
import json
import os
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from k3lib import load  # noqa: E402

FLAT = {"hidden_size": 96, "num_hidden_layers": 7, "vocab_size": 300, "rms_norm_eps": 1e-5,
        "kda_num_heads": 3, "kda_head_dim": 16, "short_conv_kernel_size": 4, "gate_lower_bound": -5.0,
        "num_attention_heads": 4, "q_lora_rank": 32, "kv_lora_rank": 16, "qk_nope_head_dim": 8,
        "qk_rope_head_dim": 4, "v_head_dim": 8, "mla_use_output_gate": False, "num_experts": 6,
        "num_experts_per_token": 2, "num_shared_experts": 1, "routed_expert_hidden_size": 32,
        "moe_intermediate_size": 24, "routed_scaling_factor": 2.5, "moe_renormalize": True,
        "latent_moe_use_norm": True, "first_k_dense_replace": 1, "intermediate_size": 40,
        "attn_res_block_size": 3, "situ_beta": 4.0, "situ_linear_beta": 25.0, "full_attn_layers": [3, 7]}


@pytest.fixture(scope="module")
def k3():
    return load()


def _cfg_mod():
    import importlib.util
    spec = importlib.util.spec_from_file_location("k3config", os.path.join(os.path.dirname(HERE),
                                                                           "kimi-k3-for-me_b200", "config.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def nested(flat):
    """The released shape of the same model."""
    txt = {k: v for k, v in flat.items()
           if k not in ("kda_num_heads", "kda_head_dim", "short_conv_kernel_size", "gate_lower_bound",
                        "full_attn_layers", "situ_beta", "situ_linear_beta")}
    txt["activation_situ_beta"] = flat["situ_beta"]
    txt["activation_situ_linear_beta"] = flat["situ_linear_beta"]
    txt["linear_attn_config"] = {"num_heads": flat["kda_num_heads"], "head_dim": flat["kda_head_dim"],
                                 "short_conv_kernel_size": flat["short_conv_kernel_size"],
                                 "gate_lower_bound": flat["gate_lower_bound"],
                                 "full_attn_layers": flat["full_attn_layers"]}
    return {"model_type": "kimi_k3", "text_config": txt, "vision_config": {"hidden_size": 1152}}


def test_both_shapes_read_the_same(tmp_path):
    m = _cfg_mod()
    a = m.read_config(dict(FLAT))
    b = m.read_config(nested(FLAT))
    assert a == b
    assert a["kda_num_heads"] == 3 and a["mla_use_output_gate"] is False and a["full_attn_layers"] == [3, 7]
    p = tmp_path / "config.json"
    import json
    p.write_text(json.dumps(nested(FLAT)))
    assert m.read_config(str(p)) == a
    assert m.attn_res_stride(a) == 7 // 3 + 2


def test_missing_keys_are_all_named_and_switches_default_on():
    m = _cfg_mod()
    bad = dict(FLAT)
    for k in ("situ_beta", "situ_linear_beta", "full_attn_layers", "mla_use_output_gate"):
        del bad[k]
    with pytest.raises(m.ConfigError) as e:
        m.read_config(bad)
    for k in ("activation_situ_beta", "activation_situ_linear_beta", "full_attn_layers"):
        assert k in str(e.value)
    ok = dict(FLAT)
    del ok["mla_use_output_gate"], ok["moe_renormalize"]
    c = m.read_config(ok)
    assert c["mla_use_output_gate"] is True and c["moe_renormalize"] is True
    tricky = copy.deepcopy(nested(FLAT))
    tricky["text_config"]["linear_attn_config"]["full_attn_layers"] = [3, "7"]
    with pytest.raises(m.ConfigError):
        m.read_config(tricky)


def test_structures_carry_every_field(k3):
    m = _cfg_mod()
    c = m.read_config(dict(FLAT))
    lc, mc = m.layer_cfg(k3, c), m.moe_cfg(k3, c)
    want_l = {"hidden": 96, "kda_heads": 3, "kda_head_dim": 16, "conv_k": 4, "gate_lb": -5.0, "attn_res_block": 3,
              "max_blocks": 4, "n_routed": 6, "n_shared": 1, "topk": 2, "moe_inter": 24, "act": k3.ACT_SITU,
              "renorm": 1, "routed_scale": 2.5, "situ_b1": 4.0, "situ_b2": 25.0, "latent": 32, "shared_inter": 24,
              "mla_heads": 4, "q_lora": 32, "kv_lora": 16, "qk_nope": 8, "qk_rope": 4, "v_head": 8}
    for n, v in want_l.items():
        assert getattr(lc, n) == pytest.approx(v), n
    assert lc.rms_eps == pytest.approx(1e-5)
    assert {n for n, _ in k3.K3GpuLayerCfg._fields_} == set(want_l) | {"rms_eps"}
    want_m = {"hidden": 96, "latent": 32, "moe_inter": 24, "shared_inter": 24, "n_routed": 6, "topk": 2,
              "act": k3.ACT_SITU, "renorm": 1, "routed_scale": 2.5, "situ_b1": 4.0, "situ_b2": 25.0}
    for n, v in want_m.items():
        assert getattr(mc, n) == pytest.approx(v), n
    with pytest.raises(m.ConfigError):
        m._fill(k3.K3GpuMoeCfg, {"hiden": 1})


# the reference loader's field names -> this reader's (canonical) names
REF_FIELDS = {"hidden": "hidden_size", "n_layers": "num_hidden_layers", "vocab": "vocab_size",
              "rms_eps": "rms_norm_eps", "kda_heads": "kda_num_heads", "kda_head_dim": "kda_head_dim",
              "conv_k": "short_conv_kernel_size", "gate_lb": "gate_lower_bound", "n_heads": "num_attention_heads",
              "q_lora": "q_lora_rank", "kv_lora": "kv_lora_rank", "qk_nope": "qk_nope_head_dim",
              "qk_rope": "qk_rope_head_dim", "v_head": "v_head_dim", "mla_out_gate": "mla_use_output_gate",
              "n_experts": "num_experts", "topk": "num_experts_per_token", "n_shared": "num_shared_experts",
              "latent": "routed_expert_hidden_size", "moe_inter": "moe_intermediate_size",
              "routed_scale": "routed_scaling_factor", "moe_renorm": "moe_renormalize",
              "latent_norm": "latent_moe_use_norm", "first_dense": "first_k_dense_replace",
              "dense_inter": "intermediate_size", "attn_res_block": "attn_res_block_size",
              "situ_b1": "situ_beta", "situ_b2": "situ_linear_beta", "full_attn": "full_attn_layers"}
GOLD = json.load(open(os.path.join(HERE, "golden", "cfg_golden.json")))


@pytest.mark.parametrize("name", sorted(GOLD))
def test_reader_matches_reference_loader(name):
    """Against the reference's own k3_cfg_load on the same document
    (tests/golden/cfg_golden.json, tests/golden/make_cfg_golden.py): the same refusals, and
    every parsed field equal (floats as the float32 the loader stores)."""
    import numpy as np
    m = _cfg_mod()
    case = GOLD[name]
    if case["ref"] == "REFUSED":
        with pytest.raises(m.ConfigError):
            m.read_config(copy.deepcopy(case["doc"]))
        return
    c = m.read_config(copy.deepcopy(case["doc"]))
    for rf, mine in REF_FIELDS.items():
        want, got = case["ref"][rf], c[mine]
        if isinstance(want, float) or isinstance(got, float):
            assert np.float32(got) == np.float32(want), rf
        else:
            assert (int(got) if isinstance(got, bool) else got) == want, rf
    assert m.attn_res_stride(c) == case["ref"]["stride"]
