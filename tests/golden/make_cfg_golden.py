"""Generate tests/golden/cfg_golden.json: the reference's own config loader's answer
(k3_cfg_load_file, include/k3/k3_cfg.h of the reference, run by oracle/_ref/cfgdump) on a
set of config documents -- the parsed fields, or REFUSED.

The documents: a small model in the fixtures' flat shape and in the released nested shape
(text_config + linear_attn_config, released key spellings), a K3-scale nested config, the
optional switches absent / numeric / malformed, every refusal the loader has (missing
keys, no layer map, a layer index outside 1..n, top-k above the build's limit or the
expert count, a zero AttnRes block, a zero conv width, every layer full attention, a
non-numeric layer entry, a required key given as a boolean, non-positive sizes), a
non-integral integer, a key present in both text_config and linear_attn_config; and the
reference's own config fixtures (tests/fixtures/cfg/*.json) and the configs inside its
model fixtures (tiny_k3.json, ref_k3.json).

Usage: python tests/golden/make_cfg_golden.py [--ref <path of the reference checkout>]
(needs oracle/_ref/cfgdump: `make -C oracle`)
"""
from __future__ import annotations

import argparse
import copy
import json
import os
import subprocess
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_dir():
    """K3_REFERENCE, else a checkout named `reference` beside this repository."""
    return os.environ.get("K3_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
DUMP = os.path.join(HERE, "..", "..", "oracle", "_ref", "cfgdump")

FLAT = {"hidden_size": 96, "num_hidden_layers": 7, "vocab_size": 300, "rms_norm_eps": 1e-5,
        "kda_num_heads": 3, "kda_head_dim": 16, "short_conv_kernel_size": 4, "gate_lower_bound": -5.0,
        "num_attention_heads": 4, "q_lora_rank": 32, "kv_lora_rank": 16, "qk_nope_head_dim": 8,
        "qk_rope_head_dim": 4, "v_head_dim": 8, "mla_use_output_gate": False, "num_experts": 6,
        "num_experts_per_token": 2, "num_shared_experts": 1, "routed_expert_hidden_size": 32,
        "moe_intermediate_size": 24, "routed_scaling_factor": 2.5, "moe_renormalize": True,
        "latent_moe_use_norm": True, "first_k_dense_replace": 1, "intermediate_size": 40,
        "attn_res_block_size": 3, "situ_beta": 4.0, "situ_linear_beta": 25.0, "full_attn_layers": [3, 7]}
LIN_KEYS = ("kda_num_heads", "kda_head_dim", "short_conv_kernel_size", "gate_lower_bound", "full_attn_layers")


def nested(flat):
    txt = {k: v for k, v in flat.items() if k not in LIN_KEYS + ("situ_beta", "situ_linear_beta")}
    if "situ_beta" in flat:
        txt["activation_situ_beta"] = flat["situ_beta"]
    if "situ_linear_beta" in flat:
        txt["activation_situ_linear_beta"] = flat["situ_linear_beta"]
    lin = {}
    for k in LIN_KEYS:
        if k in flat:
            lin[{"kda_num_heads": "num_heads", "kda_head_dim": "head_dim"}.get(k, k)] = flat[k]
    txt["linear_attn_config"] = lin
    return {"model_type": "kimi_k3", "text_config": txt}


def variants():
    v = {"flat": FLAT, "nested": nested(FLAT)}
    big = dict(FLAT, hidden_size=7168, num_hidden_layers=93, vocab_size=163840, kda_num_heads=96,
               kda_head_dim=128, num_attention_heads=64, q_lora_rank=1536, kv_lora_rank=512,
               qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128, num_experts=896,
               num_experts_per_token=16, num_shared_experts=2, routed_expert_hidden_size=3072,
               moe_intermediate_size=3072, attn_res_block_size=4, full_attn_layers=list(range(4, 94, 4)))
    v["k3_scale_nested"] = nested(big)

    def edit(name, base, **kw):
        d = copy.deepcopy(base)
        for k, val in kw.items():
            if val is None:
                d.pop(k, None)
            else:
                d[k] = val
        v[name] = d
    edit("switches_absent", FLAT, mla_use_output_gate=None, moe_renormalize=None, latent_moe_use_norm=None)
    edit("switches_numeric", FLAT, mla_use_output_gate=0, moe_renormalize=1, latent_moe_use_norm=0)
    edit("switch_string", FLAT, mla_use_output_gate="no")
    edit("missing_situ", FLAT, situ_beta=None, situ_linear_beta=None)
    edit("missing_many", FLAT, hidden_size=None, q_lora_rank=None, num_experts=None)
    edit("no_layermap", FLAT, full_attn_layers=None)
    edit("empty_layermap", FLAT, full_attn_layers=[])
    edit("layer_zero", FLAT, full_attn_layers=[0, 7])
    edit("layer_past_end", FLAT, full_attn_layers=[3, 8])
    edit("topk_65", dict(FLAT, num_experts=128), num_experts_per_token=65)
    edit("topk_over_experts", FLAT, num_experts_per_token=7)
    edit("attn_res_block_zero", FLAT, attn_res_block_size=0)
    edit("conv_zero", FLAT, short_conv_kernel_size=0)
    edit("all_mla", FLAT, full_attn_layers=list(range(1, 8)))
    edit("layer_string", FLAT, full_attn_layers=[3, "7"])
    edit("bool_for_int", FLAT, num_experts=True)
    edit("nonpositive_vocab", FLAT, vocab_size=0)
    edit("nonintegral", FLAT, hidden_size=96.7, routed_scaling_factor=2.25)
    both = nested(FLAT)
    both["text_config"]["head_dim"] = 99             # present at text_config and linear_attn_config
    v["key_in_both"] = both
    return v


def run(doc):
    with tempfile.NamedTemporaryFile("w", suffix=".json", delete=False) as f:
        json.dump(doc, f)
        path = f.name
    try:
        out = subprocess.run([DUMP, path], capture_output=True, text=True, check=True).stdout
    finally:
        os.unlink(path)
    for line in out.splitlines():
        if line.startswith("CFG "):
            return json.loads(line[4:])
        if line.strip() == "REFUSED":
            return "REFUSED"
    raise RuntimeError("no verdict from cfgdump")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=reference_dir(),
                    help="the reference checkout (default: K3_REFERENCE, else `reference` beside this repository)")
    a = ap.parse_args()
    docs = variants()
    fx = os.path.join(a.ref, "tests", "fixtures")
    for n in sorted(os.listdir(os.path.join(fx, "cfg"))):
        with open(os.path.join(fx, "cfg", n)) as f:
            docs["ref_fixture_" + n[:-5]] = json.load(f)
    for n in ("tiny_k3.json", "ref_k3.json"):
        with open(os.path.join(fx, n)) as f:
            docs["ref_model_" + n[:-5]] = json.load(f)["config"]
    cases = {name: {"doc": doc, "ref": run(doc)} for name, doc in docs.items()}
    path = os.path.join(HERE, "cfg_golden.json")
    with open(path, "w") as f:
        json.dump(cases, f, indent=1, sort_keys=True)
    print(path, len(cases), "cases,", sum(c["ref"] == "REFUSED" for c in cases.values()), "refused")


if __name__ == "__main__":
    main()
