"""The model configuration from a config JSON (host, no GPU): the reference's k3_cfg_load
(include/k3/k3_cfg.h:60-200) restated, and the layer and MoE configuration structures
this library's entry points take, built from it.

Two shapes are read the same way: the released config.json, nested (the language model
under "text_config", the KDA settings and the layer map under
text_config.linear_attn_config, the SiTU betas named activation_situ_beta /
activation_situ_linear_beta), and the reference fixtures' flat shape (situ_beta /
situ_linear_beta, kda_num_heads / kda_head_dim). Each key is looked for in text_config,
then linear_attn_config, then the top level, under its released name and then its alias.
A missing required key is an error, never a default -- every missing key is reported
together -- because a reader that defaults builds a different model that still runs;
only the three switches the reference treats as optional (mla_use_output_gate,
moe_renormalize, latent_moe_use_norm, all default on) have defaults.
"""
from __future__ import annotations

import json

# canonical name (the flat shape) -> (released name, alias, kind)
_KEYS = {
    "hidden_size": ("hidden_size", None, int),
    "num_hidden_layers": ("num_hidden_layers", None, int),
    "vocab_size": ("vocab_size", None, int),
    "rms_norm_eps": ("rms_norm_eps", None, float),
    "kda_num_heads": ("num_heads", "kda_num_heads", int),
    "kda_head_dim": ("head_dim", "kda_head_dim", int),
    "short_conv_kernel_size": ("short_conv_kernel_size", None, int),
    "gate_lower_bound": ("gate_lower_bound", None, float),
    "num_attention_heads": ("num_attention_heads", None, int),
    "q_lora_rank": ("q_lora_rank", None, int),
    "kv_lora_rank": ("kv_lora_rank", None, int),
    "qk_nope_head_dim": ("qk_nope_head_dim", None, int),
    "qk_rope_head_dim": ("qk_rope_head_dim", None, int),
    "v_head_dim": ("v_head_dim", None, int),
    "num_experts": ("num_experts", None, int),
    "num_experts_per_token": ("num_experts_per_token", None, int),
    "num_shared_experts": ("num_shared_experts", None, int),
    "routed_expert_hidden_size": ("routed_expert_hidden_size", None, int),
    "moe_intermediate_size": ("moe_intermediate_size", None, int),
    "routed_scaling_factor": ("routed_scaling_factor", None, float),
    "first_k_dense_replace": ("first_k_dense_replace", None, int),
    "intermediate_size": ("intermediate_size", None, int),
    "attn_res_block_size": ("attn_res_block_size", None, int),
    "situ_beta": ("activation_situ_beta", "situ_beta", float),
    "situ_linear_beta": ("activation_situ_linear_beta", "situ_linear_beta", float),
}
_SWITCHES = ("mla_use_output_gate", "moe_renormalize", "latent_moe_use_norm")
MAX_TOPK = 64   # the reference's K3_MAX_TOPK (include/k3/k3.h:864), also the router's limit here


class ConfigError(ValueError):
    """The config lacks required keys (all of them listed) or holds a malformed one."""


def _num(v):
    return isinstance(v, (int, float)) and not isinstance(v, bool)


def read_config(src) -> dict:
    """The flat configuration (canonical names above, plus the three switches as bools and
    full_attn_layers, one-based as stored) from a path or an already parsed dict."""
    if not isinstance(src, dict):
        with open(src) as f:
            src = json.load(f)
    txt = src.get("text_config") if isinstance(src.get("text_config"), dict) else None
    base = txt if txt is not None else src
    lin = base.get("linear_attn_config") if isinstance(base.get("linear_attn_config"), dict) else None
    objs = [o for o in (txt, lin, src) if o is not None]

    def find(primary, alias):
        for o in objs:
            for n in (primary, alias):
                if n is not None and n in o:
                    return o[n]
        return None

    out, missing = {}, []
    for canon, (primary, alias, kind) in _KEYS.items():
        v = find(primary, alias)
        if not _num(v):
            missing.append(primary)
            continue
        out[canon] = kind(v)
    for n in _SWITCHES:
        v = find(n, None)
        out[n] = True if v is None else (bool(v) if isinstance(v, (bool, int, float)) else True)
    fal = find("full_attn_layers", None)
    if not isinstance(fal, list) or not fal:
        missing.append("full_attn_layers")
    elif not all(_num(x) for x in fal):
        raise ConfigError("full_attn_layers holds a value that is not a number")
    else:
        out["full_attn_layers"] = [int(x) for x in fal]
    if missing:
        raise ConfigError("the config is missing required field(s): " + ", ".join(missing) +
                          " (no defaults are substituted: a config read in part is a different model)")
    # structural checks (k3_cfg.h:202-240): a config that parses but cannot be this model
    nl = out["num_hidden_layers"]
    if nl <= 0 or out["hidden_size"] <= 0 or out["vocab_size"] <= 0:
        raise ConfigError("non-positive layers, hidden size or vocabulary")
    if len(out["full_attn_layers"]) >= nl:
        raise ConfigError(f"{len(out['full_attn_layers'])} of {nl} layers marked full attention: no KDA layer")
    for i, x in enumerate(out["full_attn_layers"]):
        if x < 1 or x > nl:
            raise ConfigError(f"full_attn_layers[{i}] = {x} is outside 1..{nl} (the list is one-based)")
    if out["num_experts_per_token"] > MAX_TOPK:
        raise ConfigError(f"top-{out['num_experts_per_token']} routing: at most {MAX_TOPK} is supported")
    if out["num_experts_per_token"] > out["num_experts"]:
        raise ConfigError(f"top-{out['num_experts_per_token']} of {out['num_experts']} experts")
    if out["attn_res_block_size"] <= 0:
        raise ConfigError(f"attn_res_block_size {out['attn_res_block_size']}")
    if out["short_conv_kernel_size"] < 1:
        raise ConfigError(f"short_conv_kernel_size {out['short_conv_kernel_size']}")
    return out


def attn_res_stride(c) -> int:
    """The block-residual stride: layers / block + 2 (include/k3/k3.h:134-137)."""
    return c["num_hidden_layers"] // c["attn_res_block_size"] + 2


def _fill(struct_type, values):
    """struct_type with every field set from values, refusing names it does not declare
    (a misspelt attribute on a ctypes structure would otherwise be set silently beside it)
    and fields left unset."""
    declared = [n for n, _ in struct_type._fields_]
    unknown, unset = set(values) - set(declared), set(declared) - set(values)
    if unknown or unset:
        raise ConfigError(f"{struct_type.__name__}: unknown {sorted(unknown)}, unset {sorted(unset)}")
    s = struct_type()
    for n in declared:
        setattr(s, n, values[n])
    return s


def layer_cfg(k3, c):
    """K3GpuLayerCfg for the decoder-layer entry points (the K3 MoE form)."""
    return _fill(k3.K3GpuLayerCfg, {
        "hidden": c["hidden_size"], "kda_heads": c["kda_num_heads"], "kda_head_dim": c["kda_head_dim"],
        "conv_k": c["short_conv_kernel_size"], "gate_lb": c["gate_lower_bound"], "rms_eps": c["rms_norm_eps"],
        "attn_res_block": c["attn_res_block_size"], "max_blocks": attn_res_stride(c),
        "n_routed": c["num_experts"], "n_shared": c["num_shared_experts"], "topk": c["num_experts_per_token"],
        "moe_inter": c["moe_intermediate_size"], "act": k3.ACT_SITU, "renorm": int(c["moe_renormalize"]),
        "routed_scale": c["routed_scaling_factor"], "situ_b1": c["situ_beta"], "situ_b2": c["situ_linear_beta"],
        "latent": c["routed_expert_hidden_size"],
        "shared_inter": c["moe_intermediate_size"] * c["num_shared_experts"],
        "mla_heads": c["num_attention_heads"], "q_lora": c["q_lora_rank"], "kv_lora": c["kv_lora_rank"],
        "qk_nope": c["qk_nope_head_dim"], "qk_rope": c["qk_rope_head_dim"], "v_head": c["v_head_dim"]})


def moe_cfg(k3, c):
    """K3GpuMoeCfg for k3gpu_moe_prefill (the K3 MoE block)."""
    return _fill(k3.K3GpuMoeCfg, {
        "hidden": c["hidden_size"], "latent": c["routed_expert_hidden_size"], "moe_inter": c["moe_intermediate_size"],
        "shared_inter": c["moe_intermediate_size"] * c["num_shared_experts"], "n_routed": c["num_experts"],
        "topk": c["num_experts_per_token"], "act": k3.ACT_SITU, "renorm": int(c["moe_renormalize"]),
        "routed_scale": c["routed_scaling_factor"], "situ_b1": c["situ_beta"], "situ_b2": c["situ_linear_beta"],
        "rms_eps": c["rms_norm_eps"]})
