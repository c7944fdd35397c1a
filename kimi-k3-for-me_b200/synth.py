"""Synthetic K3-architecture checkpoints (host, numpy): seeded random weights written in the
released checkpoint's safetensors layout, so the same directory loads into this library
(``Model.from_checkpoint``) and into the reference engine (its ``bin/k3 <dir>``).

The tensor set, names, dtypes and shapes are the ones the reference binds
(src/model/k3_bind.c:160-240, 485-500; src/io/k3_load.c:11): the trunk's large matrices
in bf16 (stored by truncating fp32, as the reference's tiny-checkpoint writer does,
tools/make_tiny_checkpoint.py:73-74), norms, biases, convolutions, A_log (padded to
kda_head_dim, its first kda_num_heads entries meaningful), dt_bias and the router in
fp32, and every routed expert as MXFP4 (``weight_packed`` [rows][cols/2] with the even
element in the low nibble, ``weight_scale`` [rows][cols/32] E8M0). The configuration is
the flat shape the reference's config loader reads.

Two initialisation recipes:
  "reference"  the reference tiny-checkpoint generator's (tools/make_tiny_checkpoint.py:
               205-231): matrices N(0, 0.02), 1-D weights 1, other vectors 0, then expert
               w1/w3 (routed and shared) N(0, 1.2) so the SiTU caps engage, the routing
               bias linspace(-0.15, 0.15) so it reorders selection, A_log linspace(-0.4,
               1.2) over the heads, dt_bias N(0, 0.5), ShortConv weights N(0, 0.4);
  "baseline"   the benchmark text's: every matrix, experts included, N(0, 0.02), the
               routing bias N(0, 0.01), and the reference recipe's KDA vectors.
Draws come from numpy's PCG64 (``default_rng(seed)``) in tensor-name order, so a
directory is reproduced exactly from (config, seed, recipe) on any machine; it is not the
byte stream of the reference's torch-seeded generator.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

PRE = "language_model.model."

# 4 layers in a 3:1 KDA:MLA pattern, d_model 512, 8 heads of 64, MLA
# kv_lora 128 / rope 32, 16 routed experts top-2 + 1 shared, expert FFN 256, vocab 1024
CONFIG1 = {
    "hidden_size": 512, "num_hidden_layers": 4, "vocab_size": 1024, "rms_norm_eps": 1e-5,
    "kda_num_heads": 8, "kda_head_dim": 64, "short_conv_kernel_size": 4, "gate_lower_bound": -5.0,
    "num_attention_heads": 8, "q_lora_rank": 256, "kv_lora_rank": 128, "qk_nope_head_dim": 64,
    "qk_rope_head_dim": 32, "v_head_dim": 64, "mla_use_output_gate": True,
    "num_experts": 16, "num_experts_per_token": 2, "num_shared_experts": 1,
    "routed_expert_hidden_size": 512, "moe_intermediate_size": 256, "routed_scaling_factor": 1.0,
    "moe_renormalize": True, "latent_moe_use_norm": True, "first_k_dense_replace": 0,
    "intermediate_size": 256, "attn_res_block_size": 2, "situ_beta": 4.0, "situ_linear_beta": 25.0,
    "full_attn_layers": [4],
}

E2M1_MIDS = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)


def mxfp4_quant(w: np.ndarray):
    """[R][C] fp32 -> (packed [R][C/2] u8, scales [R][C/32] u8): per 32 elements the scale
    2^(floor(log2 amax) - 2) (E8M0, biased by 127), each element the nearest E2M1 value
    (ties to the smaller magnitude), the sign from the element, the even element in the
    low nibble -- the quantisation rule of the reference's checkpoint writer
    (tools/make_tiny_checkpoint.py:88-138)."""
    w = np.asarray(w, np.float32)
    R, C = w.shape
    g = C // 32
    blocks = w.reshape(R, g, 32)
    amax = np.abs(blocks).max(axis=2)
    ex = np.clip(np.floor(np.log2(np.maximum(amax, 1e-30))) - 2, -127, 127).astype(np.int32)
    scales = (ex + 127).astype(np.uint8)
    xq = blocks / np.exp2(ex.astype(np.float32)).reshape(R, g, 1)
    mag = np.searchsorted(E2M1_MIDS, np.abs(xq).ravel(), side="left").astype(np.uint8).reshape(xq.shape)
    nib = np.where(xq < 0, mag | 0x8, mag).astype(np.uint8)
    packed = (nib[:, :, 0::2] | (nib[:, :, 1::2] << 4)).reshape(R, C // 2)
    return np.ascontiguousarray(packed), np.ascontiguousarray(scales)


def bf16_trunc(w: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits by truncation (the reference writer's bf16_of)."""
    return (np.ascontiguousarray(w, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def tensor_plan(cfg: dict):
    """[(name, shape, kind)] for every tensor of the model, kind one of
    bf16 / f32 / norm (1-D weight) / vec (1-D, zero) / expert, in writing order."""
    E, V = cfg["hidden_size"], cfg["vocab_size"]
    H, D, K = cfg["kda_num_heads"], cfg["kda_head_dim"], cfg["short_conv_kernel_size"]
    P = H * D
    Hm, ql, kvl = cfg["num_attention_heads"], cfg["q_lora_rank"], cfg["kv_lora_rank"]
    nope, rope, vh = cfg["qk_nope_head_dim"], cfg["qk_rope_head_dim"], cfg["v_head_dim"]
    n, L, I = cfg["num_experts"], cfg["routed_expert_hidden_size"], cfg["moe_intermediate_size"]
    SI = I * cfg["num_shared_experts"]
    mla = set(x - 1 for x in cfg["full_attn_layers"])
    plan = []
    for li in range(cfg["num_hidden_layers"]):
        p = f"{PRE}layers.{li}."
        if li in mla:
            plan += [(p + "self_attn.q_a_proj.weight", (ql, E), "bf16"),
                     (p + "self_attn.q_a_layernorm.weight", (ql,), "norm"),
                     (p + "self_attn.q_b_proj.weight", (Hm * (nope + rope), ql), "bf16"),
                     (p + "self_attn.kv_a_proj_with_mqa.weight", (kvl + rope, E), "bf16"),
                     (p + "self_attn.kv_a_layernorm.weight", (kvl,), "norm"),
                     (p + "self_attn.kv_b_proj.weight", (Hm * (nope + vh), kvl), "bf16"),
                     (p + "self_attn.o_proj.weight", (E, Hm * vh), "bf16")]
            if cfg.get("mla_use_output_gate", True):
                plan.append((p + "self_attn.g_proj.weight", (Hm * vh, E), "bf16"))
        else:
            plan += [(p + "self_attn.A_log", (D,), "a_log"),
                     (p + "self_attn.dt_bias", (P,), "dt_bias")]
            for w in ("q", "k", "v"):
                plan.append((p + f"self_attn.{w}_proj.weight", (P, E), "bf16"))
            for w in ("q", "k", "v"):
                plan.append((p + f"self_attn.{w}_conv1d.weight", (P, 1, K), "conv"))
            plan += [(p + "self_attn.f_a_proj.weight", (D, E), "bf16"),
                     (p + "self_attn.f_b_proj.weight", (P, D), "bf16"),
                     (p + "self_attn.b_proj.weight", (H, E), "bf16"),
                     (p + "self_attn.g_proj.weight", (P, E), "bf16"),
                     (p + "self_attn.o_norm.weight", (D,), "norm"),
                     (p + "self_attn.o_proj.weight", (E, P), "bf16")]
        m = p + "block_sparse_moe."
        plan += [(m + "gate.e_score_correction_bias", (n,), "bias"),
                 (m + "gate.weight", (n, E), "f32"),
                 (m + "routed_expert_down_proj.weight", (L, E), "bf16"),
                 (m + "routed_expert_up_proj.weight", (E, L), "bf16"),
                 (m + "routed_expert_norm.weight", (L,), "norm")]
        for e in range(n):
            plan += [(m + f"experts.{e}.w1", (I, L), "expert13"),
                     (m + f"experts.{e}.w3", (I, L), "expert13"),
                     (m + f"experts.{e}.w2", (L, I), "expert2")]
        plan += [(m + "shared_experts.gate_proj.weight", (SI, E), "bf16_13"),
                 (m + "shared_experts.up_proj.weight", (SI, E), "bf16_13"),
                 (m + "shared_experts.down_proj.weight", (E, SI), "bf16")]
        plan += [(p + "input_layernorm.weight", (E,), "norm"),
                 (p + "post_attention_layernorm.weight", (E,), "norm"),
                 (p + "self_attention_res_norm.weight", (E,), "norm"),
                 (p + "self_attention_res_proj.weight", (1, E), "f32"),
                 (p + "mlp_res_norm.weight", (E,), "norm"),
                 (p + "mlp_res_proj.weight", (1, E), "f32")]
    plan += [(PRE + "embed_tokens.weight", (V, E), "bf16"),
             (PRE + "norm.weight", (E,), "norm"),
             ("language_model.lm_head.weight", (V, E), "bf16"),
             (PRE + "output_attn_res_norm.weight", (E,), "norm"),
             (PRE + "output_attn_res_proj.weight", (1, E), "f32")]
    return plan


def make_tensors(cfg: dict, seed: int = 0, recipe: str = "reference"):
    """{name: array} for the checkpoint (experts as their _packed/_scale pair)."""
    if recipe not in ("reference", "baseline"):
        raise ValueError(f"unknown recipe {recipe!r}")
    rng = np.random.default_rng(seed)
    H = cfg["kda_num_heads"]
    std13 = 1.2 if recipe == "reference" else 0.02
    out = {}
    for name, shape, kind in tensor_plan(cfg):
        f32 = lambda std: (rng.standard_normal(shape, dtype=np.float32) * np.float32(std))  # noqa: E731
        if kind in ("expert13", "expert2"):
            w = f32(std13 if kind == "expert13" else 0.02)
            packed, scales = mxfp4_quant(w)
            out[name + ".weight_packed"] = packed
            out[name + ".weight_scale"] = scales
        elif kind in ("bf16", "bf16_13"):
            out[name] = bf16_trunc(f32(std13 if kind == "bf16_13" else 0.02))
        elif kind == "f32":
            out[name] = f32(0.02)
        elif kind == "conv":
            out[name] = f32(0.4)
        elif kind == "norm":
            out[name] = np.ones(shape, np.float32)
        elif kind == "bias":
            out[name] = (np.linspace(-0.15, 0.15, shape[0]).astype(np.float32) if recipe == "reference"
                         else f32(0.01))
        elif kind == "a_log":
            a = np.zeros(shape, np.float32)
            a[:H] = np.linspace(-0.4, 1.2, H).astype(np.float32)
            out[name] = a
        elif kind == "dt_bias":
            out[name] = f32(0.5)
        else:
            raise AssertionError(kind)
    return out


def write_safetensors(path: str, tensors: dict) -> None:
    header, off = {}, 0
    codes = {np.dtype("uint8"): "U8", np.dtype("uint16"): "BF16", np.dtype("float32"): "F32"}
    for name, a in tensors.items():
        nb = a.nbytes
        header[name] = {"dtype": codes[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + nb]}
        off += nb
    hj = json.dumps(header).encode("utf-8")
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for a in tensors.values():
            f.write(np.ascontiguousarray(a).tobytes())


def write_checkpoint(out_dir: str, cfg: dict = None, seed: int = 0, recipe: str = "reference") -> str:
    """config.json + model.safetensors under out_dir; returns out_dir."""
    cfg = dict(CONFIG1 if cfg is None else cfg)
    os.makedirs(out_dir, exist_ok=True)
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    write_safetensors(os.path.join(out_dir, "model.safetensors"), make_tensors(cfg, seed, recipe))
    return out_dir
