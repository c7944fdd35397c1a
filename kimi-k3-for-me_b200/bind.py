"""Binding a checkpoint's trunk tensors to this library's layer weight structures (host
numpy, no GPU): the reference's k3_bind (src/model/k3_bind.c:160-240 per layer, :485-500
model level) for K3GpuKdaW / K3GpuMlaW / K3GpuMoeW / K3GpuKdaLayerW.

Each field is looked up by the checkpoint's name, its element count checked against the
configuration (a disagreement means every kernel downstream would read the wrong
strides; the reference refuses it, and so does this), and converted to what the
structure takes: projections as bf16 bit patterns (uint16; an fp32 or f16 tensor is
rounded to nearest even and listed in `converted`), norms, convolutions, decay
parameters, the router and MLA's kv_b as fp32. The AttnRes pairs are folded at load
(norm weight x scoring projection, in float), as the layer structures take them. The
routed experts' U8 runs come from k3_bank_read_safetensors, not from here.

`index` is anything with info(name) -> {"dtype", "shape", ...} and read(name) -> array
(the package's SafetensorsIndex); `cfg` uses the released config's keys (hidden_size,
kda_num_heads, full_attn_layers ONE-based, ...).
"""
from __future__ import annotations

import numpy as np

PRE = "language_model.model."
ST_U8, ST_BF16, ST_F16, ST_F32 = 1, 2, 3, 4


class BindError(ValueError):
    """A tensor the configuration needs is missing or has the wrong element count."""


def _to_f32(a, dtype):
    if dtype == ST_BF16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    if dtype in (ST_F16, ST_F32):
        return a.astype(np.float32)
    raise BindError(f"dtype code {dtype} cannot be widened to fp32")


def _to_bf16(a, dtype):
    if dtype == ST_BF16:
        return a.astype(np.uint16)
    x = _to_f32(a, dtype).reshape(-1)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)    # round to nearest even
    nan = np.isnan(x)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)                # keep NaN a NaN
    return r.reshape(a.shape)


def is_mla(cfg, layer):
    """The released config lists full_attn_layers one-based (src/core/k3_ops.c:119-127)."""
    return (layer + 1) in cfg.get("full_attn_layers", [])


def is_dense(cfg, layer):
    return layer < cfg.get("first_k_dense_replace", 0)


class Binder:
    def __init__(self, index, cfg):
        self.index, self.cfg = index, cfg
        self.converted: list[str] = []

    def _get(self, name, want, narrow, take=None):
        try:
            info = self.index.info(name)
        except Exception as e:  # noqa: BLE001 -- the index's own error type
            raise BindError(f"missing tensor {name}") from e
        have = int(np.prod(info["shape"])) if info["shape"] else 1
        if have != want:
            raise BindError(f"{name} has {have} elements, the configuration expects {want}")
        a = self.index.read(name).reshape(-1)
        if narrow:
            if info["dtype"] != ST_BF16:
                self.converted.append(name)
            return _to_bf16(a, info["dtype"])
        out = _to_f32(a, info["dtype"])
        return out[:take] if take is not None else out

    def layer(self, L):
        """One decoder layer's fields: {"kind": "mla"|"kda", "dense": bool, <field>: array}."""
        c = self.cfg
        E = c["hidden_size"]
        pre = f"{PRE}layers.{L}."
        f = {"kind": "mla" if is_mla(c, L) else "kda", "dense": is_dense(c, L)}
        w = lambda n, want, **k: self._get(pre + n, want, False, **k)   # noqa: E731
        nw = lambda n, want: self._get(pre + n, want, True)              # noqa: E731
        f["in_norm"] = w("input_layernorm.weight", E)
        f["post_norm"] = w("post_attention_layernorm.weight", E)
        f["attn_res_fold"] = w("self_attention_res_norm.weight", E) * w("self_attention_res_proj.weight", E)
        f["mlp_res_fold"] = w("mlp_res_norm.weight", E) * w("mlp_res_proj.weight", E)
        if f["kind"] == "mla":
            Hm, ql, kvl = c["num_attention_heads"], c["q_lora_rank"], c["kv_lora_rank"]
            nope, rope, vh = c["qk_nope_head_dim"], c["qk_rope_head_dim"], c["v_head_dim"]
            f["q_a"] = nw("self_attn.q_a_proj.weight", ql * E)
            f["q_a_norm"] = w("self_attn.q_a_layernorm.weight", ql)
            f["q_b"] = nw("self_attn.q_b_proj.weight", Hm * (nope + rope) * ql)
            f["kv_a"] = nw("self_attn.kv_a_proj_with_mqa.weight", (kvl + rope) * E)
            f["kv_a_norm"] = w("self_attn.kv_a_layernorm.weight", kvl)
            f["kv_b"] = w("self_attn.kv_b_proj.weight", Hm * (nope + vh) * kvl)   # fp32 in K3GpuMlaW
            f["o"] = nw("self_attn.o_proj.weight", E * Hm * vh)
            f["g"] = nw("self_attn.g_proj.weight", Hm * vh * E) if c.get("mla_use_output_gate") else None
        else:
            H, D, K = c["kda_num_heads"], c["kda_head_dim"], c["short_conv_kernel_size"]
            P = H * D
            for n in ("q", "k", "v", "g"):
                f[n] = nw(f"self_attn.{n}_proj.weight", P * E)
            f["o"] = nw("self_attn.o_proj.weight", E * P)
            for n in ("q", "k", "v"):
                f[f"{n}_conv"] = w(f"self_attn.{n}_conv1d.weight", P * K)
            f["f_a"] = nw("self_attn.f_a_proj.weight", D * E)
            f["f_b"] = nw("self_attn.f_b_proj.weight", P * D)
            f["b"] = nw("self_attn.b_proj.weight", H * E)
            # per head: the checkpoint ships kda_head_dim values, the first kda_heads meaningful
            f["A_log"] = w("self_attn.A_log", D, take=H)
            f["dt_bias"] = w("self_attn.dt_bias", P)
            f["o_norm"] = w("self_attn.o_norm.weight", D)
        if f["dense"]:
            DI = c["intermediate_size"]
            f["dense_gate"] = nw("mlp.gate_proj.weight", DI * E)
            f["dense_up"] = nw("mlp.up_proj.weight", DI * E)
            f["dense_down"] = nw("mlp.down_proj.weight", E * DI)
        else:
            n, Lt = c["num_experts"], c["routed_expert_hidden_size"]
            SI = c["moe_intermediate_size"] * c["num_shared_experts"]
            f["gate_W"] = w("block_sparse_moe.gate.weight", n * E)
            f["gate_bias"] = w("block_sparse_moe.gate.e_score_correction_bias", n)
            f["down"] = nw("block_sparse_moe.routed_expert_down_proj.weight", Lt * E)
            f["up"] = nw("block_sparse_moe.routed_expert_up_proj.weight", E * Lt)
            f["latent_norm"] = w("block_sparse_moe.routed_expert_norm.weight", Lt)
            f["sh1"] = nw("block_sparse_moe.shared_experts.gate_proj.weight", SI * E)
            f["sh3"] = nw("block_sparse_moe.shared_experts.up_proj.weight", SI * E)
            f["sh2"] = nw("block_sparse_moe.shared_experts.down_proj.weight", E * SI)
        return f

    def model(self, embed=True, lm_head=True):
        """The model-level fields: embed and lm_head bf16 [vocab][E], the final norm and the
        output AttnRes fold fp32 [E]."""
        c = self.cfg
        E, V = c["hidden_size"], c["vocab_size"]
        f = {}
        if embed:
            f["embed"] = self._get(PRE + "embed_tokens.weight", V * E, True)
        f["norm"] = self._get(PRE + "norm.weight", E, False)
        f["out_res_fold"] = self._get(PRE + "output_attn_res_norm.weight", E, False) * \
            self._get(PRE + "output_attn_res_proj.weight", E, False)
        if lm_head:
            f["lm_head"] = self._get("language_model.lm_head.weight", V * E, True)
        return f


def to_device(fields, device="cuda"):
    """The bound arrays as torch tensors on `device` (bf16 bit patterns as int16), keyed as
    the layer wrappers take them (kda_weights, mla_weights, moe_weights and the decoder
    layers); entries that are not arrays (kind, dense, an absent gate) are left out."""
    import torch
    out = {}
    for k, v in fields.items():
        if isinstance(v, np.ndarray):
            a = v.view(np.int16) if v.dtype == np.uint16 else v
            out[k] = torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return out
