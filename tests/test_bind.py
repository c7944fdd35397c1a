"""Binding a checkpoint's trunk tensors to the layer weight structures (bind.Binder), CPU.

Shards are written here with the checkpoint's tensor names (src/model/k3_bind.c:174-239,
495-500) for a small configuration in the released config's keys: layer kinds from the
one-based full_attn_layers and first_k_dense_replace, projections stored bf16 (one stored
fp32, so it must be rounded to nearest even and reported), norms fp32 and f16, A_log with
kda_head_dim entries of which the first kda_num_heads count. Every bound field must be
the stored tensor in the dtype the structure takes, the AttnRes folds the products, and a
missing tensor or a wrong element count must be refused by name.
"""
import json
import os
import struct
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from k3lib import load  # noqa: E402

torch = pytest.importorskip("torch")

CFG = {"hidden_size": 32, "num_hidden_layers": 4, "vocab_size": 64, "kda_num_heads": 2, "kda_head_dim": 8,
       "short_conv_kernel_size": 4, "num_attention_heads": 2, "q_lora_rank": 16, "kv_lora_rank": 8,
       "qk_nope_head_dim": 6, "qk_rope_head_dim": 4, "v_head_dim": 4, "mla_use_output_gate": True,
       "num_experts": 4, "num_shared_experts": 2, "routed_expert_hidden_size": 16, "moe_intermediate_size": 8,
       "first_k_dense_replace": 1, "intermediate_size": 24, "full_attn_layers": [2, 4]}
FP32_PROJ = "language_model.model.layers.2.self_attn.q_proj.weight"     # stored fp32
F16_NORM = "language_model.model.layers.3.input_layernorm.weight"       # stored f16


@pytest.fixture(scope="module")
def k3():
    return load()


def _bind_mod():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bind", os.path.join(os.path.dirname(HERE), "kimi-k3-for-me_b200",
                                                                       "bind.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def bf16_bits(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).view(torch.int16).numpy() \
        .view(np.uint16)


def tensors(rng):
    """name -> (float32 values, stored dtype) for the whole small model."""
    c, E = CFG, CFG["hidden_size"]
    t = {}
    P = c["kda_num_heads"] * c["kda_head_dim"]
    Hm, ql, kvl = c["num_attention_heads"], c["q_lora_rank"], c["kv_lora_rank"]
    nope, rope, vh = c["qk_nope_head_dim"], c["qk_rope_head_dim"], c["v_head_dim"]
    SI = c["moe_intermediate_size"] * c["num_shared_experts"]
    r = lambda *s: rng.standard_normal(s).astype(np.float32)    # noqa: E731
    for L in range(c["num_hidden_layers"]):
        p = f"language_model.model.layers.{L}."
        for n in ("input_layernorm", "post_attention_layernorm", "self_attention_res_norm",
                  "self_attention_res_proj", "mlp_res_norm", "mlp_res_proj"):
            t[p + n + ".weight"] = (r(E), "F32")
        if (L + 1) in c["full_attn_layers"]:
            a = p + "self_attn."
            t[a + "q_a_proj.weight"] = (r(ql, E), "BF16")
            t[a + "q_a_layernorm.weight"] = (r(ql), "F32")
            t[a + "q_b_proj.weight"] = (r(Hm * (nope + rope), ql), "BF16")
            t[a + "kv_a_proj_with_mqa.weight"] = (r(kvl + rope, E), "BF16")
            t[a + "kv_a_layernorm.weight"] = (r(kvl), "F32")
            t[a + "kv_b_proj.weight"] = (r(Hm * (nope + vh), kvl), "BF16")
            t[a + "o_proj.weight"] = (r(E, Hm * vh), "BF16")
            t[a + "g_proj.weight"] = (r(Hm * vh, E), "BF16")
        else:
            a = p + "self_attn."
            for n in ("q", "k", "v", "g"):
                t[a + f"{n}_proj.weight"] = (r(P, E), "BF16")
            t[a + "o_proj.weight"] = (r(E, P), "BF16")
            for n in ("q", "k", "v"):
                t[a + f"{n}_conv1d.weight"] = (r(P, 1, c["short_conv_kernel_size"]), "F32")
            t[a + "f_a_proj.weight"] = (r(c["kda_head_dim"], E), "BF16")
            t[a + "f_b_proj.weight"] = (r(P, c["kda_head_dim"]), "BF16")
            t[a + "b_proj.weight"] = (r(c["kda_num_heads"], E), "BF16")
            t[a + "A_log"] = (r(c["kda_head_dim"]), "F32")
            t[a + "dt_bias"] = (r(P), "F32")
            t[a + "o_norm.weight"] = (r(c["kda_head_dim"]), "F32")
        if L < c["first_k_dense_replace"]:
            DI = c["intermediate_size"]
            t[p + "mlp.gate_proj.weight"] = (r(DI, E), "BF16")
            t[p + "mlp.up_proj.weight"] = (r(DI, E), "BF16")
            t[p + "mlp.down_proj.weight"] = (r(E, DI), "BF16")
        else:
            m = p + "block_sparse_moe."
            n, Lt = c["num_experts"], c["routed_expert_hidden_size"]
            t[m + "gate.weight"] = (r(n, E), "F32")
            t[m + "gate.e_score_correction_bias"] = (r(n), "F32")
            t[m + "routed_expert_down_proj.weight"] = (r(Lt, E), "BF16")
            t[m + "routed_expert_up_proj.weight"] = (r(E, Lt), "BF16")
            t[m + "routed_expert_norm.weight"] = (r(Lt), "F32")
            t[m + "shared_experts.gate_proj.weight"] = (r(SI, E), "BF16")
            t[m + "shared_experts.up_proj.weight"] = (r(SI, E), "BF16")
            t[m + "shared_experts.down_proj.weight"] = (r(E, SI), "BF16")
    t["language_model.model.embed_tokens.weight"] = (r(c["vocab_size"], E), "BF16")
    t["language_model.model.norm.weight"] = (r(E), "F32")
    t["language_model.model.output_attn_res_norm.weight"] = (r(E), "F32")
    t["language_model.model.output_attn_res_proj.weight"] = (r(E), "F32")
    t["language_model.lm_head.weight"] = (r(c["vocab_size"], E), "BF16")
    t[FP32_PROJ] = (t[FP32_PROJ][0], "F32")
    t[F16_NORM] = (t[F16_NORM][0], "F16")
    return t


def stored(vals, dt):
    if dt == "BF16":
        return bf16_bits(vals).tobytes()
    if dt == "F16":
        return vals.astype(np.float16).tobytes()
    return vals.astype(np.float32).tobytes()


def write(path, t):
    header, blobs, off = {"__metadata__": {"format": "pt"}}, [], 0
    for name, (vals, dt) in t.items():
        raw = stored(vals, dt)
        header[name] = {"dtype": dt, "shape": list(vals.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def as_stored_f32(vals, dt):
    if dt == "BF16":
        return (bf16_bits(vals).astype(np.uint32) << 16).view(np.float32)
    if dt == "F16":
        return vals.astype(np.float16).astype(np.float32)
    return vals.astype(np.float32)


def test_binds_every_layer_and_the_model(k3, tmp_path):
    b = _bind_mod()
    rng = np.random.default_rng(3)
    t = tensors(rng)
    names = list(t)
    write(str(tmp_path / "model-00001-of-00002.safetensors"), {n: t[n] for n in names[: len(names) // 2]})
    write(str(tmp_path / "model-00002-of-00002.safetensors"), {n: t[n] for n in names[len(names) // 2:]})
    idx = k3.SafetensorsIndex(str(tmp_path))
    bd = b.Binder(idx, CFG)
    kinds = [bd.layer(L)["kind"] for L in range(4)]
    assert kinds == ["kda", "mla", "kda", "mla"]            # full_attn_layers [2, 4] is one-based
    for L in range(4):
        f = bd.layer(L)
        p = f"language_model.model.layers.{L}."
        assert f["dense"] == (L == 0)
        v = lambda n: as_stored_f32(*t[p + n])               # noqa: E731
        np.testing.assert_array_equal(f["in_norm"], v("input_layernorm.weight"))
        np.testing.assert_array_equal(f["attn_res_fold"], v("self_attention_res_norm.weight") *
                                      v("self_attention_res_proj.weight"))
        np.testing.assert_array_equal(f["mlp_res_fold"], v("mlp_res_norm.weight") * v("mlp_res_proj.weight"))
        if f["kind"] == "kda":
            np.testing.assert_array_equal(f["q"], bf16_bits(t[p + "self_attn.q_proj.weight"][0]).reshape(-1))
            np.testing.assert_array_equal(f["q_conv"], v("self_attn.q_conv1d.weight").reshape(-1))
            np.testing.assert_array_equal(f["A_log"], v("self_attn.A_log")[:CFG["kda_num_heads"]])
            assert f["b"].dtype == np.uint16 and f["dt_bias"].dtype == np.float32
        else:
            np.testing.assert_array_equal(f["kv_b"], v("self_attn.kv_b_proj.weight").reshape(-1))
            np.testing.assert_array_equal(f["q_b"], bf16_bits(t[p + "self_attn.q_b_proj.weight"][0]).reshape(-1))
            assert f["g"] is not None and f["kv_b"].dtype == np.float32
        if f["dense"]:
            assert f["dense_down"].size == CFG["hidden_size"] * CFG["intermediate_size"]
        else:
            np.testing.assert_array_equal(f["gate_W"], v("block_sparse_moe.gate.weight").reshape(-1))
            assert f["sh2"].dtype == np.uint16
    assert set(bd.converted) == {FP32_PROJ}                   # rounded to bf16 and reported
    m = bd.model()
    np.testing.assert_array_equal(m["lm_head"], bf16_bits(t["language_model.lm_head.weight"][0]).reshape(-1))
    np.testing.assert_array_equal(m["out_res_fold"], as_stored_f32(*t["language_model.model.output_attn_res_norm"
                                                                       ".weight"]) *
                                  as_stored_f32(*t["language_model.model.output_attn_res_proj.weight"]))
    idx.close()


def test_refuses_missing_and_misshaped_tensors(k3, tmp_path):
    b = _bind_mod()
    rng = np.random.default_rng(4)
    t = tensors(rng)
    missing = "language_model.model.layers.1.self_attn.kv_a_layernorm.weight"
    del t[missing]
    bad = "language_model.model.layers.2.block_sparse_moe.gate.e_score_correction_bias"
    t[bad] = (rng.standard_normal(CFG["num_experts"] + 1).astype(np.float32), "F32")
    write(str(tmp_path / "m.safetensors"), t)
    idx = k3.SafetensorsIndex(str(tmp_path))
    bd = b.Binder(idx, CFG)
    bd.layer(0)
    with pytest.raises(b.BindError, match="kv_a_layernorm"):
        bd.layer(1)
    with pytest.raises(b.BindError, match="e_score_correction_bias has 5 elements"):
        bd.layer(2)
    idx.close()


def test_bound_fields_fill_the_layer_structures(k3, tmp_path):
    """Every field K3GpuKdaW, K3GpuMlaW, K3GpuMoeW (the K3 form) and the decoder layer
    structures read comes out of the binder under the same name, so the package's
    kda_weights / mla_weights / moe_weights and decoder-layer wrappers take to_device's
    tensors as they are (those wrappers accept only CUDA tensors; here the names and
    dtypes are checked)."""
    b = _bind_mod()
    write(str(tmp_path / "m.safetensors"), tensors(np.random.default_rng(5)))
    idx = k3.SafetensorsIndex(str(tmp_path))
    bd = b.Binder(idx, CFG)
    kda, mla = bd.layer(2), bd.layer(3)
    layer_fields = {"attn_res_fold", "mlp_res_fold", "in_norm", "post_norm", "gate_W", "gate_bias"}
    moe_fields = {"down", "up", "sh1", "sh3", "sh2", "gate_W", "gate_bias", "latent_norm"}
    assert {n for n, _ in k3.K3GpuKdaW._fields_} | layer_fields | moe_fields <= set(kda)
    assert {n for n, _ in k3.K3GpuMlaW._fields_} | layer_fields | moe_fields <= set(mla)
    dk = b.to_device(kda, "cpu")
    assert "kind" not in dk and "dense" not in dk
    for n, _ in k3.K3GpuKdaW._fields_:
        assert dk[n].dtype == (torch.int16 if kda[n].dtype == np.uint16 else torch.float32), n
    assert dk["q"].numel() == CFG["kda_num_heads"] * CFG["kda_head_dim"] * CFG["hidden_size"]
    assert dk["A_log"].numel() == CFG["kda_num_heads"]
    idx.close()
