"""Test helpers for the decode graph: read the reference's tiny MLX
checkpoints (tests/golden/tiny-*) straight from their safetensors bytes and
hand them to the FP64 oracle; build the synthetic 27B-shaped configuration.

This reader is test infrastructure (it feeds the oracle); the product loads
checkpoints with its own C++ loader (libqmr, qmr_checkpoint_* / qmr_model_load).
"""
from __future__ import annotations

import json
import pathlib
import struct

import numpy as np

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def read_safetensors(path):
    data = pathlib.Path(path).read_bytes()
    n = struct.unpack("<Q", data[:8])[0]
    header = json.loads(data[8:8 + n])
    body = data[8 + n:]
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        a, b = meta["data_offsets"]
        dt = {"U32": "<u4", "F32": "<f4", "F16": "<f2", "BF16": "<u2"}[meta["dtype"]]
        arr = np.frombuffer(body[a:b], dtype=dt).reshape(meta["shape"])
        out[name] = (meta["dtype"], arr)
    return out


def config_of(fixture_dir, context=8):
    c = json.loads((pathlib.Path(fixture_dir) / "config.json").read_text())
    t = c["text_config"]
    rope = t["rope_parameters"]
    return dict(hidden=t["hidden_size"], inter=t["intermediate_size"], layers=t["num_hidden_layers"],
                heads=t["num_attention_heads"], kv_heads=t["num_key_value_heads"], head_dim=t["head_dim"],
                vocab=t["vocab_size"], lin_key_heads=t["linear_num_key_heads"],
                lin_value_heads=t["linear_num_value_heads"], lin_key_dim=t["linear_key_head_dim"],
                lin_value_dim=t["linear_value_head_dim"], conv_width=t["linear_conv_kernel_dim"],
                rotary_dim=int(t["head_dim"] * rope["partial_rotary_factor"]), eps=t["rms_norm_eps"],
                theta=rope["rope_theta"], is_attn=[s == "full_attention" for s in t["layer_types"]],
                context=context, quant=c["quantization"])


def _f32(dtype, arr):
    if dtype == "BF16":
        return (arr.astype(np.uint32) << 16).view(np.float32)
    return arr.astype(np.float32)


def tiny_oracle(fixture_dir, context=8):
    """DecodeOracle loaded with a tiny MLX checkpoint (names `language_model.*`,
    norms already +1, metadata as stored: BF16 bits or F16 widened to f32)."""
    import oracle
    cfg = config_of(fixture_dir, context)
    t = read_safetensors(pathlib.Path(fixture_dir) / "model.safetensors")
    bits, group = cfg["quant"]["bits"], cfg["quant"]["group_size"]
    o = oracle.DecodeOracle(cfg)

    def mat(prefix):
        _, w = t[prefix + ".weight"]
        sd, s = t[prefix + ".scales"]
        bd, b = t[prefix + ".biases"]
        meta_s = s if sd == "BF16" else _f32(sd, s)
        meta_b = b if bd == "BF16" else _f32(bd, b)
        rows = w.shape[0]
        cols = w.shape[1] * 32 // bits
        return dict(weight=w, scales=meta_s, biases=meta_b), rows, cols

    def vec(name):
        d, a = t[name]
        return _f32(d, a).ravel()

    m, r, c = mat("language_model.model.embed_tokens")
    o.set_matrix(-1, "embed", m, r, c, bits, group)
    m, r, c = mat("language_model.lm_head")
    o.set_matrix(-1, "head", m, r, c, bits, group)
    o.set_vector(-1, None, vec("language_model.model.norm.weight"))
    for li, att in enumerate(cfg["is_attn"]):
        p = f"language_model.model.layers.{li}"
        o.set_vector(li, "input_norm", vec(p + ".input_layernorm.weight"))
        o.set_vector(li, "post_norm", vec(p + ".post_attention_layernorm.weight"))
        for name in ("gate", "up", "down"):
            m, r, c = mat(f"{p}.mlp.{name}_proj")
            o.set_matrix(li, name, m, r, c, bits, group)
        if att:
            for name in ("q", "k", "v", "o"):
                m, r, c = mat(f"{p}.self_attn.{name}_proj")
                o.set_matrix(li, name, m, r, c, bits, group)
            o.set_vector(li, "q_norm", vec(p + ".self_attn.q_norm.weight"))
            o.set_vector(li, "k_norm", vec(p + ".self_attn.k_norm.weight"))
        else:
            for name, tname in (("qkv", "in_proj_qkv"), ("z", "in_proj_z"), ("a", "in_proj_a"),
                                ("b", "in_proj_b"), ("out", "out_proj")):
                m, r, c = mat(f"{p}.linear_attn.{tname}")
                o.set_matrix(li, name, m, r, c, bits, group)
            o.set_vector(li, "conv", vec(p + ".linear_attn.conv1d.weight"))
            o.set_vector(li, "A_log", vec(p + ".linear_attn.A_log"))
            o.set_vector(li, "dt_bias", vec(p + ".linear_attn.dt_bias"))
            o.set_vector(li, "delta_norm", vec(p + ".linear_attn.norm.weight"))
    return o, cfg


def golden(fixture_dir):
    g = json.loads((pathlib.Path(fixture_dir) / "golden.json").read_text())
    return g["tokens"], np.array(g["logits"], dtype=np.float64)
