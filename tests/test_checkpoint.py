"""The C++ checkpoint loader (qmr_checkpoint_*, the reference's
src/weights.rs Checkpoint and src/config.rs ModelConfig) on CPU.

* The reference's tiny MLX checkpoints load: config fields, packed words bit
  for bit, BF16 and F16 metadata widened exactly to f32, vectors as stored.
* Its matrices equal the ones the reference's own fixture script wrote
  (tests/golden/matrices.npz).
* Malformed checkpoints fail with the reference's rules: duplicate JSON keys,
  overlapping or holed safetensors data, unsupported dtypes, layer types
  out of the full_attention_interval pattern, MoE fields, quantisation
  without metadata.
* Raw Hugging Face naming (model.* without quantisation, HF conv layout)
  shifts zero-centred norms by +1; MLX names do not.
"""
import json
import pathlib
import struct

import numpy as np
import pytest

import qmr
from qmr._lib import QmrError
from _model_util import GOLDEN, read_safetensors


def f16_to_f32(a):
    """F16 tensors as read_safetensors returns them (float16) widened to f32 (exact)."""
    return np.asarray(a, dtype=np.float16).astype(np.float32)


def bf16_to_f32(a):
    return (np.asarray(a, dtype=np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("fixture", ["tiny-bf16", "tiny-q4"])
def test_tiny_checkpoint_matrices_vectors_and_config(fixture):
    path = GOLDEN / fixture
    cp = qmr.Checkpoint(path)
    cfg = cp.config()
    assert (cfg["hidden"], cfg["inter"], cfg["layers"], cfg["vocab"]) == (32, 64, 4, 64)
    assert cfg["is_attn"] == [False, False, False, True]
    assert cfg["rotary_dim"] == 16 and cfg["max_position"] == 128 and not cfg["tied"]
    raw = read_safetensors(path / "model.safetensors")
    for name in ["model.embed_tokens", "lm_head", "model.layers.0.linear_attn.in_proj_qkv",
                 "model.layers.3.self_attn.o_proj", "model.layers.2.mlp.down_proj"]:
        m = cp.matrix(name)
        mlx = "language_model." + name
        _, w = raw[mlx + ".weight"]
        sd, s = raw[mlx + ".scales"]
        bd, b = raw[mlx + ".biases"]
        assert (m["rows"], m["bits"], m["group"]) == (w.shape[0], 4, 32)
        assert m["cols"] == w.shape[1] * 8
        assert np.array_equal(m["weight"], w)
        widen = bf16_to_f32 if sd == "BF16" else f16_to_f32
        assert np.array_equal(m["scales"].view(np.uint32), widen(s).view(np.uint32))
        assert np.array_equal(m["biases"].view(np.uint32), widen(b).view(np.uint32))
    d, v = raw["language_model.model.layers.0.input_layernorm.weight"]
    assert np.array_equal(cp.vector("model.layers.0.input_layernorm"), v)  # MLX norms: already +1
    d, v = raw["language_model.model.layers.1.linear_attn.A_log"]
    assert np.array_equal(cp.vector("model.layers.1.linear_attn.A_log"), f16_to_f32(v))
    with pytest.raises(QmrError):
        cp.matrix("model.layers.0.mlp.missing_proj")
    with pytest.raises(QmrError):
        cp.vector("model.layers.0.mlp.gate_proj")  # rank 2 is not a vector
    cp.close()


def test_loader_matrices_equal_the_reference_fixture_dump():
    data = np.load(GOLDEN / "matrices.npz")
    cp = qmr.Checkpoint(GOLDEN / "tiny-bf16")
    for idx, name in enumerate(data["names"]):
        m = cp.matrix(str(name))
        assert np.array_equal(m["weight"], data[f"m{idx}_weight"])
        assert np.array_equal(m["scales"], bf16_to_f32(data[f"m{idx}_scales"]))
        assert np.array_equal(m["biases"], bf16_to_f32(data[f"m{idx}_biases"]))
    cp.close()


# ---- synthetic checkpoints for the error rules ------------------------------------

def write_safetensors(path, tensors, raw_header=None, body_extra=b""):
    """tensors: [(name, dtype, shape, bytes)]."""
    header, body = {}, b""
    for name, dtype, shape, data in tensors:
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [len(body), len(body) + len(data)]}
        body += data
    hdr = raw_header.encode() if raw_header is not None else json.dumps(header).encode()
    hdr += b" " * ((-len(hdr)) % 8)
    path.write_bytes(struct.pack("<Q", len(hdr)) + hdr + body + body_extra)


def small_config(**over):
    t = {"model_type": "qwen3_5_text", "hidden_size": 8, "intermediate_size": 16, "num_hidden_layers": 2,
         "num_attention_heads": 2, "num_key_value_heads": 1, "head_dim": 4, "vocab_size": 32,
         "linear_num_key_heads": 2, "linear_num_value_heads": 2, "linear_key_head_dim": 4,
         "linear_value_head_dim": 4, "linear_conv_kernel_dim": 4, "full_attention_interval": 2,
         "rms_norm_eps": 1e-6, "rope_theta": 10000, "partial_rotary_factor": 0.5, "max_position_embeddings": 128,
         "layer_types": ["linear_attention", "full_attention"]}
    t.update(over)
    return {"model_type": "qwen3_5", "text_config": t}


def make_checkpoint(tmp_path, config=None, tensors=None, **kw):
    d = tmp_path / "ckpt"
    d.mkdir(exist_ok=True)
    (d / "config.json").write_text(json.dumps(config or small_config()))
    f32 = lambda v: np.asarray(v, np.float32).tobytes()  # noqa: E731
    write_safetensors(d / "model.safetensors", tensors or [("model.norm.weight", "F32", [8], f32(np.zeros(8)))],
                      **kw)
    return d


def test_config_rules(tmp_path):
    make_checkpoint(tmp_path)
    cp = qmr.Checkpoint(tmp_path / "ckpt")
    cfg = cp.config()
    assert cfg["is_attn"] == [False, True] and cfg["rotary_dim"] == 2
    cp.close()
    bad = [small_config(layer_types=["full_attention", "full_attention"]),
           small_config(num_experts=8),
           small_config(hidden_act="gelu"),
           small_config(num_attention_heads=3, num_key_value_heads=2),
           small_config(partial_rotary_factor=0.25),  # rotary dim 1 is odd
           {"model_type": "llama", "text_config": small_config()["text_config"]}]
    for i, c in enumerate(bad):
        (tmp_path / f"b{i}").mkdir()
        d = make_checkpoint(tmp_path / f"b{i}", config=c)
        with pytest.raises(QmrError):
            qmr.Checkpoint(d)


def test_safetensors_rules(tmp_path):
    f32 = lambda v: np.asarray(v, np.float32).tobytes()  # noqa: E731
    cases = {
        "duplicate key": dict(raw_header='{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4]},'
                                         '"a":{"dtype":"F32","shape":[1],"data_offsets":[4,8]}}',
                              tensors=[("a", "F32", [2], f32([1, 2]))]),
        "trailing bytes": dict(body_extra=b"\0" * 4),
        "unsupported dtype": dict(tensors=[("a", "C64", [1], b"\0" * 8)]),
        "length mismatch": dict(tensors=[("a", "F32", [3], f32([1, 2]))]),
        "zero dimension": dict(tensors=[("a", "F32", [0], b"")]),
    }
    for i, (what, kw) in enumerate(cases.items()):
        d = tmp_path / f"c{i}"
        d.mkdir()
        with pytest.raises(QmrError):
            qmr.Checkpoint(make_checkpoint(d, **kw))


def test_quantisation_and_hf_norm_offset(tmp_path):
    f32 = lambda v: np.asarray(v, np.float32).tobytes()  # noqa: E731
    words = np.arange(8 * 1, dtype=np.uint32)  # 8 rows x 8 columns at 4 bits = 1 word per row
    scales = np.full((8, 1), 0.5, np.float32)
    conv_hf = ("model.layers.0.linear_attn.conv1d.weight", "F32", [24, 1, 4], f32(np.zeros(96)))
    # Raw HF names, no quantisation metadata: packed U32 matrices are rejected, zero-centred norms get +1.
    d = tmp_path / "hf"
    d.mkdir()
    make_checkpoint(d, tensors=[("model.norm.weight", "F32", [8], f32(np.zeros(8))), conv_hf,
                                ("model.layers.0.mlp.gate_proj.weight", "U32", [8, 1], words.tobytes())])
    cp = qmr.Checkpoint(d / "ckpt")
    assert np.array_equal(cp.vector("model.norm"), np.ones(8, np.float32))
    with pytest.raises(QmrError, match="quantization"):
        cp.matrix("model.layers.0.mlp.gate_proj")
    cp.close()
    # MLX names with a quantisation config (group 8): metadata found, no norm offset.
    cfg = small_config()
    cfg["quantization"] = {"bits": 4, "group_size": 8, "mode": "affine"}
    d = tmp_path / "mlx"
    d.mkdir()
    make_checkpoint(d, config=cfg, tensors=[
        ("language_model.model.norm.weight", "F32", [8], f32(np.zeros(8))),
        ("language_model.model.layers.0.mlp.gate_proj.weight", "U32", [8, 1], words.tobytes()),
        ("language_model.model.layers.0.mlp.gate_proj.scales", "F32", [8, 1], scales.tobytes()),
        ("language_model.model.layers.0.mlp.gate_proj.biases", "F32", [8, 1], scales.tobytes())])
    cp = qmr.Checkpoint(d / "ckpt")
    assert np.array_equal(cp.vector("model.norm"), np.zeros(8, np.float32))
    m = cp.matrix("model.layers.0.mlp.gate_proj")
    assert (m["rows"], m["cols"], m["bits"], m["group"]) == (8, 8, 4, 8)
    assert np.array_equal(m["weight"].ravel(), words)
    cp.close()
