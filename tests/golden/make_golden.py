"""Regenerate tests/golden/ from the reference's own scalar Python oracle.

Runs rucin93/qwen-mlx-runner's scripts/make_fixture.py (stdlib-only,
double-precision scalar oracle for tiny hybrid models) in a scratch copy, then
stores:
  * tiny-bf16/{model.safetensors,config.json,golden.json}: the packed Q4/g32
    checkpoint with BF16 metadata and the reference's golden logits;
  * tiny-q4/{model.safetensors,config.json,golden.json}: the same model
    quantised with F16 scale/bias (not all BF16-exact, so it loads with f32
    metadata) and its golden logits;
  * matrices.npz: for several packed matrices of that checkpoint the packed
    words, BF16 scale/bias bits, the reference's dequantised values
    (q*scale+bias in f64) and y = mv(name, x) computed by the reference's own
    `mv` for fixed activation vectors.

Usage (needs the reference checkout, only where it is mounted):
    python tests/golden/make_golden.py /path/to/qwen-mlx-runner
"""
from __future__ import annotations

import json
import math
import pathlib
import runpy
import shutil
import struct
import sys
import tempfile

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
MATRICES = [
    "lm_head",
    "model.layers.0.mlp.gate_proj",
    "model.layers.0.mlp.down_proj",
    "model.layers.1.linear_attn.in_proj_qkv",
    "model.layers.3.self_attn.q_proj",
]


def read_safetensors(path: pathlib.Path):
    data = path.read_bytes()
    n = struct.unpack("<Q", data[:8])[0]
    header = json.loads(data[8:8 + n])
    body = data[8 + n:]
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        a, b = meta["data_offsets"]
        out[name] = (meta["dtype"], meta["shape"], body[a:b])
    return out


def main(reference_root: str) -> None:
    script = pathlib.Path(reference_root) / "scripts" / "make_fixture.py"
    with tempfile.TemporaryDirectory() as tmp:
        tmp = pathlib.Path(tmp)
        (tmp / "scripts").mkdir()
        shutil.copy(script, tmp / "scripts" / "make_fixture.py")
        g = runpy.run_path(str(tmp / "scripts" / "make_fixture.py"), run_name="__main__")
        for fixture in ("tiny-bf16", "tiny-q4"):
            dst = HERE / fixture
            dst.mkdir(exist_ok=True)
            for f in ("model.safetensors", "config.json", "golden.json"):
                shutil.copy(tmp / "tests" / "fixtures" / fixture / f, dst / f)
        src = tmp / "tests" / "fixtures" / "tiny-bf16"
        tensors = read_safetensors(src / "model.safetensors")
        weights, mv = g["weights"], g["mv"]
        arrays = {}
        for idx, name in enumerate(MATRICES):
            mlx = "language_model." + name
            _, wshape, wbytes = tensors[mlx + ".weight"]
            _, _, sbytes = tensors[mlx + ".scales"]
            _, _, bbytes = tensors[mlx + ".biases"]
            rows, packed_cols = wshape
            cols = packed_cols * 8
            x = [math.sin(0.37 * (i + 1) + idx) * (1.0 + 0.25 * (i % 5)) for i in range(cols)]
            x = [struct.unpack("<f", struct.pack("<f", v))[0] for v in x]  # f32-representable
            y = mv(name, x)
            key = f"m{idx}"
            arrays[key + "_weight"] = np.frombuffer(wbytes, dtype="<u4").reshape(rows, packed_cols)
            arrays[key + "_scales"] = np.frombuffer(sbytes, dtype="<u2").reshape(rows, cols // 32)
            arrays[key + "_biases"] = np.frombuffer(bbytes, dtype="<u2").reshape(rows, cols // 32)
            arrays[key + "_dequant"] = np.array(weights[name + ".weight"], dtype=np.float64).reshape(rows, cols)
            arrays[key + "_x"] = np.array(x, dtype=np.float32)
            arrays[key + "_y"] = np.array(y, dtype=np.float64)
            arrays[key + "_shape"] = np.array([rows, cols, 4, 32], dtype=np.int64)
        np.savez_compressed(HERE / "matrices.npz", names=np.array(MATRICES), **arrays)
    print(f"wrote {HERE / 'matrices.npz'} and {HERE / 'tiny-bf16'}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (a checkout of rucin93/qwen-mlx-runner v0.7.3)")
    main(sys.argv[1])
