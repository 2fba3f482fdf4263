"""Seeded synthetic inputs with the distributions of the benchmark configs.

No public dataset is involved: every input is generated here.  The random
stream is splitmix64 with the constants of the reference's
Sampler::uniform (src/chat.rs:353-359); uniforms are its 53-bit draws,
normals use Box-Muller on two uniforms.  Output is numpy, so the same bytes
feed the device path and the CPU oracle.

Distributions (benchmark configs 0-3):
  Q4/g64: nibbles uniform 0..15, scale uniform [0.002, 0.02] rounded to BF16
          (nearest-even), bias = BF16(-8*scale + N(0, 1e-3)).
  Q8/g64: bytes uniform 0..255, scale uniform [1e-4, 1e-3] -> BF16,
          bias = BF16(-128*scale + N(0, 1e-4)).
  x:      FP32 N(0, 1), token-major [batch, cols].
"""
from __future__ import annotations

import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int, start: int = 0) -> np.ndarray:
    """Outputs start..start+n-1 of splitmix64 seeded with `seed` (vectorised)."""
    with np.errstate(over="ignore"):
        i = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + i * GAMMA
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, n: int) -> np.ndarray:
    """n f64 uniforms in [0, 1): (z >> 11) * 2^-53, as Sampler::uniform."""
    return (splitmix64(seed, n) >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))


def normal(seed: int, n: int) -> np.ndarray:
    """n standard normals (f64) by Box-Muller."""
    m = (n + 1) // 2
    u = uniform(seed, 2 * m)
    u1 = 1.0 - u[:m]  # (0, 1]
    u2 = u[m:]
    r = np.sqrt(-2.0 * np.log(u1))
    out = np.empty(2 * m)
    out[0::2] = r * np.cos(2 * np.pi * u2)
    out[1::2] = r * np.sin(2 * np.pi * u2)
    return out[:n]


def bf16_rne(values) -> np.ndarray:
    """FP32 -> BF16 bits, round to nearest even (finite inputs)."""
    b = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)).astype(np.uint16)


def bf16_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def _sub(seed: int, tag: int) -> int:
    return int(splitmix64(seed ^ (tag * 0xD1B54A32D192ED03 & 0xFFFFFFFFFFFFFFFF), 1)[0])


DISTRIBUTIONS = {
    # bits: (scale_lo, scale_hi, bias_center_factor, bias_sigma)
    4: (0.002, 0.02, -8.0, 1e-3),
    8: (1e-4, 1e-3, -128.0, 1e-4),
}


def affine_matrix(rows: int, cols: int, bits: int = 4, group: int = 64, seed: int = 1, meta: str = "bf16"):
    """Packed affine matrix with the benchmark distributions.

    Returns dict(weight=uint32 [rows, cols*bits/32], scales, biases) with
    metadata as uint16 BF16 bits (meta="bf16") or the same values as f32
    (meta="f32").
    """
    if cols % group or cols % (32 // bits):
        raise ValueError("cols must divide by the group and the pack factor")
    words = rows * cols * bits // 32
    raw = splitmix64(_sub(seed, 1), (words + 1) // 2)
    weight = raw.view(np.uint32)[:words].reshape(rows, cols * bits // 32).copy()
    lo, hi, center, sigma = DISTRIBUTIONS[bits]
    ng = rows * cols // group
    scale32 = (lo + (hi - lo) * uniform(_sub(seed, 2), ng)).astype(np.float32)
    s16 = bf16_rne(scale32)
    scale = bf16_to_f32(s16)
    bias32 = (center * scale.astype(np.float64) + sigma * normal(_sub(seed, 3), ng)).astype(np.float32)
    b16 = bf16_rne(bias32)
    s16 = s16.reshape(rows, cols // group)
    b16 = b16.reshape(rows, cols // group)
    if meta == "bf16":
        return dict(weight=weight, scales=s16, biases=b16)
    if meta == "f32":
        return dict(weight=weight, scales=bf16_to_f32(s16).reshape(s16.shape),
                    biases=bf16_to_f32(b16).reshape(b16.shape))
    raise ValueError("meta must be bf16 or f32")


def activations(batch: int, cols: int, seed: int = 2) -> np.ndarray:
    """Token-major FP32 N(0, 1) activations [batch, cols]."""
    return normal(_sub(seed, 4), batch * cols).astype(np.float32).reshape(batch, cols)


def to_device(mat: dict, rows: int, cols: int, bits: int, group: int, device="cuda"):
    """Upload a synthetic matrix as an ops.PackedMatrix."""
    import torch

    from .ops import PackedMatrix
    w = torch.from_numpy(mat["weight"].view(np.int32)).to(device)
    if mat["scales"].dtype == np.uint16:
        s = torch.from_numpy(mat["scales"].view(np.int16)).to(device)
        b = torch.from_numpy(mat["biases"].view(np.int16)).to(device)
    else:
        s = torch.from_numpy(mat["scales"]).to(device)
        b = torch.from_numpy(mat["biases"]).to(device)
    return PackedMatrix(w, s, b, rows, cols, bits, group)
