"""Helpers shared by the GPU tests: reference input generators, uploads, guards."""
from __future__ import annotations

import functools

import numpy as np


@functools.lru_cache(maxsize=64)
def _xorshift32(seed: int, n: int) -> bytes:
    """tests/quantized.rs:17-29 word stream (seed ^= seed<<13; >>17; <<5)."""
    out = np.empty(n, dtype=np.uint32)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        out[i] = s
    return out.tobytes()


def xorshift32(seed: int, n: int) -> np.ndarray:
    return np.frombuffer(_xorshift32(seed, n), dtype=np.uint32).copy()


def rotl32(v: int, r: int) -> int:
    v &= 0xFFFFFFFF
    return ((v << r) | (v >> (32 - r))) & 0xFFFFFFFF


def quantized_seed(bits, group, cols, rows):
    """Seed of tests/quantized.rs:22-27."""
    return 0x84213957 ^ bits ^ rotl32(group, 7) ^ rotl32(cols, 13) ^ rotl32(rows, 19)


def ref_scales(n):
    return np.array([0.001 * (1 + (i % 11)) for i in range(n)], dtype=np.float32)


def ref_biases(n):
    return np.array([-0.07 + (i % 9) * 0.003 for i in range(n)], dtype=np.float32)


def ref_x(n):
    i = np.arange(n)
    return (((i * 13 % 101).astype(np.float32) - 50.0) / 50.0).astype(np.float32)


def hash_words(n, mul, add):
    """(i * mul + add) mod 2^32 (tests/batch_matrix.rs:24, 252)."""
    i = np.arange(n, dtype=np.uint64)
    return ((i * np.uint64(mul) + np.uint64(add)) & np.uint64(0xFFFFFFFF)).astype(np.uint32)


def high_half(v):
    return (np.ascontiguousarray(v, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def truncate_bf16(v):
    return (np.ascontiguousarray(v, np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)


def dev_bytes(arr, device="cuda", pad_front=0, pad_back=0, fill=0):
    """Upload raw bytes of arr into a uint8 CUDA tensor with optional guard bytes."""
    import torch
    raw = np.ascontiguousarray(arr).view(np.uint8).ravel()
    buf = np.full(pad_front + raw.size + pad_back, fill, dtype=np.uint8)
    buf[pad_front:pad_front + raw.size] = raw
    return torch.from_numpy(buf).to(device)


def host_f32(t, offset_bytes=0, n=None):
    b = t.cpu().numpy().view(np.uint8)
    v = b[offset_bytes:].view(np.float32) if (b.size - offset_bytes) % 4 == 0 else \
        b[offset_bytes:offset_bytes + ((b.size - offset_bytes) // 4) * 4].view(np.float32)
    return v if n is None else v[:n]
