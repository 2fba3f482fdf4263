"""The CPU oracle against the reference's known-answer tests and golden vectors.

Pins: src/gpu.rs:1636-1731 (Q4/Q8 matvec and embed KATs),
src/weights.rs:816-870 (nibble order), tests/batch_matrix.rs:357-381
(constant 0x76543210 row = 1792), src/gpu/metadata.rs:24-70 (exact BF16
packing), scripts/make_fixture.py:262-267 (BF16 rounding), src/chat.rs:383-390
(greedy ties), and tests/golden/matrices.npz produced by the reference's
own scalar oracle (scripts/make_fixture.py `mv`).
"""
import math
import pathlib
import struct

import numpy as np
import pytest

import oracle

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def f32_from_bits(u):
    return struct.unpack("<f", struct.pack("<I", u))[0]


def test_q4_little_nibbles_and_bias_kat():
    # src/gpu.rs:1637-1657
    w = np.array([0x76543210, 0xFEDCBA98], np.uint32)
    y, _ = oracle.matmul_f64(w, np.array([2, 0.5], np.float32), np.array([-1, -4], np.float32),
                             np.ones(8, np.float32), 2, 8, 4, 8)
    assert y.ravel().tolist() == [48.0, 14.0]


def test_q8_matvec_and_embedding_kat():
    # src/gpu.rs:1714-1730
    w = np.array([0xFF800100, 0x04030201], np.uint32)
    s = np.array([0.5, 2.0], np.float32)
    b = np.array([-1.0, -3.0], np.float32)
    y, _ = oracle.matmul_f64(w, s, b, np.array([1, 2, 3, 4], np.float32), 2, 4, 8, 4)
    assert y.ravel().tolist() == [693.0, 30.0]
    assert oracle.embed(w, s, b, 0, 4, 8, 4).tolist() == [-1.0, -0.5, 63.0, 126.5]


def test_nibble_order_decode_kat():
    # src/weights.rs:816-870: F16 scale 0x3800 = 0.5, bias 0xbc00 = -1.0
    w = np.array([0x76543210], np.uint32)
    got = oracle.embed(w, np.array([0.5], np.float32), np.array([-1.0], np.float32), 0, 8, 4, 8)
    assert got.tolist() == [-1.0, -0.5, 0.0, 0.5, 1.0, 1.5, 2.0, 2.5]


def test_constant_row_kat():
    # tests/batch_matrix.rs:357-381: all words 0x76543210, s=1, b=0, x=1 over 512 cols -> 1792
    w = np.full(4 * 512 // 8, 0x76543210, np.uint32)
    y, _ = oracle.matmul_f64(w, np.ones(32, np.float32), np.zeros(32, np.float32), np.ones(512, np.float32),
                             4, 512, 4, 64)
    assert y.ravel().tolist() == [1792.0] * 4


def test_bf16_metadata_expansion_is_high_half():
    # kernels/affine_bf16.metal:294-296; BF16 metadata decodes as bits << 16
    w = np.array([0x76543210], np.uint32)
    s = np.array([0x3F00], np.uint16)  # 0.5
    b = np.array([0xBF80], np.uint16)  # -1.0
    assert oracle.embed(w, s, b, 0, 8, 4, 8).tolist() == [-1.0, -0.5, 0.0, 0.5, 1.0, 1.5, 2.0, 2.5]


def test_pack_bf16_exact_patterns():
    # src/gpu/metadata.rs:24-45
    patterns = [0x00000000, 0x80000000, 0x3FC00000, 0xC0200000, 0x00010000, 0x80010000, 0x00800000,
                0x7F7F0000]
    packed = oracle.pack_bf16_exact(np.array([f32_from_bits(p) for p in patterns], np.float32))
    assert [int(v) << 16 for v in packed] == patterns
    for bad in [0.1, f32_from_bits(1), math.inf, -math.inf, math.nan]:
        assert oracle.pack_bf16_exact(np.array([1.0, bad, -0.0], np.float32)) is None


def test_bf16_round_to_nearest_even():
    # scripts/make_fixture.py:262-267
    def ref(value):
        bits = struct.unpack("<I", struct.pack("<f", value))[0]
        return (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    for v in [0.1, 1.0 / 3, -2.5e-3, 0.0078125, 65504.0, 1.00390625, 1.01171875, -0.0]:
        assert oracle.bf16_rne(v) == ref(struct.unpack("<f", struct.pack("<f", v))[0])


def test_greedy_ties_to_lowest_index_and_total_order():
    # src/chat.rs:383-390
    assert oracle.argmax_f32(np.array([1.0, 3.0, 3.0, 2.0], np.float32)) == 1
    assert oracle.argmax_f32(np.array([-0.0, 0.0], np.float32)) == 1  # total_cmp: -0 < +0
    assert oracle.argmax_f32(np.array([0.0, -0.0], np.float32)) == 0
    assert oracle.argmax_f32(np.array([-5.0, -1.0, -1.0], np.float32)) == 1


@pytest.mark.parametrize("idx", range(5))
def test_golden_matrices_from_reference_oracle(idx):
    """Dequantisation and FP64 matvec equal the reference's scalar Python oracle."""
    d = np.load(GOLDEN / "matrices.npz")
    rows, cols, bits, group = (int(v) for v in d[f"m{idx}_shape"])
    w, s, b = d[f"m{idx}_weight"], d[f"m{idx}_scales"], d[f"m{idx}_biases"]
    deq = d[f"m{idx}_dequant"]
    for r in (0, rows // 2, rows - 1):
        got = oracle.embed(w, s, b, r, cols, bits, group).astype(np.float64)
        # The reference dequantises in f64 (q*scale+bias); with BF16 metadata the
        # f32 product is exact, so only the final add may round.
        np.testing.assert_allclose(got, deq[r], rtol=0, atol=np.abs(deq[r]).max() * 2 ** -23)
        assert np.array_equal(got.astype(np.float32), deq[r].astype(np.float32))
    y, _ = oracle.matmul_f64(w, s, b, d[f"m{idx}_x"], rows, cols, bits, group)
    # Same f64 arithmetic in the same order as the reference's `mv`.
    np.testing.assert_array_equal(y.ravel(), d[f"m{idx}_y"])


def test_fp64_block_is_token_major():
    rng = np.random.default_rng(5)
    rows, cols = 7, 64
    w = rng.integers(0, 2 ** 32, size=rows * cols // 8, dtype=np.uint32)
    s = rng.uniform(0.001, 0.01, size=rows * cols // 32).astype(np.float32)
    b = rng.uniform(-0.05, 0.0, size=rows * cols // 32).astype(np.float32)
    x = rng.standard_normal(3 * cols).astype(np.float32)
    y3, _ = oracle.matmul_f64(w, s, b, x, rows, cols, 4, 32, batch=3)
    for t in range(3):
        y1, _ = oracle.matmul_f64(w, s, b, x[t * cols:(t + 1) * cols], rows, cols, 4, 32)
        np.testing.assert_array_equal(y3[t], y1[0])


def test_tolerance_helper_flags_nan_and_excess():
    r, _ = oracle.tolerance_ratio([1.0, float("nan")], [1.0, 1.0], [1.0, 1.0])
    assert r == math.inf
    r, i = oracle.tolerance_ratio([1.0, 1.0 + 4e-5], [1.0, 1.0], [1.0, 1.0])
    assert r > 1 and i == 1
