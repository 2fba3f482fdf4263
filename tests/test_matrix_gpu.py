"""CUDA parity of the packed-affine path against the FP64 oracle.

Restates the reference's real-GPU matrix tests (tests/quantized.rs,
tests/bf16_metadata.rs, tests/batch_matrix.rs, src/gpu.rs:1636-1731) through
libqmr's dispatch ABI, then checks the benchmark shapes.  Tolerances:
  * the reference's own per-test tolerances, and in addition
  * the north-star bound |err| <= 2e-5 * sum_j |w_ij x_j| against the FP64
    oracle (rtol 2e-5 of the absolute-product sum);
  * dequantisation (embed) bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle
import qmr
from qmr import Gpu, QmrError
from qmr import synth
from qmr.ops import PackedMatrix

from _util import (dev_bytes, hash_words, high_half, host_f32, quantized_seed, ref_biases, ref_scales, ref_x,
                   truncate_bf16, xorshift32)

pytestmark = pytest.mark.gpu

NS_RTOL = 2e-5  # north-star per-output bound, relative to sum |w x|


def f32_tensor(v, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device)


def assert_ns_bound(got, want, mag, what, slack_atol=0.0):
    ratio, i = oracle.tolerance_ratio(got, want, mag, rtol=NS_RTOL, atol=slack_atol)
    assert ratio <= 1.0, f"{what}: output {i} got {np.ravel(got)[i]} want {np.ravel(want)[i]} ratio {ratio}"


def encode_matvec(gpu, name, w, s, b, x, rows, cols, bits, group):
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    gpu.encode(name, [w, s, b, x, y], [rows, cols, bits, group], rows * 32, 128)
    gpu.finish()
    return y.cpu().numpy()


# ---------------------------------------------------------------------------
# src/gpu.rs known-answer tests
# ---------------------------------------------------------------------------

def test_affine_q4_little_nibbles_and_bias(cuda):
    gpu = Gpu()
    w = dev_bytes(np.array([0x76543210, 0xFEDCBA98], np.uint32))
    y = encode_matvec(gpu, "matvec_affine", w, f32_tensor([2.0, 0.5]), f32_tensor([-1.0, -4.0]),
                      f32_tensor(np.ones(8)), 2, 8, 4, 8)
    assert y.tolist() == [48.0, 14.0]


def test_q8_matvec_and_embedding(cuda):
    gpu = Gpu()
    q = dev_bytes(np.array([0xFF800100, 0x04030201], np.uint32))
    s, b = f32_tensor([0.5, 2.0]), f32_tensor([-1.0, -3.0])
    y = encode_matvec(gpu, "matvec_affine", q, s, b, f32_tensor([1, 2, 3, 4]), 2, 4, 8, 4)
    np.testing.assert_allclose(y, [693.0, 30.0], rtol=3e-5)
    emb = torch.zeros(4, dtype=torch.float32, device="cuda")
    gpu.encode("embed_affine", [q, s, b, emb], [0, 4, 8, 4], 4, 128)
    gpu.finish()
    assert emb.cpu().tolist() == [-1.0, -0.5, 63.0, 126.5]


def test_stream_offset_weights_fall_back_to_packed_alignment(cuda):
    """tests/batch_matrix.rs:357-381: W at a 4-byte offset, constant rows = 1792."""
    gpu = Gpu.new_with_variant(False, "stream")
    values = np.concatenate([[0], np.full(4 * 512 // 8, 0x76543210)]).astype(np.uint32)
    w = dev_bytes(values)
    y = torch.zeros(4, dtype=torch.float32, device="cuda")
    gpu.encode_offsets("matvec_affine", [w, f32_tensor(np.ones(32)), f32_tensor(np.zeros(32)),
                                         f32_tensor(np.ones(512)), y], [4, 0, 0, 0, 0], [4, 512, 4, 64], 128, 128)
    gpu.finish()
    assert y.cpu().tolist() == [1792.0] * 4


# ---------------------------------------------------------------------------
# tests/quantized.rs and tests/bf16_metadata.rs
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_specialized_q4_q8_match_scalar_across_groups_and_row_tails(cuda, bits, group):
    gpus = [Gpu.new_with_variant(False, "packed4"), Gpu.new_with_variant(False, "aligned"),
            Gpu.new_with_variant(False, "stream"), Gpu.new_with_reference(True)]
    pack = 32 // bits
    for cols in [group, 3 * group, 5120]:
        for rows in [1, 3, 7, 19, 20]:
            w = xorshift32(quantized_seed(bits, group, cols, rows), rows * cols // pack)
            scales = ref_scales(rows * cols // group)
            biases = ref_biases(rows * cols // group)
            x = ref_x(cols)
            want, mag = oracle.matmul_f64(w, scales, biases, x, rows, cols, bits, group)
            want32 = want.astype(np.float32).astype(np.float64)
            for gpu in gpus:
                got = encode_matvec(gpu, "matvec_affine", dev_bytes(w), f32_tensor(scales), f32_tensor(biases),
                                    f32_tensor(x), rows, cols, bits, group)
                tol = 2e-4 + np.abs(want32) * 2e-5  # tests/quantized.rs:73-77
                assert np.all(np.abs(got - want32) < tol), (gpu.kernel_mode(), bits, group, cols, rows)
                assert_ns_bound(got, want, mag, f"{gpu.kernel_mode()} Q{bits}/g{group} {rows}x{cols}")


@pytest.mark.parametrize("mode", ["aligned", "packed4", "stream"])
@pytest.mark.parametrize("bits", [4, 8])
def test_bf16_metadata_matches_scalar_for_packing_groups_shapes_and_embeddings(cuda, mode, bits):
    gpu = Gpu.new_with_variant(False, mode)
    pack = 32 // bits
    for group in [32, 64, 128]:
        for cols in [group, 3 * group, 5120]:
            for rows in [1, 3, 7, 19, 20]:
                weights = xorshift32(0x1478ABCF, rows * cols // pack)
                scales = truncate_bf16(ref_scales(rows * cols // group))
                biases = truncate_bf16(ref_biases(rows * cols // group))
                x = ref_x(cols)
                s16, b16 = high_half(scales), high_half(biases)
                want, mag = oracle.matmul_f64(weights, s16, b16, x, rows, cols, bits, group)
                wb, sb, bb = dev_bytes(weights), dev_bytes(s16), dev_bytes(b16)
                got = encode_matvec(gpu, "matvec_affine_bf16", wb, sb, bb, f32_tensor(x), rows, cols, bits, group)
                want32 = want.astype(np.float32).astype(np.float64)
                assert np.all(np.abs(got - want32) < 2e-4 + np.abs(want32) * 2e-5)
                assert_ns_bound(got, want, mag, f"{mode} bf16 Q{bits}/g{group} {rows}x{cols}")
                emb = torch.zeros(cols, dtype=torch.float32, device="cuda")
                gpu.encode("embed_affine_bf16", [wb, sb, bb, emb], [rows - 1, cols, bits, group], cols, 128)
                gpu.finish()
                exact = oracle.embed(weights, s16, b16, rows - 1, cols, bits, group)
                assert np.array_equal(emb.cpu().numpy().view(np.uint32), exact.view(np.uint32))


# ---------------------------------------------------------------------------
# tests/batch_matrix.rs
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_affine_blocks_share_weights_for_all_batches_formats_tails_and_offsets(cuda, bits, group):
    gpu = Gpu.new_with_variant(False, "aligned")
    pack = 32 // bits
    for rows, cols in [(1, group), (3, 3 * group), (7, 512), (20, 5120)]:
        weights = hash_words(rows * cols // pack, 0x9E3779B9, 0x1478ABCF)
        scales = np.array([(1 + i % 11) * 0.001953125 for i in range(rows * cols // group)], np.float32)
        biases = np.array([(i % 9) * 0.00390625 - 0.0625 for i in range(rows * cols // group)], np.float32)
        x = ref_x(4 * cols)
        want, mag = oracle.matmul_f64(weights, scales, biases, x, rows, cols, bits, group, batch=4)
        for bf16 in [False, True]:
            meta = (lambda v: high_half(v)) if bf16 else (lambda v: v)
            w = dev_bytes(weights, pad_front=4)
            s = dev_bytes(meta(scales), pad_front=4)
            b = dev_bytes(meta(biases), pad_front=4)
            xb = f32_tensor(np.concatenate([[99.0], x, [99.0]]))
            name = "matmul_affine_bf16" if bf16 else "matmul_affine"
            for batch in range(1, 5):
                yb = f32_tensor(np.full(batch * rows + 2, 12345.0))
                gpu.encode_offsets(name, [w, s, b, xb, yb], [4] * 5, [rows, cols, bits, group, batch],
                                   rows * 32, 128)
                gpu.finish()
                got = yb.cpu().numpy()
                assert got[0] == 12345.0 and got[batch * rows + 1] == 12345.0
                g = got[1:batch * rows + 1]
                wv = want[:batch].ravel()
                assert np.all(np.abs(g - wv) <= 4e-4 + np.abs(wv) * 3e-5), f"{name} B{batch} Q{bits} g{group}"
                assert_ns_bound(g, wv, mag[:batch].ravel(), f"{name} B{batch} Q{bits} g{group} {rows}x{cols}")


def test_offset_dispatch_rejects_bounds_and_unsafe_aliases_and_preserves_scalar_fallback(cuda):
    gpu = Gpu.new_with_reference(False)
    inp = f32_tensor(np.full(1028, 2.0))
    out = f32_tensor(np.zeros(1028))
    for offsets in [[], [0], [2, 0], [0, 2 ** 64 - 1], [4, 4]]:
        with pytest.raises(QmrError):
            gpu.encode_offsets("copy_f32", [inp, out], offsets, [1028], 1028, 128)
    with pytest.raises(QmrError):
        gpu.encode_offsets("copy_f32", [inp, inp], [0, 4], [32], 32, 128)
    w = dev_bytes(np.zeros(512 * 4 // 2, np.uint8))
    s = f32_tensor(np.ones(32))
    b = f32_tensor(np.ones(32))
    gpu.encode_offsets("matvec_affine", [w, s, b, inp, out], [0, 0, 0, 4, 4], [4, 512, 4, 64], 128, 128)
    s16 = dev_bytes(np.zeros(64, np.uint8))
    with pytest.raises(QmrError):
        gpu.encode_offsets("matvec_affine_bf16", [w, s16, s16, inp, out], [0, 0, 0, 4, 4], [4, 512, 4, 64], 128,
                           128)
    gpu.finish()
    got = out.cpu().numpy()
    assert got[0] == 0.0 and got[1027] == 0.0
    np.testing.assert_allclose(got[1:5], [1024.0] * 4, rtol=3e-5)


def test_matmul_output_may_not_overlap_inputs(cuda):
    gpu = Gpu()
    rows, cols = 4, 512
    big = torch.zeros(4096, dtype=torch.uint8, device="cuda")  # holds w and y
    s = f32_tensor(np.ones(32))
    x = f32_tensor(np.ones(cols))
    with pytest.raises(QmrError) as e:
        gpu.encode_offsets("matmul_affine", [big, s, s, x, big], [0, 0, 0, 0, 512], [rows, cols, 4, 64, 1],
                           rows * 32, 128)
    assert e.value.code == qmr._lib.QMR_EOVERLAP
    # Disjoint views of one allocation are fine.
    gpu.encode_offsets("matmul_affine", [big, s, s, x, big], [0, 0, 0, 0, 2048], [rows, cols, 4, 64, 1],
                       rows * 32, 128)
    gpu.finish()


def test_aligned_q4_blocks_match_independent_oracle_and_single_token_path(cuda):
    gpu = Gpu.new_with_variant(False, "aligned")
    legacy_outputs = []
    for matmul in ["legacy", "shared", "mlp-r2"]:
        gpu.set_block_kernel_mode(qmr.BlockKernelMode(matmul, False))
        case = 0
        for cols in [512, 5120, 17408]:
            rows = 20
            weights = hash_words(rows * cols // 8, 0x1478ABCF, 0x9E3779B9)
            scales = np.array([(1 + i % 11) * 0.001953125 for i in range(rows * cols // 64)], np.float32)
            biases = np.array([(i % 9) * 0.00390625 - 0.0625 for i in range(rows * cols // 64)], np.float32)
            x = ref_x(4 * cols)
            want, mag = oracle.matmul_f64(weights, scales, biases, x, rows, cols, 4, 64, batch=4)
            wb = dev_bytes(weights)
            xb = f32_tensor(x)
            for bf16 in [False, True]:
                up = (lambda v: dev_bytes(high_half(v))) if bf16 else f32_tensor
                sb, bb = up(scales), up(biases)
                for batch in range(1, 5):
                    y = torch.zeros(rows * batch, dtype=torch.float32, device="cuda")
                    seq = torch.zeros(rows * batch, dtype=torch.float32, device="cuda")
                    mm = "matmul_affine_bf16" if bf16 else "matmul_affine"
                    mv = "matvec_affine_bf16" if bf16 else "matvec_affine"
                    gpu.encode(mm, [wb, sb, bb, xb, y], [rows, cols, 4, 64, batch], rows * 32, 128)
                    for bi in range(batch):
                        gpu.encode_offsets(mv, [wb, sb, bb, xb, seq], [0, 0, 0, bi * cols * 4, bi * rows * 4],
                                           [rows, cols, 4, 64], rows * 32, 128)
                    gpu.finish()
                    actual = y.cpu().numpy()
                    wv = want[:batch].ravel()
                    assert np.all(np.abs(actual - wv) <= 4e-4 + np.abs(wv) * 3e-5)
                    assert_ns_bound(actual, wv, mag[:batch].ravel(), f"{matmul} B{batch} cols{cols} bf16={bf16}")
                    if matmul != "legacy":
                        assert np.array_equal(actual.view(np.uint32), legacy_outputs[case].view(np.uint32)), \
                            f"{matmul} schedule must preserve every bit B{batch} cols{cols} BF16={bf16}"
                    else:
                        legacy_outputs.append(actual.copy())
                    case += 1
                    # This build's block equals B single-token GEMVs bit for bit.
                    assert np.array_equal(actual.view(np.uint32), seq.cpu().numpy().view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(17408, 5120), (5120, 17408)])
def test_selective_mlp_r2_real_shapes_match_legacy_bits_and_fp64_with_guards(cuda, rows, cols):
    gpu = Gpu.new_with_variant(False, "aligned")
    weights = hash_words(rows * cols // 8, 0x1478ABCF, 0x9E3779B9)
    scales = np.array([(1 + i % 11) * 0.001953125 for i in range(rows * cols // 64)], np.float32)
    biases = np.array([(i % 9) * 0.00390625 - 0.0625 for i in range(rows * cols // 64)], np.float32)
    x = ref_x(3 * cols)
    guard = dict(pad_front=16, pad_back=16, fill=0xA5)
    wb = dev_bytes(weights, **guard)
    sb = dev_bytes(high_half(scales), **guard)
    bb = dev_bytes(high_half(biases), **guard)
    xb = dev_bytes(x, **guard)
    outs = []
    for matmul in ["legacy", "mlp-r2"]:
        gpu.set_block_kernel_mode(qmr.BlockKernelMode(matmul, True))
        y = f32_tensor(np.full(rows * 3 + 8, 12345.0))
        gpu.encode_offsets("matmul_affine_bf16", [wb, sb, bb, xb, y], [16] * 4 + [16],
                           [rows, cols, 4, 64, 3], rows * 32, 128)
        gpu.finish()
        outs.append(y.cpu().numpy())
    for o in outs:
        assert np.all(o[:4] == 12345.0) and np.all(o[rows * 3 + 4:] == 12345.0)
        assert np.all(np.isfinite(o[4:rows * 3 + 4]))
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    # Every row of every RHS against FP64: the reference's tolerance and the north-star bound.
    want, mag = oracle.matmul_f64(weights, high_half(scales), high_half(biases), x, rows, cols, 4, 64, batch=3)
    got = outs[0][4:rows * 3 + 4].reshape(3, rows).astype(np.float64)
    assert np.all(np.abs(got - want) <= 4e-4 + np.abs(want) * 3e-5), f"R2 {rows}x{cols}"
    assert_ns_bound(got, want, mag, f"R2 {rows}x{cols}")
    for buf in [wb, sb, bb, xb]:
        raw = buf.cpu().numpy()
        assert np.all(raw[:16] == 0xA5) and np.all(raw[-16:] == 0xA5)


# ---------------------------------------------------------------------------
# Benchmark shapes (configs 0-3) with the benchmark distributions
# ---------------------------------------------------------------------------

def check_all_rows(mat, m, x, y, batch, what):
    """Compare every output row of y [batch, rows] with the FP64 oracle."""
    want, mag = oracle.matmul_f64(mat["weight"], mat["scales"], mat["biases"], x, m.rows, m.cols, m.bits, m.group,
                                  batch=batch)
    assert_ns_bound(y, want, mag, what)
    return want, mag


@pytest.mark.parametrize("bits", [4, 8])
def test_config_shapes_b1_b3_parity_and_block_equals_gemv(cuda, bits):
    rows, cols = 17408, 5120
    mat = synth.affine_matrix(rows, cols, bits, 64, seed=11 + bits)
    m = synth.to_device(mat, rows, cols, bits, 64)
    x = synth.activations(3, cols, seed=7)
    xd = f32_tensor(x.ravel())
    y3 = torch.empty(3 * rows, dtype=torch.float32, device="cuda")
    qmr.matmul_affine(m, xd, y3, 3)
    y1 = torch.empty((3, rows), dtype=torch.float32, device="cuda")
    for b in range(3):
        qmr.matvec_affine(m, xd[b * cols:(b + 1) * cols], y1[b])
    torch.cuda.synchronize()
    y3h = y3.cpu().numpy().reshape(3, rows)
    y1h = y1.cpu().numpy()
    assert np.array_equal(y3h.view(np.uint32), y1h.view(np.uint32))
    check_all_rows(mat, m, x, y3h, 3, f"Q{bits} B3 {rows}x{cols}")
    # The B1 GEMV (config 0 for Q4) on its own, every row.
    check_all_rows(mat, m, x[:1], y1h[:1], 1, f"Q{bits} B1 {rows}x{cols}")


def test_gateup_swiglu_matches_oracle_and_separate_projections(cuda):
    rows, cols = 17408, 5120
    g = synth.affine_matrix(rows, cols, 4, 64, seed=21)
    u = synth.affine_matrix(rows, cols, 4, 64, seed=22)
    gm, um = synth.to_device(g, rows, cols, 4, 64), synth.to_device(u, rows, cols, 4, 64)
    for batch in (1, 3):
        x = synth.activations(batch, cols, seed=30 + batch)
        xd = f32_tensor(x)
        act = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
        qmr.gateup_swiglu(gm, um, xd, act, batch)
        gy = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
        uy = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
        qmr.matmul_affine(gm, xd, gy, batch)
        qmr.matmul_affine(um, xd, uy, batch)
        torch.cuda.synchronize()
        a = act.cpu().numpy().reshape(batch, rows)
        gh = gy.cpu().numpy().astype(np.float64)
        uh = uy.cpu().numpy().astype(np.float64)
        ref = (gh / (1.0 + np.exp(-gh)) * uh).reshape(batch, rows)
        # Every row against FP64: first-order error scale |u|*1.1*sum|g_j| + |silu(g)|*sum|u_j| at the
        # per-product bound, plus the f32 silu/product rounding (a few ulps of the result).
        want, mag = oracle.swiglu_f64(g["weight"], g["scales"], g["biases"], u["weight"], u["scales"], u["biases"],
                                      x, rows, cols, 4, 64, batch)
        assert_ns_bound(a, want, mag + np.abs(want) * 0.05, f"swiglu B{batch}")
        # The fused pair against the two plain projections (whose split of the columns may differ):
        # both sides carry the bound once.
        assert_ns_bound(a, ref, 2 * mag + np.abs(ref) * 0.1, f"swiglu vs separate B{batch}")
        if batch == 3:
            # The fused pair is B-independent too: RHS 1 of the block equals a single-RHS call.
            a1 = torch.empty(rows, dtype=torch.float32, device="cuda")
            qmr.gateup_swiglu(gm, um, xd.reshape(-1)[cols:2 * cols], a1, 1)
            torch.cuda.synchronize()
            assert np.array_equal(a[1].view(np.uint32), a1.cpu().numpy().view(np.uint32))


@pytest.mark.parametrize("batch", [1, 3])
def test_mlp_down_of_swiglu_every_row(cuda, batch):
    """Config 2 end to end: y = down(silu(gate x) * (up x)) through the fused
    gate/up kernel and the 5120x17408 down projection; every activation row
    against FP64 swiglu, every output row against FP64 down of the device
    activations (the down stage's own bound)."""
    H, F = 5120, 17408
    g = synth.affine_matrix(F, H, 4, 64, seed=81)
    u = synth.affine_matrix(F, H, 4, 64, seed=82)
    d = synth.affine_matrix(H, F, 4, 64, seed=83)
    gm, um, dm = (synth.to_device(t, r, c, 4, 64) for t, r, c in ((g, F, H), (u, F, H), (d, H, F)))
    x = synth.activations(batch, H, seed=84 + batch)
    act = torch.empty(batch * F, dtype=torch.float32, device="cuda")
    y = torch.empty(batch * H, dtype=torch.float32, device="cuda")
    qmr.gateup_swiglu(gm, um, f32_tensor(x), act, batch)
    qmr.matmul_affine(dm, act, y, batch)
    torch.cuda.synchronize()
    a = act.cpu().numpy().reshape(batch, F)
    want_a, mag_a = oracle.swiglu_f64(g["weight"], g["scales"], g["biases"], u["weight"], u["scales"], u["biases"],
                                      x, F, H, 4, 64, batch)
    assert_ns_bound(a, want_a, mag_a + np.abs(want_a) * 0.05, f"MLP swiglu B{batch}")
    check_all_rows(d, dm, a, y.cpu().numpy().reshape(batch, H), batch, f"MLP down B{batch}")


def test_head_argmax_matches_logits_and_oracle(cuda):
    rows, cols = 152064, 5120
    mat = synth.affine_matrix(rows, cols, 4, 64, seed=41)
    m = synth.to_device(mat, rows, cols, 4, 64)
    for batch in (1, 3):
        x = synth.activations(batch, cols, seed=50 + batch)
        xd = f32_tensor(x)
        logits = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
        idx = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
        keys = torch.zeros(batch, dtype=torch.int64, device="cuda")
        qmr.head_argmax(m, xd, logits, idx, batch, best_key=keys)
        plain = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
        qmr.matmul_affine(m, xd, plain, batch)
        torch.cuda.synchronize()
        lg = logits.cpu().numpy().reshape(batch, rows)
        assert np.array_equal(lg.view(np.uint32), plain.cpu().numpy().reshape(batch, rows).view(np.uint32))
        got = idx.cpu().numpy()
        for b in range(batch):
            assert got[b] == oracle.argmax_f32(lg[b])
            k = int(keys.cpu().numpy()[b]) & 0xFFFFFFFFFFFFFFFF
            i, v = qmr.ops.decode_key(k)
            assert i == got[b] and v == lg[b, got[b]]
            # The FP64 winner agrees when the margin exceeds the error bound.
            top = np.argsort(lg[b])[-8:]
            want, mag = oracle.matmul_f64(mat["weight"], mat["scales"], mat["biases"], x[b], rows, cols, 4, 64,
                                          row0=0, nrows=rows)
            w = want[0]
            best = oracle.argmax_f64(w)
            second = np.partition(w, -2)[-2]
            if w[best] - second > 4 * NS_RTOL * mag[0, best]:
                assert got[b] == best
            assert best in top
        check_all_rows(mat, m, x, lg, batch, f"head B{batch}")


def test_head_argmax_ties_go_to_lowest_index(cuda):
    rows, cols = 4096, 512
    mat = synth.affine_matrix(rows, cols, 4, 64, seed=61)
    # Rows 100 and 3000 identical and dominant: weights all 15, scale large.
    for r in (3000, 100):
        mat["weight"][r] = 0xFFFFFFFF
        mat["scales"][r] = synth.bf16_rne(np.float32(0.5))
        mat["biases"][r] = 0
    m = synth.to_device(mat, rows, cols, 4, 64)
    x = np.abs(synth.activations(1, cols, seed=62)) + 0.1
    logits = torch.empty(rows, dtype=torch.float32, device="cuda")
    idx = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    qmr.head_argmax(m, f32_tensor(x), logits, idx, 1, row_base=1000)
    torch.cuda.synchronize()
    lg = logits.cpu().numpy()
    assert lg[100] == lg[3000] and lg.argmax() == 100
    assert int(idx.cpu()[0]) == 1100


def test_golden_matrices_from_reference_oracle_on_device(cuda):
    """The reference's own scalar oracle outputs (tests/golden/matrices.npz)."""
    import pathlib
    d = np.load(pathlib.Path(__file__).resolve().parent / "golden" / "matrices.npz")
    gpu = Gpu()
    for idx in range(len(d["names"])):
        rows, cols, bits, group = (int(v) for v in d[f"m{idx}_shape"])
        w, s, b = d[f"m{idx}_weight"], d[f"m{idx}_scales"], d[f"m{idx}_biases"]
        x = d[f"m{idx}_x"]
        wb, sb, bb = dev_bytes(w), dev_bytes(s), dev_bytes(b)
        got = encode_matvec(gpu, "matvec_affine_bf16", wb, sb, bb, f32_tensor(x), rows, cols, bits, group)
        _, mag = oracle.matmul_f64(w, s, b, x, rows, cols, bits, group)
        assert_ns_bound(got, d[f"m{idx}_y"], mag[0], f"golden {d['names'][idx]}")
        for r in (0, rows - 1):
            emb = torch.zeros(cols, dtype=torch.float32, device="cuda")
            gpu.encode("embed_affine_bf16", [wb, sb, bb, emb], [r, cols, bits, group], cols, 128)
            gpu.finish()
            assert np.array_equal(emb.cpu().numpy(), d[f"m{idx}_dequant"][r].astype(np.float32))


def test_extreme_activation_ranges_stay_accurate(cuda):
    """Per-chunk exponent selection keeps tiny and huge activations exact to f32."""
    rows, cols = 64, 1024
    mat = synth.affine_matrix(rows, cols, 4, 64, seed=71)
    m = synth.to_device(mat, rows, cols, 4, 64)
    base = synth.activations(1, cols, seed=72)[0]
    for scale in (1e-30, 1e-10, 1.0, 1e10, 1e30):
        x = (base * np.float32(scale)).astype(np.float32)
        x[5] = 0.0
        y = torch.empty(rows, dtype=torch.float32, device="cuda")
        qmr.matvec_affine(m, f32_tensor(x), y)
        torch.cuda.synchronize()
        want, mag = oracle.matmul_f64(mat["weight"], mat["scales"], mat["biases"], x, rows, cols, 4, 64)
        assert_ns_bound(y.cpu().numpy(), want[0], mag[0], f"scale {scale}")
    # Mixed magnitudes inside one chunk.
    x = base.copy()
    x[::7] *= np.float32(1e20)
    x[1::7] *= np.float32(1e-20)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    qmr.matvec_affine(m, f32_tensor(x), y)
    torch.cuda.synchronize()
    want, mag = oracle.matmul_f64(mat["weight"], mat["scales"], mat["biases"], x, rows, cols, 4, 64)
    assert_ns_bound(y.cpu().numpy(), want[0], mag[0], "mixed magnitudes")


def test_prepared_activations_feed_several_matrices_bit_exactly(cuda):
    rows, cols = 4096, 5120
    mats = [synth.affine_matrix(rows, cols, 4, 64, seed=80 + i) for i in range(3)]
    dm = [synth.to_device(m, rows, cols, 4, 64) for m in mats]
    for batch in (1, 3):
        x = f32_tensor(synth.activations(batch, cols, seed=90 + batch).ravel())
        prepared = qmr.ops.alloc_prepared(4, cols, batch)
        qmr.ops.prepare_activations(x, cols, 4, batch, prepared)
        for m in dm:
            a = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
            b = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
            qmr.ops.matmul_prepared(m, prepared, a, batch)
            qmr.matmul_affine(m, x, b, batch)
            torch.cuda.synchronize()
            assert np.array_equal(a.cpu().numpy().view(np.uint32), b.cpu().numpy().view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(1024, 5120), (512, 17408)])
def test_in_kernel_image_equals_the_prep_kernel_image(cuda, rows, cols):
    """Device-resident x: every streaming CTA builds its slice of the
    activation image in its prologue (one CTA per row slice at 5120 columns,
    4-CTA clusters at 17408).  Pinned host x and the prepared-activation
    API: the prep kernel writes the image once and the CTAs copy it.  Same
    image bits, same kernel and plan: the outputs agree bit for bit, for
    the plain product and for the fused gate/up SwiGLU."""
    g = synth.to_device(synth.affine_matrix(rows, cols, 4, 64, seed=61), rows, cols, 4, 64)
    u = synth.to_device(synth.affine_matrix(rows, cols, 4, 64, seed=62), rows, cols, 4, 64)
    for batch in (1, 4):
        xs = synth.activations(batch, cols, seed=63 + batch).ravel()
        xd = f32_tensor(xs)
        xh = torch.from_numpy(xs.copy()).pin_memory()
        outs = []
        for x in (xd, xh):
            y = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
            a = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
            qmr.matmul_affine(g, x, y, batch)
            qmr.ops.gateup_swiglu(g, u, x, a, batch)
            torch.cuda.synchronize()
            outs.append((y.cpu().numpy().view(np.uint32), a.cpu().numpy().view(np.uint32)))
        prepared = qmr.ops.alloc_prepared(4, cols, batch)
        qmr.ops.prepare_activations(xd, cols, 4, batch, prepared)
        yp = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
        qmr.ops.matmul_prepared(g, prepared, yp, batch)
        torch.cuda.synchronize()
        assert np.array_equal(outs[0][0], outs[1][0]), batch
        assert np.array_equal(outs[0][1], outs[1][1]), batch
        assert np.array_equal(outs[0][0], yp.cpu().numpy().view(np.uint32)), batch


def test_typed_wrappers_reject_undersized_views_before_launch(cuda):
    rows, cols = 64, 512
    m = synth.to_device(synth.affine_matrix(rows, cols, 4, 64, seed=3), rows, cols, 4, 64)
    x = torch.zeros((3, cols), dtype=torch.float32, device="cuda")
    y = torch.zeros(3 * rows, dtype=torch.float32, device="cuda")
    with pytest.raises(QmrError):
        qmr.matvec_affine(m, x[5:], y)  # empty view
    with pytest.raises(QmrError):
        qmr.matmul_affine(m, x[:1], y, 3)
    with pytest.raises(QmrError):
        qmr.matmul_affine(m, x, y[:rows], 3)
    with pytest.raises(QmrError):
        qmr.embed_affine(m, rows, y)


@pytest.mark.parametrize("meta", ["f32", "bf16"])
def test_fresh_matrices_keep_blocks_equal_to_gemv(cuda, meta):
    """Freshly uploaded matrices (cold L2, metadata arriving late) still give a
    B4 block equal to the single-RHS call and within the oracle bound: every
    metadata copy is complete and visible before any lane reads it."""
    rows, cols = 17408, 5120
    for it in range(6):
        mat = synth.affine_matrix(rows, cols, 4, 64, seed=900 + it, meta=meta)
        m = synth.to_device(mat, rows, cols, 4, 64)
        x_np = synth.activations(4, cols, seed=950 + it)
        x = f32_tensor(x_np.ravel())
        y4 = torch.full((4 * rows,), float("nan"), dtype=torch.float32, device="cuda")
        qmr.matmul_affine(m, x, y4, 4)
        y1 = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        qmr.matvec_affine(m, x[2 * cols:3 * cols], y1)
        torch.cuda.synchronize()
        got = y4.cpu().numpy().reshape(4, rows)
        assert np.array_equal(got[2].view(np.uint32), y1.cpu().numpy().view(np.uint32)), f"iteration {it}"
        check_all_rows(mat, m, x_np, got, 4, f"fresh {meta} it {it}")
        del m


@pytest.mark.parametrize("bits,meta", [(4, "bf16"), (4, "f32"), (8, "bf16")])
def test_all_streaming_paths_meet_the_bound(cuda, bits, meta):
    """The tensor-core kernel, the FP32 TMA tile kernel (split-K, partial
    slices and tiles) and the FP32 register-streaming kernel all meet the
    oracle bound on every shape, and
    within each path a B-wide block equals B single-RHS calls bit for bit.
    Also checks that no bounded device wait ran out."""
    # 40008 x 5120 has enough (tile, window) units for the 12-warp plan (Q4).
    shapes = [(17408, 5120), (5120, 17408), (4, 512), (37, 2176), (1000, 3072), (300, 1024), (40008, 5120)]
    try:
        for rows, cols in shapes:
            mat = synth.affine_matrix(rows, cols, bits, 64, seed=rows + cols, meta=meta)
            m = synth.to_device(mat, rows, cols, bits, 64)
            x_np = synth.activations(4, cols, seed=rows)
            x = f32_tensor(x_np.ravel())
            want, mag = oracle.matmul_f64(mat["weight"], mat["scales"], mat["biases"], x_np, rows, cols, bits, 64,
                                          batch=4)
            for path in ("mma", "tma", "registers"):
                qmr.ops.set_stream_path(path)
                y4 = torch.full((4 * rows,), float("nan"), dtype=torch.float32, device="cuda")
                qmr.matmul_affine(m, x, y4, 4)
                y1 = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
                qmr.matvec_affine(m, x[2 * cols:3 * cols], y1)
                torch.cuda.synchronize()
                got = y4.cpu().numpy().reshape(4, rows)
                assert np.array_equal(got[2].view(np.uint32), y1.cpu().numpy().view(np.uint32)), (path, rows, cols)
                assert_ns_bound(got, want, mag, f"{path} {rows}x{cols}")
            if rows >= 1000 and bits == 4 and meta == "bf16":
                upm = synth.affine_matrix(rows, cols, bits, 64, seed=7, meta=meta)
                up = synth.to_device(upm, rows, cols, bits, 64)
                x3 = x_np[:3]
                want_a, amag = oracle.swiglu_f64(mat["weight"], mat["scales"], mat["biases"], upm["weight"],
                                                 upm["scales"], upm["biases"], x3, rows, cols, bits, 64, 3)
                for path in ("mma", "tma", "registers"):
                    qmr.ops.set_stream_path(path)
                    act = torch.empty(3 * rows, dtype=torch.float32, device="cuda")
                    qmr.gateup_swiglu(m, up, f32_tensor(x3.ravel()), act, 3)
                    lg = torch.empty(3 * rows, dtype=torch.float32, device="cuda")
                    idx = torch.empty(3, dtype=torch.int32, device="cuda")
                    qmr.head_argmax(m, f32_tensor(x3.ravel()), lg, idx, 3)
                    torch.cuda.synchronize()
                    lgh = lg.cpu().numpy().reshape(3, rows)
                    assert [oracle.argmax_f32(lgh[b]) for b in range(3)] == idx.cpu().numpy().tolist()
                    a = act.cpu().numpy().reshape(3, rows)
                    assert_ns_bound(a, want_a, amag + np.abs(want_a) * 0.1, f"{path} swiglu {rows}x{cols}")
        assert qmr.ops.device_error() == 0
    finally:
        qmr.ops.set_stream_path("mma")


def test_pinned_host_activations_give_the_same_bits(cuda):
    """x may be a pinned host tensor (read by the kernels over the host link):
    the same bits as the device copy for the block, the GEMV, the fused
    gate/up pair and the head."""
    rows, cols = 4096, 5120
    mat = synth.affine_matrix(rows, cols, 4, 64, seed=61)
    m = synth.to_device(mat, rows, cols, 4, 64)
    x_np = synth.activations(3, cols, seed=62)
    xd = f32_tensor(x_np.ravel())
    xh = torch.from_numpy(np.ascontiguousarray(x_np.ravel(), np.float32)).pin_memory()
    outs = {}
    for name, x in (("dev", xd), ("host", xh)):
        y3 = torch.empty(3 * rows, dtype=torch.float32, device="cuda")
        qmr.matmul_affine(m, x, y3, 3)
        y1 = torch.empty(rows, dtype=torch.float32, device="cuda")
        qmr.matvec_affine(m, x[:cols], y1)
        act = torch.empty(3 * rows, dtype=torch.float32, device="cuda")
        qmr.gateup_swiglu(m, m, x, act, 3)
        lg = torch.empty(3 * rows, dtype=torch.float32, device="cuda")
        idx = torch.empty(3, dtype=torch.int32, device="cuda")
        qmr.head_argmax(m, x, lg, idx, 3)
        torch.cuda.synchronize()
        outs[name] = [t.cpu().numpy() for t in (y3, y1, act, lg, idx)]
    for a, b in zip(outs["dev"], outs["host"]):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # copy_f32 into pinned host memory (and device to device) moves the bits unchanged.
    yh = torch.empty(3 * rows, dtype=torch.float32).pin_memory()
    yd = torch.empty(3 * rows, dtype=torch.float32, device="cuda")
    qmr.copy_f32(y3, yh, 3 * rows)
    qmr.copy_f32(y3, yd, 3 * rows - 1)
    torch.cuda.synchronize()
    assert np.array_equal(yh.numpy().view(np.uint32), outs["host"][0].view(np.uint32))
    assert np.array_equal(yd.cpu().numpy()[:-1].view(np.uint32), outs["host"][0][:-1].view(np.uint32))
    pageable = torch.from_numpy(np.ascontiguousarray(x_np.ravel(), np.float32))
    with pytest.raises(qmr.QmrError):
        qmr.matmul_affine(m, pageable, torch.empty(3 * rows, dtype=torch.float32, device="cuda"), 3)
