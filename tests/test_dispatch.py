"""Host dispatch rules through libqmr's C ABI (no GPU): the reference's own
GPU-free unit tests of src/gpu.rs:1298-1634 and src/gpu/metadata.rs, restated."""
import ctypes
import pathlib
import re

import numpy as np
import pytest

import qmr
from qmr import BlockKernelMode, QmrError, dispatch_layout, select

ROOT = pathlib.Path(__file__).resolve().parents[1]
U32_MAX = 0xFFFFFFFF


def test_library_exports_every_header_symbol():
    header = (ROOT / "include" / "qmr.h").read_text()
    names = set(re.findall(r"^(?:int|void|uint64_t|const char \*)\s*(qmr_\w+)\(", header, flags=re.M))
    assert len(names) >= 49
    lib = qmr.lib()
    for n in sorted(names):
        assert hasattr(lib, n), n
    assert lib.qmr_abi_version() == 1


def test_block_kernel_device_defaults_are_limited_to_measured_m5_pro():
    for device, expected in [("Apple M5 Pro", "mlp-r2"), ("Apple M5", "legacy"), ("Apple M5 Max", "legacy"),
                             ("Apple M1", "legacy"), ("Apple M1 Pro", "legacy"), ("Apple M4 Pro", "legacy"),
                             ("Apple M5 Pro Max", "legacy"), ("apple m5 pro", "legacy"),
                             ("Apple M5 Pro ", "legacy"), ("", "legacy"), ("NVIDIA B200", "legacy")]:
        assert BlockKernelMode.parse_for_device(device, None, None) == BlockKernelMode(expected, True), device
    assert BlockKernelMode().matmul == "legacy"


def test_block_kernel_explicit_modes_override_device_defaults():
    for device in ["Apple M5 Pro", "Apple M1"]:
        for matmul in ["legacy", "shared", "mlp-r2"]:
            for delta, batched in [("sequential", False), ("batched", True)]:
                assert BlockKernelMode.parse_for_device(device, matmul, delta) == BlockKernelMode(matmul, batched)
    assert BlockKernelMode.parse_for_device("Apple M5 Pro", None, "sequential") == BlockKernelMode("mlp-r2", False)


def test_block_kernel_device_defaults_reject_invalid_overrides():
    for device in ["Apple M5 Pro", "Apple M1"]:
        for invalid in ["", "auto", "LEGACY", "legacy ", "mlp_r2", "MLP-R2"]:
            with pytest.raises(QmrError):
                BlockKernelMode.parse_for_device(device, invalid, None)
            with pytest.raises(QmrError):
                BlockKernelMode.parse_for_device(device, None, invalid)


def test_block_kernel_modes_are_independent_and_reject_unknown_values():
    assert BlockKernelMode.parse("legacy", "batched") == BlockKernelMode()
    for value in ["legacy", "shared", "mlp-r2"]:
        for delta, batched in [("sequential", False), ("batched", True)]:
            assert BlockKernelMode.parse(value, delta) == BlockKernelMode(value, batched)
    for invalid in ["", "auto", "SHARED", "shared ", "mlp_r2", "MLP-R2"]:
        with pytest.raises(QmrError):
            BlockKernelMode.parse(invalid, "sequential")
        with pytest.raises(QmrError):
            BlockKernelMode.parse("legacy", invalid)


def test_shared_matmul_selection_changes_only_supported_aligned_batches():
    for batch in range(1, 5):
        for name in ["matmul_affine", "matmul_affine_bf16"]:
            params = [20, 5120, 4, 64, batch]
            legacy = select(name, params, True, "legacy")
            shared = select(name, params, True, "shared")
            assert "_shared" not in legacy
            assert ("_shared" in shared) == (batch in (2, 3))
            if batch in (1, 4):
                assert legacy == shared
            for fallback, aligned in [(params, False), ([19, 5120, 4, 64, batch], True),
                                      ([20, 5120, 8, 64, batch], True), ([20, 5120, 4, 32, batch], True)]:
                assert select(name, fallback, aligned, "legacy") == select(name, fallback, aligned, "shared")


def test_mlp_r2_selection_is_limited_to_measured_shapes_and_format():
    for rows, cols in [(17408, 5120), (5120, 17408), (248320, 5120), (20, 5120), (17408, 512), (17412, 5120)]:
        for batch in range(1, 5):
            for name in ["matmul_affine", "matmul_affine_bf16"]:
                for bits, group in [(4, 32), (4, 64), (4, 128), (8, 64)]:
                    for aligned in [False, True]:
                        params = [rows, cols, bits, group, batch]
                        want_r2 = (aligned and name == "matmul_affine_bf16" and batch == 3 and bits == 4
                                   and group == 64 and (rows, cols) in [(17408, 5120), (5120, 17408)])
                        got = select(name, params, aligned, "mlp-r2")
                        if want_r2:
                            assert got == "matmul_q4_g64_b3_mlp_r2_aligned_bf16"
                        else:
                            assert got == select(name, params, aligned, "legacy"), (name, params, aligned)
            dense = [rows, cols, batch]
            assert select("matmul_f16", dense, True, "mlp-r2") == select("matmul_f16", dense, True, "legacy")


def test_buffer_views_reject_misalignment_bounds_and_integer_wraparound():
    qmr.checked_buffer_range(4, 12, 16)
    qmr.checked_buffer_range(0, 16, 16)
    for args in [(4, 16, 16), (2, 12, 16), (2 ** 64 - 4, 8, 2 ** 64 - 1)]:
        with pytest.raises(QmrError):
            qmr.checked_buffer_range(*args)


def test_block_specialization_preserves_alignment_and_all_batch_sizes():
    for batch in range(1, 5):
        p = [20, 5120, 4, 64, batch]
        assert select("matmul_affine", p, True).endswith("_aligned")
        assert select("matmul_affine_bf16", p, True).endswith("_aligned_bf16")
        assert not select("matmul_affine", p, False).endswith("_aligned")
        assert not select("matmul_affine", [19, 5120, 4, 64, batch], True).endswith("_aligned")
        assert not select("matmul_affine", [20, 5120, 8, 64, batch], True).endswith("_aligned")


def test_batch_dispatch_layout_sizes_all_rhs_and_rejects_invalid_batches():
    for batch in range(1, 5):
        sizes, threads = dispatch_layout("matmul_affine", [3, 128, 4, 64, batch])
        assert sizes == [192, 24, 24, 512 * batch, 12 * batch]
        assert threads == 96
        sizes, _ = dispatch_layout("matmul_affine_bf16", [3, 128, 8, 32, batch])
        assert sizes == [384, 24, 24, 512 * batch, 12 * batch]
        sizes, _ = dispatch_layout("matmul_f16", [3, 127, batch])
        assert sizes == [762, 508 * batch, 12 * batch]
    for batch in [0, 5, U32_MAX]:
        with pytest.raises(QmrError):
            dispatch_layout("matmul_affine", [3, 128, 4, 64, batch])
        with pytest.raises(QmrError):
            dispatch_layout("matmul_f16", [3, 127, batch])
    for p in [[3, 127, 4, 64, 2], [3, 256, 4, 256, 2], [3, 128, 2, 64, 2], [U32_MAX, 128, 4, 64, 4]]:
        with pytest.raises(QmrError):
            dispatch_layout("matmul_affine", p)
    with pytest.raises(QmrError):
        dispatch_layout("matmul_f16", [1, U32_MAX, 4])
    assert dispatch_layout("copy_f32", [7]) == ([28, 28], 7)
    with pytest.raises(QmrError):
        dispatch_layout("copy_f32", [0])


def test_bf16_dispatch_keeps_metadata_typed_and_rejects_unsupported_groups():
    assert dispatch_layout("matvec_affine_bf16", [20, 5120, 4, 64]) == ([51200, 3200, 3200, 20480, 80], 640)
    assert dispatch_layout("embed_affine_bf16", [249999, 5120, 4, 64]) == (
        [640_000_000, 40_000_000, 40_000_000, 20480], 5120)
    for name in ["matvec_affine_bf16", "embed_affine_bf16"]:
        for p in [[2, 256, 4, 256], [2, 128, 4, 8], [2, 128, 2, 64], [2, 127, 4, 64]]:
            with pytest.raises(QmrError):
                dispatch_layout(name, p)


def test_bf16_aligned_kernel_requires_q4_group64_and_safe_dimensions():
    assert select("matvec_affine_bf16", [20, 5120, 4, 64], True) == "matvec_q4_g64_aligned_bf16"
    for p in [[19, 5120, 4, 64], [20, 192, 4, 64], [524288, 8192, 4, 64]]:
        assert select("matvec_affine_bf16", p, True) == "matvec_q4_g64_bf16"
    for aligned in [True, False]:
        assert select("matvec_affine_bf16", [20, 5120, 4, 32], aligned) == "matvec_q4_g32_bf16"
        assert select("matvec_affine_bf16", [20, 5120, 4, 128], aligned) == "matvec_q4_g128_bf16"
        assert select("matvec_affine_bf16", [20, 5120, 8, 64], aligned) == "matvec_q8_g64_bf16"
        assert select("matvec_affine_bf16", [20, 5120, 4, 256], aligned) is None
    assert select("matvec_affine_bf16", [20, 5120, 4, 64], False) == "matvec_q4_g64_bf16"


def test_aligned_dispatch_requires_safe_dimensions():
    assert select("matvec_affine", [20, 5120, 4, 64], True) == "matvec_q4_g64_aligned"
    for p in [[19, 5120, 4, 64], [20, 192, 4, 64], [524288, 8192, 4, 64]]:
        assert select("matvec_affine", p, True) == "matvec_q4_g64"
    assert select("matvec_affine", [20, 5120, 4, 256], True) is None
    assert select("matvec_affine", [20, 5120, 8, 64], True) == "matvec_q8_g64"
    assert select("matvec_affine", [20, 5120, 4, 64], False) == "matvec_q4_g64"


def test_rejects_invalid_shapes_and_index_overflow_before_dispatch():
    f = lambda v: int(np.array(v, np.float32).view(np.uint32))  # noqa: E731
    for name, p in [("matvec_affine", [2, 7, 4, 8]), ("matvec_affine", [2, 8, 3, 8]),
                    ("matvec_f16", [U32_MAX, 2]), ("delta_step", [3, 4, 2, 2]), ("attn_scores", [3, 2, 2, 2]),
                    ("rope", [1, 4, 6, 0, f(10000.0)]), ("head_rms", [1, 2, f(float("nan"))]),
                    ("conv_silu", [2, 0]), ("typo", [2])]:
        with pytest.raises(QmrError):
            dispatch_layout(name, p)


def test_packed_large_vocabulary_and_cache_bounds_use_checked_sizes():
    assert dispatch_layout("embed_affine", [249999, 5120, 4, 64]) == (
        [640_000_000, 80_000_000, 80_000_000, 20480], 5120)
    assert dispatch_layout("kv_append", [2, 4, 9])[0] == [32, 32, 320, 320]


def test_error_codes_are_typed():
    with pytest.raises(QmrError) as e:
        dispatch_layout("typo", [2])
    assert e.value.code == qmr._lib.QMR_EUNSUPPORTED
    with pytest.raises(QmrError) as e:
        qmr.checked_buffer_range(2, 4, 16)
    assert e.value.code == qmr._lib.QMR_EALIGN
    with pytest.raises(QmrError) as e:
        dispatch_layout("matvec_affine", [2, 8, 3, 8])
    assert e.value.code == qmr._lib.QMR_EINVAL


def test_pack_bf16_exact_matches_oracle_semantics():
    patterns = np.array([0x00000000, 0x80000000, 0x3FC00000, 0x7F7F0000], np.uint32)
    v = patterns.view(np.float32)
    assert (qmr.pack_bf16_exact(v).astype(np.uint32) << 16).tolist() == patterns.tolist()
    assert qmr.pack_bf16_exact(np.array([0.1], np.float32)) is None


def test_encode_requires_init_or_device():
    """qmr_encode refuses to run before qmr_init (no device state yet)."""
    lib = qmr.lib()
    if lib.qmr_get_modes(ctypes.create_string_buffer(256), 256) != 0:
        pytest.skip("modes unavailable")
    bufs = (qmr._lib.qmr_buffer * 1)()
    p = (ctypes.c_uint32 * 1)(4)
    rc = lib.qmr_encode(b"copy_f32", bufs, None, 1, p, 1, 4, 32, None)
    assert rc in (qmr._lib.QMR_ENOTINIT, qmr._lib.QMR_EINVAL)
