"""qmr_matmul_affine_static, the entry point that allocates no device memory.

Callers that cannot allocate device memory once they run -- a serving engine
that reserves its whole HBM budget at start-up, or a foreign binding that has
no way to own a scratch buffer -- use this entry point.  It runs the same
kernels and launch plan as qmr_matmul_affine on a fixed per-device array, so
its result must equal qmr_matmul_affine's bit for bit, and both must meet the
north-star bound against the FP64 oracle.

This file is collected last so that it also runs after every other test has
used the per-stream scratch path; it passes on its own as well.  Its first
test makes the first static call of a fresh process on a non-blocking stream,
which is where the set-up's clear of the array must already have finished.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import qmr
from qmr import _lib, synth
from qmr._lib import QmrError

pytestmark = pytest.mark.gpu

NS_RTOL = 2e-5


def f32_tensor(v):
    return torch.from_numpy(np.ascontiguousarray(v, np.float32)).to("cuda")


def call_static(m, x, y, batch, stream):
    """Through the C ABI directly, as a foreign binding would."""
    lib = _lib.lib()
    w, s, b = (ctypes.c_void_p(t.data_ptr()) for t in (m.weight, m.scales, m.biases))
    return lib.qmr_matmul_affine_static(w, s, b, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                        m.rows, m.cols, m.bits, m.group, batch, int(m.meta_bf16),
                                        ctypes.c_void_p(stream.cuda_stream))


def check_static(rows, cols, bits, batch, meta, seed, stream):
    mat = synth.affine_matrix(rows, cols, bits, 64, seed=seed, meta=meta)
    m = synth.to_device(mat, rows, cols, bits, 64)
    x_np = synth.activations(batch, cols, seed=seed + 10)
    x = f32_tensor(x_np.ravel())
    ref = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
    qmr.matmul_affine(m, x, ref, batch)
    torch.cuda.synchronize()
    want_bits = ref.cpu().numpy().view(np.uint32)
    want, mag = oracle.matmul_f64(mat["weight"], mat["scales"], mat["biases"], x_np, rows, cols, bits, 64,
                                  batch=batch)
    for call in range(2):  # the first call may set up, the second reuses the array's last contents
        y = torch.full((batch * rows,), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        assert call_static(m, x, y, batch, stream) == 0, _lib.lib().qmr_last_error()
        stream.synchronize()
        got = y.cpu().numpy()
        # Same kernels and launch plan on a different scratch base: identical bits.
        bad = np.flatnonzero(got.view(np.uint32) != want_bits)
        assert bad.size == 0, f"call {call}: {bad.size} outputs differ from qmr_matmul_affine, first {bad[0]}"
        ratio, i = oracle.tolerance_ratio(got.reshape(batch, rows), want, mag, rtol=NS_RTOL, atol=0.0)
        assert ratio <= 1.0, f"call {call}: output {i} ratio {ratio}"
    assert qmr.ops.device_error() == 0


def test_first_static_call_on_a_non_blocking_stream(cuda):
    stream = torch.cuda.Stream()  # cudaStreamNonBlocking: no implicit order with the legacy stream
    check_static(2048, 5120, 4, 3, "bf16", 690, stream)


@pytest.mark.parametrize("rows,cols,bits,batch,meta", [
    (4096, 5120, 4, 3, "bf16"),
    (4096, 5120, 8, 1, "f32"),
    (4096, 5120, 4, 4, "f32"),
    (1024, 32768, 4, 4, "bf16"),  # the documented limit: cols 32768 at batch 4
    (1024, 32768, 8, 4, "bf16"),  # the largest scratch the array must hold
])
def test_static_scratch_matches_the_allocating_entry_point(cuda, rows, cols, bits, batch, meta):
    stream = torch.cuda.current_stream()
    check_static(rows, cols, bits, batch, meta, 700 + bits + batch + cols // 1024, stream)


def test_static_scratch_rejects_shapes_beyond_its_size(cuda):
    rows, cols = 16, 32768 + 512
    w = torch.zeros(rows * cols // 8, dtype=torch.int32, device="cuda")
    s = torch.zeros(rows * cols // 64, dtype=torch.float32, device="cuda")
    m = qmr.ops.PackedMatrix(w, s, s, rows, cols, 4, 64)
    x = torch.zeros(cols, dtype=torch.float32, device="cuda")
    y = torch.zeros(rows, dtype=torch.float32, device="cuda")
    with pytest.raises(QmrError) as e:
        qmr.ops.matmul_affine_static(m, x, y, 1)
    assert e.value.code == _lib.QMR_ERANGE
    assert "static scratch" in str(e.value)
