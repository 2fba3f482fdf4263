"""qmr_matmul_affine_static, the entry point that allocates no device memory.

This file is collected last so that it also runs after every other test has
used the per-stream scratch path; it passes on its own as well.
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


def call_static(m, x, y, batch):
    """Through the C ABI directly, as a foreign binding would."""
    lib = _lib.lib()
    w, s, b = (ctypes.c_void_p(t.data_ptr()) for t in (m.weight, m.scales, m.biases))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.qmr_matmul_affine_static(w, s, b, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                        m.rows, m.cols, m.bits, m.group, batch, int(m.meta_bf16), stream)


@pytest.mark.parametrize("bits,batch,meta", [(4, 3, "bf16"), (8, 1, "f32"), (4, 4, "f32")])
def test_static_scratch_matches_the_allocating_entry_point(cuda, bits, batch, meta):
    rows, cols = 4096, 5120
    mat = synth.affine_matrix(rows, cols, bits, 64, seed=700 + bits + batch, meta=meta)
    m = synth.to_device(mat, rows, cols, bits, 64)
    x_np = synth.activations(batch, cols, seed=710 + batch)
    x = f32_tensor(x_np.ravel())
    ref = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
    qmr.matmul_affine(m, x, ref, batch)
    torch.cuda.synchronize()
    want_dev = ref.cpu().numpy().reshape(batch, rows)
    want, mag = oracle.matmul_f64(mat["weight"], mat["scales"], mat["biases"], x_np, rows, cols, bits, 64,
                                  batch=batch)
    for call in range(2):  # the first call sets up, the second reuses the array
        y = torch.full((batch * rows,), float("nan"), dtype=torch.float32, device="cuda")
        assert call_static(m, x, y, batch) == 0, _lib.lib().qmr_last_error()
        torch.cuda.synchronize()
        got = y.cpu().numpy().reshape(batch, rows)
        # Same kernels on a different scratch: within the north-star bound of
        # the FP64 oracle and of the allocating entry point's result.
        ratio, i = oracle.tolerance_ratio(got, want, mag, rtol=NS_RTOL, atol=0.0)
        assert ratio <= 1.0, f"call {call}: output {i} ratio {ratio}"
        ratio, i = oracle.tolerance_ratio(got, want_dev, 2 * mag, rtol=NS_RTOL, atol=0.0)
        assert ratio <= 1.0, f"call {call} vs qmr_matmul_affine: output {i} ratio {ratio}"
    assert qmr.ops.device_error() == 0


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
