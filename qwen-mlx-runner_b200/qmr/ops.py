"""Typed entry points over torch CUDA tensors (include/qmr.h typed section).

These stand in for the engine-side calls of the reference:
Matrix::matvec (src/engine.rs:137-164), Matrix::matmul_block
(src/engine/block.rs:191-229), Matrix::embed (src/engine.rs:166-188), the
gate/up + swiglu step (src/engine.rs:755-763) and the head + greedy argmax
(src/engine.rs:777-780, src/chat.rs:383-390).  All arithmetic runs in
libqmr's sm_100a kernels; these wrappers only pass pointers.
"""
from __future__ import annotations

import dataclasses
from typing import Optional

from . import _lib
from ._lib import QmrError, check


def _ptr(t, min_bytes: int = 0, what: str = "tensor"):
    """Device address of t after checking it is a contiguous CUDA tensor with
    at least min_bytes bytes (the C ABI cannot see tensor extents)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise QmrError(_lib.QMR_EINVAL, f"{what} must live on a CUDA device")
    if not t.is_contiguous():
        raise QmrError(_lib.QMR_EINVAL, f"{what} must be contiguous")
    nbytes = t.nbytes
    if nbytes < min_bytes:
        raise QmrError(_lib.QMR_ERANGE, f"{what} holds {nbytes} bytes, the call needs {min_bytes}")
    return t.data_ptr()


def _act(t, min_bytes: int, what: str = "x"):
    """Address of an activation input: a contiguous CUDA tensor, or a pinned
    (page-locked) host tensor, which the kernels read directly over the host
    link (unified addressing) instead of a separate copy."""
    if t is not None and not t.is_cuda and t.is_pinned():
        if not t.is_contiguous():
            raise QmrError(_lib.QMR_EINVAL, f"{what} must be contiguous")
        if t.nbytes < min_bytes:
            raise QmrError(_lib.QMR_ERANGE, f"{what} holds {t.nbytes} bytes, the call needs {min_bytes}")
        return t.data_ptr()
    return _ptr(t, min_bytes, what)


def _mat(m: "PackedMatrix"):
    """Pointers of a packed matrix after checking its buffers cover the shape
    (checked once per set of buffer objects, then reused)."""
    key = (id(m.weight), id(m.scales), id(m.biases), m.rows, m.cols, m.bits, m.group)
    cached = m.__dict__.get("_ptrs")
    if cached is not None and cached[0] == key:
        return cached[1]
    elems = m.rows * m.cols
    wbytes = elems * m.bits // 8
    mbytes = (elems // m.group) * (2 if m.meta_bf16 else 4) if m.group else 0
    ptrs = (_ptr(m.weight, wbytes, "weights"), _ptr(m.scales, mbytes, "scales"),
            _ptr(m.biases, mbytes, "biases"))
    m.__dict__["_ptrs"] = (key, ptrs)
    return ptrs


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


@dataclasses.dataclass
class PackedMatrix:
    """A packed affine matrix resident on the device (MatrixData::Packed,
    src/weights.rs): u32 words [rows, cols*bits/32], metadata [rows, cols/group]
    as float32 or as uint16 bf16 high halves."""
    weight: "object"
    scales: "object"
    biases: "object"
    rows: int
    cols: int
    bits: int
    group: int

    @property
    def meta_bf16(self) -> bool:
        import torch
        return self.scales.dtype in (torch.int16, torch.uint16, torch.bfloat16)

    @property
    def nbytes(self) -> int:
        return (self.weight.numel() * self.weight.element_size()
                + 2 * self.scales.numel() * self.scales.element_size())


def matvec_affine(m: PackedMatrix, x, y, stream=None) -> None:
    w, sc, bi = _mat(m)
    check(_lib.lib().qmr_matvec_affine(w, sc, bi, _act(x, 4 * m.cols), _ptr(y, 4 * m.rows, "y"),
                                       m.rows, m.cols, m.bits, m.group, int(m.meta_bf16), _stream(stream)))


def matmul_affine(m: PackedMatrix, x, y, batch: int, stream=None) -> None:
    w, sc, bi = _mat(m)
    check(_lib.lib().qmr_matmul_affine(w, sc, bi, _act(x, 4 * batch * m.cols),
                                       _ptr(y, 4 * batch * m.rows, "y"), m.rows, m.cols, m.bits, m.group, batch,
                                       int(m.meta_bf16), _stream(stream)))


def matmul_affine_static(m: PackedMatrix, x, y, batch: int, stream=None) -> None:
    """matmul_affine on the library's fixed per-device scratch: allocates no
    device memory (cols <= 32768); calls must not overlap in time."""
    w, sc, bi = _mat(m)
    check(_lib.lib().qmr_matmul_affine_static(w, sc, bi, _act(x, 4 * batch * m.cols),
                                              _ptr(y, 4 * batch * m.rows, "y"), m.rows, m.cols, m.bits, m.group,
                                              batch, int(m.meta_bf16), _stream(stream)))


def embed_affine(m: PackedMatrix, row: int, y, stream=None) -> None:
    w, sc, bi = _mat(m)
    if not 0 <= row < m.rows:
        raise QmrError(_lib.QMR_ERANGE, f"row {row} outside a {m.rows}-row matrix")
    check(_lib.lib().qmr_embed_affine(w, sc, bi, row, _ptr(y, 4 * m.cols, "y"), m.cols, m.bits, m.group,
                                      int(m.meta_bf16), _stream(stream)))


def gateup_swiglu(gate: PackedMatrix, up: PackedMatrix, x, act, batch: int, stream=None) -> None:
    if (gate.rows, gate.cols, gate.bits, gate.group, gate.meta_bf16) != (up.rows, up.cols, up.bits, up.group,
                                                                         up.meta_bf16):
        raise QmrError(_lib.QMR_EINVAL, "gate and up matrices must share shape and format")
    gw, gs, gb = _mat(gate)
    uw, us, ub = _mat(up)
    check(_lib.lib().qmr_gateup_swiglu(gw, gs, gb, uw, us, ub, _act(x, 4 * batch * gate.cols),
                                       _ptr(act, 4 * batch * gate.rows, "act"), gate.rows, gate.cols, gate.bits,
                                       gate.group, batch, int(gate.meta_bf16), _stream(stream)))


def head_argmax(m: PackedMatrix, x, logits, argmax, batch: int, best_key=None, row_base: int = 0,
                stream=None) -> None:
    w, sc, bi = _mat(m)
    check(_lib.lib().qmr_head_argmax(w, sc, bi, _act(x, 4 * batch * m.cols),
                                     _ptr(logits, 4 * batch * m.rows, "logits"), _ptr(argmax, 4 * batch, "argmax"),
                                     _ptr(best_key, 8 * batch, "best_key"), m.rows, m.cols, m.bits, m.group,
                                     batch, int(m.meta_bf16), row_base, _stream(stream)))


def prepared_bytes(bits: int, cols: int, batch: int) -> int:
    return int(_lib.lib().qmr_prepared_bytes(bits, cols, batch))


def alloc_prepared(bits: int, cols: int, batch: int, device="cuda"):
    """A caller-owned prepared-activation buffer (uint8 CUDA tensor, 256-aligned)."""
    import torch
    return torch.empty(prepared_bytes(bits, cols, batch), dtype=torch.uint8, device=device)


def prepare_activations(x, cols: int, bits: int, batch: int, prepared, group: int = 64, stream=None) -> None:
    check(_lib.lib().qmr_prepare_activations(_act(x, 4 * batch * cols), cols, bits, group, batch,
                                             _ptr(prepared, prepared_bytes(bits, cols, batch), "prepared"),
                                             prepared.numel() * prepared.element_size(), _stream(stream)))


def matmul_prepared(m: PackedMatrix, prepared, y, batch: int, overlap: bool = False, stream=None) -> None:
    """overlap=True lets the kernel read this matrix while the previous kernel
    on the stream still runs (it must not write the matrix)."""
    w, sc, bi = _mat(m)
    check(_lib.lib().qmr_matmul_prepared(w, sc, bi, _ptr(prepared, prepared_bytes(m.bits, m.cols, batch),
                                                         "prepared"),
                                         _ptr(y, 4 * batch * m.rows, "y"), m.rows, m.cols, m.bits, m.group, batch,
                                         int(m.meta_bf16), 1 if overlap else 0, _stream(stream)))


def gateup_swiglu_exchange(gate: PackedMatrix, up: PackedMatrix, x, batch: int, exchange, stream=None) -> None:
    """This rank's rows of silu(gate x) * (up x) into every rank's full
    activation buffer (`exchange`: a _lib.QmrExchange; see qmr.parallel)."""
    wg, sg, bg = _mat(gate)
    wu, su, bu = _mat(up)
    check(_lib.lib().qmr_gateup_swiglu_exchange(wg, sg, bg, wu, su, bu, _act(x, 4 * batch * gate.cols),
                                                gate.rows, gate.cols, gate.bits, gate.group, batch,
                                                int(gate.meta_bf16), exchange, _stream(stream)))


def matmul_affine_exchange(m: PackedMatrix, x, batch: int, exchange, stream=None) -> None:
    """This rank's rows of m x into every rank's full output buffer."""
    w, sc, bi = _mat(m)
    check(_lib.lib().qmr_matmul_affine_exchange(w, sc, bi, _act(x, 4 * batch * m.cols), m.rows, m.cols, m.bits,
                                                m.group, batch, int(m.meta_bf16), exchange, _stream(stream)))


def head_argmax_exchange(m: PackedMatrix, x, logits, batch: int, exchange, stream=None) -> None:
    """This rank's vocabulary shard: local logits, its best key per RHS to
    every rank."""
    w, sc, bi = _mat(m)
    check(_lib.lib().qmr_head_argmax_exchange(w, sc, bi, _act(x, 4 * batch * m.cols),
                                              _ptr(logits, 4 * batch * m.rows, "logits"), m.rows, m.cols, m.bits,
                                              m.group, batch, int(m.meta_bf16), exchange, _stream(stream)))


def exchange_wait(exchange, batch: int, argmax=None, best_key=None, stream=None) -> None:
    """Wait for every rank's current exchange; for a head exchange also write
    the merged token ids (int32 [batch]) and keys (int64 [batch])."""
    check(_lib.lib().qmr_exchange_wait(exchange, batch, _ptr(argmax, 4 * batch, "argmax"),
                                       _ptr(best_key, 8 * batch, "best_key"), _stream(stream)))


def copy_f32(x, y, n: int, stream=None) -> None:
    check(_lib.lib().qmr_copy_f32(_act(x, 4 * n, "x"), _act(y, 4 * n, "y"), n, _stream(stream)))


def init(device: int = 0, reference: bool = False) -> None:
    check(_lib.lib().qmr_init(device, _lib.INIT_REFERENCE if reference else _lib.INIT_FROM_ENV))


def set_stream_path(path: str) -> None:
    """"mma" (default), "tma" or "registers": the streaming kernel of the fast path."""
    check(_lib.lib().qmr_set_stream_path(path.encode()))


def device_error(clear: bool = False) -> int:
    """Error word of the bounded device waits (0 = none).  Synchronises."""
    import ctypes
    code = ctypes.c_int()
    check(_lib.lib().qmr_device_error(ctypes.byref(code), int(clear)))
    return code.value


def decode_key(key: int):
    """(index, f32 logit) from a packed argmax key (qmr_head_argmax best_key)."""
    import struct
    hi = (key >> 32) & 0xFFFFFFFF
    bits = (hi & 0x7FFFFFFF) if hi & 0x80000000 else (~hi) & 0xFFFFFFFF
    value = struct.unpack("<f", struct.pack("<I", bits))[0]
    return 0xFFFFFFFF - (key & 0xFFFFFFFF), value
