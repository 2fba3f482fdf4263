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


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise QmrError(_lib.QMR_EINVAL, "tensors must live on a CUDA device")
    return t.data_ptr()


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
    check(_lib.lib().qmr_matvec_affine(_ptr(m.weight), _ptr(m.scales), _ptr(m.biases), _ptr(x), _ptr(y),
                                       m.rows, m.cols, m.bits, m.group, int(m.meta_bf16), _stream(stream)))


def matmul_affine(m: PackedMatrix, x, y, batch: int, stream=None) -> None:
    check(_lib.lib().qmr_matmul_affine(_ptr(m.weight), _ptr(m.scales), _ptr(m.biases), _ptr(x), _ptr(y),
                                       m.rows, m.cols, m.bits, m.group, batch, int(m.meta_bf16),
                                       _stream(stream)))


def embed_affine(m: PackedMatrix, row: int, y, stream=None) -> None:
    check(_lib.lib().qmr_embed_affine(_ptr(m.weight), _ptr(m.scales), _ptr(m.biases), row, _ptr(y), m.cols,
                                      m.bits, m.group, int(m.meta_bf16), _stream(stream)))


def gateup_swiglu(gate: PackedMatrix, up: PackedMatrix, x, act, batch: int, stream=None) -> None:
    if (gate.rows, gate.cols, gate.bits, gate.group, gate.meta_bf16) != (up.rows, up.cols, up.bits, up.group,
                                                                         up.meta_bf16):
        raise QmrError(_lib.QMR_EINVAL, "gate and up matrices must share shape and format")
    check(_lib.lib().qmr_gateup_swiglu(_ptr(gate.weight), _ptr(gate.scales), _ptr(gate.biases), _ptr(up.weight),
                                       _ptr(up.scales), _ptr(up.biases), _ptr(x), _ptr(act), gate.rows,
                                       gate.cols, gate.bits, gate.group, batch, int(gate.meta_bf16),
                                       _stream(stream)))


def head_argmax(m: PackedMatrix, x, logits, argmax, batch: int, best_key=None, row_base: int = 0,
                stream=None) -> None:
    check(_lib.lib().qmr_head_argmax(_ptr(m.weight), _ptr(m.scales), _ptr(m.biases), _ptr(x), _ptr(logits),
                                     _ptr(argmax), _ptr(best_key), m.rows, m.cols, m.bits, m.group, batch,
                                     int(m.meta_bf16), row_base, _stream(stream)))


def copy_f32(x, y, n: int, stream=None) -> None:
    check(_lib.lib().qmr_copy_f32(_ptr(x), _ptr(y), n, _stream(stream)))


def init(device: int = 0, reference: bool = False) -> None:
    check(_lib.lib().qmr_init(device, _lib.INIT_REFERENCE if reference else _lib.INIT_FROM_ENV))


def decode_key(key: int):
    """(index, f32 logit) from a packed argmax key (qmr_head_argmax best_key)."""
    import struct
    hi = (key >> 32) & 0xFFFFFFFF
    bits = (hi & 0x7FFFFFFF) if hi & 0x80000000 else (~hi) & 0xFFFFFFFF
    value = struct.unpack("<f", struct.pack("<I", bits))[0]
    return 0xFFFFFFFF - (key & 0xFFFFFFFF), value
