"""Host-side mirror of the reference's matrix dispatch surface.

`Gpu` and `DispatchEncoder` keep the names, argument meaning and error
behaviour of rucin93/qwen-mlx-runner's src/gpu.rs (Gpu::new*,
DispatchEncoder::encode / encode_offsets, set_block_kernel_mode,
kernel_mode, metadata_mode) on top of libqmr's C ABI.  Buffers are torch
CUDA tensors; a tensor's whole storage is the "buffer" and byte offsets
select views inside it, as Metal buffers and offsets do in the reference.
Every call goes through libqmr; errors raise QmrError before anything is
enqueued.
"""
from __future__ import annotations

import ctypes
import dataclasses
from typing import Optional, Sequence

from . import _lib
from ._lib import QmrError, check, enc, u32_array

BLOCK_MODES = {"legacy": _lib.BLOCK_LEGACY, "shared": _lib.BLOCK_SHARED, "mlp-r2": _lib.BLOCK_MLP_R2}
BLOCK_MODE_NAMES = {v: k for k, v in BLOCK_MODES.items()}


@dataclasses.dataclass(frozen=True)
class BlockKernelMode:
    """BlockKernelMode (src/gpu.rs:33-47): matmul schedule + batched DeltaNet."""
    matmul: str = "legacy"
    batched_delta: bool = True

    @staticmethod
    def parse_for_device(device_name: str, matmul: Optional[str], delta: Optional[str]) -> "BlockKernelMode":
        mode = ctypes.c_int()
        batched = ctypes.c_int()
        check(_lib.lib().qmr_parse_block_mode(enc(device_name), enc(matmul), enc(delta),
                                              ctypes.byref(mode), ctypes.byref(batched)))
        return BlockKernelMode(BLOCK_MODE_NAMES[mode.value], bool(batched.value))

    @staticmethod
    def parse(matmul: str, delta: str) -> "BlockKernelMode":
        return BlockKernelMode.parse_for_device("", matmul, delta)


def dispatch_layout(name: str, params: Sequence[int]):
    """dispatch_layout (src/gpu.rs:1041): (buffer byte sizes, logical threads)."""
    p = u32_array(params)
    sizes = (ctypes.c_uint64 * 8)()
    count = ctypes.c_size_t()
    threads = ctypes.c_uint64()
    check(_lib.lib().qmr_dispatch_layout(name.encode(), p, len(params), sizes, ctypes.byref(count),
                                         ctypes.byref(threads)))
    return [int(sizes[i]) for i in range(count.value)], int(threads.value)


def checked_buffer_range(offset: int, minimum: int, length: int) -> None:
    check(_lib.lib().qmr_checked_buffer_range(offset, minimum, length))


def select(name: str, params: Sequence[int], aligned: bool, mode: str = "legacy") -> Optional[str]:
    """specialized_matmul / specialized_matvec[_bf16]: the reference's kernel name, or None."""
    p = u32_array(params)
    out = ctypes.create_string_buffer(96)
    rc = _lib.lib().qmr_select(name.encode(), p, len(params), int(aligned), BLOCK_MODES[mode], out, 96)
    if rc == _lib.QMR_EUNSUPPORTED:
        return None
    check(rc)
    return out.value.decode()


def pack_bf16_exact(values):
    """pack_bf16_exact (src/gpu/metadata.rs:6): uint16 array or None."""
    import numpy as np
    v = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(v.shape, dtype=np.uint16)
    ok = _lib.lib().qmr_pack_bf16_exact(v.ctypes.data, v.size, out.ctypes.data)
    return out if ok else None


def _stream_handle(stream) -> Optional[int]:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


def _buffer(t) -> _lib.qmr_buffer:
    """A torch tensor as a qmr_buffer: its storage base and byte length."""
    if not t.is_cuda:
        raise QmrError(_lib.QMR_EINVAL, "buffers must be CUDA tensors")
    storage = t.untyped_storage()
    return _lib.qmr_buffer(storage.data_ptr(), storage.nbytes())


class Gpu:
    """Gpu (src/gpu.rs:95-110, 293-470) over libqmr.

    reference=True mirrors Gpu::new_with_reference(true): per-element
    reference kernels, no block dispatch, no BF16 metadata.  variant mirrors
    Gpu::new_with_variant (packed4 | aligned | stream).
    """

    def __init__(self, device: int = 0, reference: Optional[bool] = None, variant: Optional[str] = None):
        flags = _lib.INIT_REFERENCE if reference else _lib.INIT_FROM_ENV
        self.device = device
        check(_lib.lib().qmr_init(device, flags))
        if variant is not None:
            check(_lib.lib().qmr_set_modes(variant.encode(), None, None, None))
        self._activate()

    @classmethod
    def new_with_reference(cls, reference: bool, device: int = 0) -> "Gpu":
        return cls(device=device, reference=reference)

    @classmethod
    def new_with_variant(cls, reference: bool, variant: str, device: int = 0) -> "Gpu":
        return cls(device=device, reference=reference, variant=variant)

    # libqmr keeps one mode set per process; each Gpu re-applies its own before use.
    def _activate(self):
        self._modes = self.modes()

    def _apply(self):
        m = self._modes
        if (self.modes() != m):
            flags = _lib.INIT_REFERENCE if m["reference"] == "1" else _lib.INIT_FROM_ENV
            check(_lib.lib().qmr_init(self.device, flags))
            gemv = None if m["gemv"] == "reference" else m["gemv"]
            check(_lib.lib().qmr_set_modes(enc(gemv), enc(m["metadata"]), enc(m["block_matmul"]),
                                           enc(m["block_delta"])))

    def modes(self) -> dict:
        buf = ctypes.create_string_buffer(256)
        check(_lib.lib().qmr_get_modes(buf, 256))
        return dict(kv.split("=") for kv in buf.value.decode().split(","))

    def kernel_mode(self) -> str:
        return self._modes["gemv"]

    def metadata_mode(self) -> str:
        return self._modes["metadata"]

    def block_kernel_mode(self) -> BlockKernelMode:
        return BlockKernelMode(self._modes["block_matmul"], self._modes["block_delta"] == "batched")

    def set_block_kernel_mode(self, mode: BlockKernelMode) -> None:
        self._apply()
        check(_lib.lib().qmr_set_modes(None, None, mode.matmul.encode(),
                                       b"batched" if mode.batched_delta else b"sequential"))
        self._activate()

    def begin_encoding(self, stream=None) -> "DispatchEncoder":
        return DispatchEncoder(self, stream)

    def encode(self, name, buffers, params, threads, group_size, stream=None):
        return DispatchEncoder(self, stream).encode(name, buffers, params, threads, group_size)

    def encode_offsets(self, name, buffers, offsets, params, threads, group_size, stream=None):
        return DispatchEncoder(self, stream).encode_offsets(name, buffers, offsets, params, threads,
                                                            group_size)

    def finish(self, stream=None) -> None:
        check(_lib.lib().qmr_stream_sync(_stream_handle(stream)))


class DispatchEncoder:
    """DispatchEncoder::encode / encode_offsets (src/gpu.rs:120-174)."""

    def __init__(self, gpu: Gpu, stream=None):
        self.gpu = gpu
        self.stream = _stream_handle(stream)

    def encode(self, name, buffers, params, threads, group_size):
        return self._encode(name, buffers, None, params, threads, group_size)

    def encode_offsets(self, name, buffers, offsets, params, threads, group_size):
        return self._encode(name, buffers, offsets, params, threads, group_size)

    def _encode(self, name, buffers, offsets, params, threads, group_size):
        self.gpu._apply()
        bufs = (_lib.qmr_buffer * len(buffers))(*[_buffer(b) for b in buffers])
        if offsets is not None:
            if len(offsets) != len(buffers):
                raise QmrError(_lib.QMR_EINVAL, f"{name}: offset count must match buffers")
            for o in offsets:
                if not 0 <= int(o) < 2 ** 64:
                    raise QmrError(_lib.QMR_ERANGE, "GPU buffer view byte range overflow")
            offs = (ctypes.c_uint64 * len(offsets))(*[int(o) for o in offsets])
        else:
            offs = None
        p = u32_array(params)
        check(_lib.lib().qmr_encode(name.encode(), bufs, offs, len(buffers), p, len(params), int(threads),
                                    int(group_size), self.stream))

    def end_encoding(self):
        return None
