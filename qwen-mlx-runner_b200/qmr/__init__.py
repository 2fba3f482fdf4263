"""qmr: B200 (sm_100a) packed-affine GEMV / block-matmul path behind the
reference engine's matrix-dispatch ABI (include/qmr.h).

Python here is host glue over libqmr.so: the dispatch mirror (gpu.py), typed
entry points (ops.py), the checkpoint loader and decode engine mirror
(engine.py), synthetic benchmark inputs (synth.py) and the build recipe
(build.py).  All arithmetic runs in the CUDA library.
"""
from ._lib import QmrError, lib  # noqa: F401
from .gpu import BlockKernelMode, DispatchEncoder, Gpu, checked_buffer_range, dispatch_layout, pack_bf16_exact, select  # noqa: F401
from .ops import PackedMatrix, copy_f32, embed_affine, gateup_swiglu, head_argmax, matmul_affine, matvec_affine  # noqa: F401
from .engine import Checkpoint, Engine  # noqa: F401

__all__ = [
    "QmrError", "lib", "BlockKernelMode", "DispatchEncoder", "Gpu", "checked_buffer_range", "dispatch_layout",
    "pack_bf16_exact", "select", "PackedMatrix", "copy_f32", "embed_affine", "gateup_swiglu", "head_argmax",
    "matmul_affine", "matvec_affine", "Checkpoint", "Engine",
]
