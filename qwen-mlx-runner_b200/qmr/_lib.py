"""ctypes binding of libqmr.so (include/qmr.h).

The library is loaded from the package directory only; a missing or stale
library is an error, never a reason to fall back to another implementation.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import threading

PKG_ROOT = pathlib.Path(__file__).resolve().parents[1]
LIB_PATH = PKG_ROOT / "libqmr.so"

QMR_OK = 0
QMR_EINVAL = -1
QMR_ERANGE = -2
QMR_EALIGN = -3
QMR_EOVERLAP = -4
QMR_EUNSUPPORTED = -5
QMR_ECUDA = -6
QMR_ETIMEOUT = -7
QMR_ENOTINIT = -8

ERROR_NAMES = {
    QMR_EINVAL: "EINVAL", QMR_ERANGE: "ERANGE", QMR_EALIGN: "EALIGN",
    QMR_EOVERLAP: "EOVERLAP", QMR_EUNSUPPORTED: "EUNSUPPORTED", QMR_ECUDA: "ECUDA",
    QMR_ETIMEOUT: "ETIMEOUT", QMR_ENOTINIT: "ENOTINIT",
}

BLOCK_LEGACY, BLOCK_SHARED, BLOCK_MLP_R2 = 0, 1, 2
INIT_FROM_ENV, INIT_REFERENCE = 0, 1


class QmrError(RuntimeError):
    """A negative status from libqmr, with the library's message."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message


class qmr_buffer(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("length", ctypes.c_uint64)]


_lib = None
_lock = threading.Lock()

_vp = ctypes.c_void_p

QMR_MAX_RANKS = 8
QMR_IPC_HANDLE_BYTES = 64


class QmrExchange(ctypes.Structure):
    """struct QmrExchange (include/qmr.h): the peer buffers of one output
    exchange."""
    _fields_ = [("world", ctypes.c_uint32), ("rank", ctypes.c_uint32), ("total_rows", ctypes.c_uint32),
                ("row_base", ctypes.c_uint32), ("out", ctypes.c_void_p * QMR_MAX_RANKS),
                ("flags", ctypes.c_void_p * QMR_MAX_RANKS), ("keys", ctypes.c_void_p * QMR_MAX_RANKS),
                ("epoch", ctypes.c_void_p)]
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_int = ctypes.c_int
_sz = ctypes.c_size_t
_cstr = ctypes.c_char_p

QMR_MAX_LAYERS = 256


class QmrModelConfig(ctypes.Structure):
    """struct QmrModelConfig (include/qmr.h): ModelConfig (src/config.rs:4-25)."""
    _fields_ = [("hidden_size", ctypes.c_uint32), ("intermediate_size", ctypes.c_uint32),
                ("num_layers", ctypes.c_uint32), ("num_heads", ctypes.c_uint32), ("num_kv_heads", ctypes.c_uint32),
                ("head_dim", ctypes.c_uint32), ("vocab_size", ctypes.c_uint32),
                ("linear_key_heads", ctypes.c_uint32), ("linear_value_heads", ctypes.c_uint32),
                ("linear_key_dim", ctypes.c_uint32), ("linear_value_dim", ctypes.c_uint32),
                ("conv_width", ctypes.c_uint32), ("rotary_dim", ctypes.c_uint32), ("rms_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float), ("is_attention", ctypes.c_uint8 * QMR_MAX_LAYERS)]

# name -> (restype, argtypes)
SIGNATURES = {
    "qmr_abi_version": (_int, []),
    "qmr_last_error": (_cstr, []),
    "qmr_init": (_int, [_int, _u32]),
    "qmr_set_modes": (_int, [_cstr, _cstr, _cstr, _cstr]),
    "qmr_get_modes": (_int, [ctypes.c_char_p, _sz]),
    "qmr_parse_block_mode": (_int, [_cstr, _cstr, _cstr, ctypes.POINTER(_int), ctypes.POINTER(_int)]),
    "qmr_dispatch_layout": (_int, [_cstr, ctypes.POINTER(_u32), _sz, ctypes.POINTER(_u64),
                                   ctypes.POINTER(_sz), ctypes.POINTER(_u64)]),
    "qmr_checked_buffer_range": (_int, [_u64, _u64, _u64]),
    "qmr_select": (_int, [_cstr, ctypes.POINTER(_u32), _sz, _int, _int, ctypes.c_char_p, _sz]),
    "qmr_pack_bf16_exact": (_int, [_vp, _u64, _vp]),
    "qmr_encode": (_int, [_cstr, ctypes.POINTER(qmr_buffer), ctypes.POINTER(_u64), _sz,
                          ctypes.POINTER(_u32), _sz, _u64, _u64, _vp]),
    "qmr_matvec_affine": (_int, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _int, _vp]),
    "qmr_matmul_affine": (_int, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _int, _vp]),
    "qmr_matmul_affine_static": (_int, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _int, _vp]),
    "qmr_embed_affine": (_int, [_vp, _vp, _vp, _u32, _vp, _u32, _u32, _u32, _int, _vp]),
    "qmr_gateup_swiglu": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32,
                                 _u32, _int, _vp]),
    "qmr_head_argmax": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32,
                               _int, _u32, _vp]),
    "qmr_prepared_bytes": (_u64, [_u32, _u32, _u32]),
    "qmr_prepare_activations": (_int, [_vp, _u32, _u32, _u32, _u32, _vp, _u64, _vp]),
    "qmr_matmul_prepared": (_int, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _int, _u32, _vp]),
    "qmr_copy_f32": (_int, [_vp, _vp, _u32, _vp]),
    "qmr_stream_sync": (_int, [_vp]),
    "qmr_set_stream_path": (_int, [_cstr]),
    "qmr_device_error": (_int, [ctypes.POINTER(_int), _int]),
    "qmr_exchange_alloc": (_int, [_sz, ctypes.POINTER(_vp)]),
    "qmr_exchange_free": (_int, [_vp]),
    "qmr_ipc_handle": (_int, [_vp, ctypes.c_char_p]),
    "qmr_ipc_open": (_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "qmr_ipc_close": (_int, [_vp]),
    "qmr_matmul_affine_exchange": (_int, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _int,
                                          ctypes.POINTER(QmrExchange), _vp]),
    "qmr_gateup_swiglu_exchange": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _int,
                                          ctypes.POINTER(QmrExchange), _vp]),
    "qmr_head_argmax_exchange": (_int, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _int,
                                        ctypes.POINTER(QmrExchange), _vp]),
    "qmr_exchange_wait": (_int, [ctypes.POINTER(QmrExchange), _u32, _vp, _vp, _vp]),
    "qmr_checkpoint_open": (_int, [_cstr, ctypes.POINTER(_vp)]),
    "qmr_checkpoint_close": (None, [_vp]),
    "qmr_checkpoint_config": (_int, [_vp, ctypes.POINTER(QmrModelConfig), ctypes.POINTER(_u32),
                                     ctypes.POINTER(_int)]),
    "qmr_checkpoint_matrix": (_int, [_vp, _cstr, ctypes.POINTER(_u32), ctypes.POINTER(_u32), ctypes.POINTER(_u32),
                                     ctypes.POINTER(_u32), _vp, _vp, _vp]),
    "qmr_checkpoint_vector": (_int, [_vp, _cstr, _vp, _u64, ctypes.POINTER(_u64)]),
    "qmr_model_load": (_int, [_cstr, _u32, ctypes.POINTER(_vp)]),
    "qmr_model_synthetic": (_int, [ctypes.POINTER(QmrModelConfig), _u64, _u32, ctypes.POINTER(_vp)]),
    "qmr_model_free": (None, [_vp]),
    "qmr_model_config": (_int, [_vp, ctypes.POINTER(QmrModelConfig), ctypes.POINTER(_u32)]),
    "qmr_model_reset": (_int, [_vp]),
    "qmr_model_position": (_int, [_vp, ctypes.POINTER(_u32)]),
    "qmr_model_forward": (_int, [_vp, _u32, _vp, _vp]),
    "qmr_model_generate": (_int, [_vp, _vp, _u32, _u32, _vp, ctypes.POINTER(ctypes.c_double),
                                  ctypes.POINTER(ctypes.c_double)]),
    "qmr_model_verify_block": (_int, [_vp, _vp, _u32, _vp, _vp]),
    "qmr_model_commit_block": (_int, [_vp, _u32]),
    "qmr_model_mtp_generate": (_int, [_vp, _vp, _u32, _u32, _u32, _vp, _u32, _vp, ctypes.POINTER(_u32),
                                      ctypes.POINTER(_u32), ctypes.POINTER(ctypes.c_double),
                                      ctypes.POINTER(ctypes.c_double)]),
    "qmr_model_mlp_r2_eligible": (_int, [_vp, ctypes.POINTER(_u32)]),
    "qmr_model_metadata_stats": (_int, [_vp, ctypes.POINTER(_u64), ctypes.POINTER(_u64)]),
    "qmr_model_step_launches": (_int, [_vp, ctypes.POINTER(_u32), ctypes.POINTER(_u32)]),
    "qmr_model_synthetic_sharded": (_int, [ctypes.POINTER(QmrModelConfig), _u64, _u32, _u32, _u32,
                                           ctypes.POINTER(_vp)]),
    "qmr_model_exchange_handle": (_int, [_vp, _vp]),
    "qmr_model_exchange_open": (_int, [_vp, _vp]),
    "qmr_model_shard": (_int, [_vp, ctypes.POINTER(_u32), ctypes.POINTER(_u32), ctypes.POINTER(_u32),
                               ctypes.POINTER(_u32)]),
}


def lib() -> ctypes.CDLL:
    """Load libqmr.so once.  Raises if it is absent: there is no fallback."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                    "(python qwen-mlx-runner_b200/qmr/build.py)")
            handle = ctypes.CDLL(os.fspath(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
        return _lib


def check(rc: int) -> int:
    if rc < 0:
        msg = lib().qmr_last_error()
        raise QmrError(rc, msg.decode() if msg else "")
    return rc


def u32_array(values) -> ctypes.Array:
    values = [int(v) for v in values]
    for v in values:
        if not 0 <= v <= 0xFFFFFFFF:
            raise ValueError(f"parameter {v} does not fit u32")
    return (_u32 * len(values))(*values)


def enc(s):
    return None if s is None else s.encode()
