"""CPU oracle for the packed-affine matrix path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline legs may
import this package; the product (libqmr, qmr) never does.  It wraps
oracle/liboracle.so, a C restatement of the reference's scalar arithmetic
(see oracle.c for the file:line each function follows).

Parity pins: the reference's own known-answer tests (src/gpu.rs:1636-1731,
src/weights.rs:816-870, tests/batch_matrix.rs:357-381, src/gpu/metadata.rs
tests) are checked against this oracle in tests/test_oracle.py, and the
reference's Python scalar oracle (scripts/make_fixture.py) output is pinned
through tests/golden/.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
SRC = HERE / "oracle.c"
SOURCES = [HERE / "oracle.c", HERE / "decode.c"]

# -ffp-contract=off: Rust never fuses a*b+c, so neither may the restatement.
CFLAGS = ["-O3", "-march=x86-64-v2", "-fPIC", "-ffp-contract=off", "-fopenmp", "-shared"]

_lib = None


def build(force: bool = False) -> pathlib.Path:
    if force or not LIB.exists() or any(LIB.stat().st_mtime < src.stat().st_mtime for src in SOURCES):
        tmp = LIB.with_suffix(".so.tmp")
        subprocess.run(["gcc", *CFLAGS, "-o", os.fspath(tmp), *map(os.fspath, SOURCES), "-lm"], check=True)
        os.replace(tmp, LIB)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists() and SRC.exists():
            build()
        h = ctypes.CDLL(os.fspath(LIB))
        vp, u32, u64, i32 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
        h.or_embed.argtypes = [vp, vp, vp, i32, u64, u32, u32, u32, vp]
        h.or_matmul_f64.argtypes = [vp, vp, vp, i32, vp, u32, u32, u32, u32, u32, u32, u32, vp, vp]
        h.or_swiglu_f64.argtypes = [vp, vp, vp, vp, vp, vp, i32, vp, u32, u32, u32, u32, u32, vp, vp]
        h.or_argmax_f32.argtypes = [vp, u64]
        h.or_argmax_f32.restype = ctypes.c_longlong
        h.or_argmax_f64.argtypes = [vp, u64]
        h.or_argmax_f64.restype = ctypes.c_longlong
        h.or_pack_bf16_exact.argtypes = [vp, u64, vp]
        h.or_bf16_rne.argtypes = [ctypes.c_float]
        h.or_bf16_rne.restype = ctypes.c_uint16
        h.or_num_threads.restype = i32
        h.or_set_threads.argtypes = [i32]
        h.or_model_new.restype = vp
        h.or_model_new.argtypes = [vp, vp, vp, u32]
        h.or_model_free.argtypes = [vp]
        h.or_model_set_matrix.argtypes = [vp, i32, i32, vp, vp, vp, i32, u32, u32, u32, u32]
        h.or_model_set_synth.argtypes = [vp, i32, i32, u64, u32, u32, u32]
        h.or_model_set_vector.argtypes = [vp, i32, i32, vp]
        h.or_model_reset.argtypes = [vp]
        h.or_model_forward.argtypes = [vp, u32, vp]
        h.or_model_forward.restype = i32
        h.or_model_position.argtypes = [vp]
        h.or_model_position.restype = u32
        h.or_synth_matrix.argtypes = [u64, u32, u32, u32, vp, vp, vp]
        _lib = h
    return _lib


def _c(a, dtype):
    a = np.ascontiguousarray(a, dtype=dtype)
    return a, a.ctypes.data


def _meta(m):
    m = np.ascontiguousarray(m)
    if m.dtype == np.uint16:
        return m, 1
    return np.ascontiguousarray(m, dtype=np.float32), 0


def matmul_f64(w, s, b, x, rows, cols, bits, group, batch=1, row0=0, nrows=None):
    """FP64 expansion (tests/quantized.rs:39-51): (y[batch, rows], |w.x| sums).

    Rows outside [row0, row0+nrows) are left as NaN."""
    nrows = rows - row0 if nrows is None else nrows
    w, wp = _c(w, np.uint32)
    s, sb = _meta(s)
    b, _ = _meta(b)
    x, xp = _c(x, np.float32)
    y = np.full(batch * rows, np.nan)
    mag = np.full(batch * rows, np.nan)
    lib().or_matmul_f64(wp, s.ctypes.data, b.ctypes.data, sb, xp, rows, cols, bits, group, batch, row0, nrows,
                        y.ctypes.data, mag.ctypes.data)
    return y.reshape(batch, rows), mag.reshape(batch, rows)


def swiglu_f64(wg, sg, bg, wu, su, bu, x, rows, cols, bits, group, batch=1):
    """FP64 silu(gate.x)*(up.x) and its first-order error scale."""
    wg, wgp = _c(wg, np.uint32)
    wu, wup = _c(wu, np.uint32)
    sg, sb = _meta(sg)
    bg, _ = _meta(bg)
    su, _ = _meta(su)
    bu, _ = _meta(bu)
    x, xp = _c(x, np.float32)
    act = np.empty(batch * rows)
    mag = np.empty(batch * rows)
    lib().or_swiglu_f64(wgp, sg.ctypes.data, bg.ctypes.data, wup, su.ctypes.data, bu.ctypes.data, sb, xp, rows,
                        cols, bits, group, batch, act.ctypes.data, mag.ctypes.data)
    return act.reshape(batch, rows), mag.reshape(batch, rows)


def embed(w, s, b, row, cols, bits, group):
    """FP32 dequantisation of one row, float(q)*s + b (kernels/qwen.metal:40-47)."""
    w, wp = _c(w, np.uint32)
    s, sb = _meta(s)
    b, _ = _meta(b)
    y = np.empty(cols, dtype=np.float32)
    lib().or_embed(wp, s.ctypes.data, b.ctypes.data, sb, row, cols, bits, group, y.ctypes.data)
    return y


def argmax_f32(v) -> int:
    v, p = _c(v, np.float32)
    return int(lib().or_argmax_f32(p, v.size))


def argmax_f64(v) -> int:
    v, p = _c(v, np.float64)
    return int(lib().or_argmax_f64(p, v.size))


def pack_bf16_exact(values):
    v, p = _c(values, np.float32)
    out = np.empty(v.size, dtype=np.uint16)
    return out if lib().or_pack_bf16_exact(p, v.size, out.ctypes.data) else None


def bf16_rne(v: float) -> int:
    return int(lib().or_bf16_rne(v))


def threads() -> int:
    return int(lib().or_num_threads())


def set_threads(n: int) -> None:
    lib().or_set_threads(n)


def tolerance_ratio(got, want, scale, rtol=2e-5, atol=0.0):
    """Worst |got - want| / (atol + rtol*scale); <= 1 passes.  NaN fails."""
    got = np.asarray(got, dtype=np.float64).ravel()
    want = np.asarray(want, dtype=np.float64).ravel()
    scale = np.asarray(scale, dtype=np.float64).ravel()
    err = np.abs(got - want)
    lim = atol + rtol * scale
    with np.errstate(divide="ignore", invalid="ignore"):
        ratio = np.where(err == 0, 0.0, err / lim)
    ratio = np.where(np.isnan(ratio), np.inf, ratio)
    i = int(np.argmax(ratio)) if ratio.size else -1
    return (float(ratio[i]) if ratio.size else 0.0), i


# ---------------------------------------------------------------------------
# FP64 decode graph (decode.c)
# ---------------------------------------------------------------------------

MATRIX_SLOTS = {"qkv": 0, "z": 1, "a": 2, "b": 3, "out": 4, "q": 5, "k": 6, "v": 7, "o": 8, "gate": 9, "up": 10,
                "down": 11}
VECTOR_SLOTS = {"input_norm": 0, "post_norm": 1, "conv": 2, "A_log": 3, "dt_bias": 4, "delta_norm": 5,
                "q_norm": 6, "k_norm": 7}


def synth_matrix(seed: int, mid: int, rows: int, cols: int):
    """The counter-based synthetic Q4/g64 matrix (words, BF16 scale and bias bits)."""
    w = np.empty(rows * cols // 8, dtype=np.uint32)
    s = np.empty(rows * cols // 64, dtype=np.uint16)
    b = np.empty(rows * cols // 64, dtype=np.uint16)
    lib().or_synth_matrix(seed, mid, rows, cols, w.ctypes.data, s.ctypes.data, b.ctypes.data)
    return dict(weight=w.reshape(rows, cols // 8), scales=s.reshape(rows, cols // 64),
                biases=b.reshape(rows, cols // 64))


class DecodeOracle:
    """FP64 restatement of the reference's per-token graph (decode.c).

    cfg: dict with hidden, inter, layers, heads, kv_heads, head_dim, vocab,
    lin_key_heads, lin_value_heads, lin_key_dim, lin_value_dim, conv_width,
    rotary_dim, eps, theta, is_attn (list of bools), context."""

    def __init__(self, cfg):
        self.cfg = cfg
        u = np.array([cfg["hidden"], cfg["inter"], cfg["layers"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"],
                      cfg["vocab"], cfg["lin_key_heads"], cfg["lin_value_heads"], cfg["lin_key_dim"],
                      cfg["lin_value_dim"], cfg["conv_width"], cfg["rotary_dim"]], dtype=np.uint32)
        f = np.array([cfg["eps"], cfg["theta"]], dtype=np.float64)
        att = np.array([1 if a else 0 for a in cfg["is_attn"]], dtype=np.uint8)
        self._keep = []
        self.h = lib().or_model_new(u.ctypes.data, f.ctypes.data, att.ctypes.data, cfg["context"])

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_model_free(self.h)
            self.h = None

    def set_matrix(self, layer, which, mat, rows, cols, bits, group):
        """layer -1: which "embed" / "head"; else a MATRIX_SLOTS name."""
        slot = (0 if which == "embed" else 1) if layer < 0 else MATRIX_SLOTS[which]
        w = np.ascontiguousarray(mat["weight"], dtype=np.uint32)
        s, bf = _meta(mat["scales"])
        b, _ = _meta(mat["biases"])
        self._keep += [w, s, b]
        lib().or_model_set_matrix(self.h, layer, slot, w.ctypes.data, s.ctypes.data, b.ctypes.data, bf, rows,
                                  cols, bits, group)

    def set_synth(self, layer, which, seed, mid, rows, cols):
        slot = (0 if which == "embed" else 1) if layer < 0 else MATRIX_SLOTS[which]
        lib().or_model_set_synth(self.h, layer, slot, seed, mid, rows, cols)

    def set_vector(self, layer, which, values):
        v = np.ascontiguousarray(values, dtype=np.float32)
        self._keep.append(v)
        lib().or_model_set_vector(self.h, layer, 0 if layer < 0 else VECTOR_SLOTS[which], v.ctypes.data)

    def reset(self):
        lib().or_model_reset(self.h)

    @property
    def position(self):
        return int(lib().or_model_position(self.h))

    def forward(self, token: int, logits: bool = True):
        out = np.empty(self.cfg["vocab"], dtype=np.float64) if logits else None
        rc = lib().or_model_forward(self.h, token, out.ctypes.data if logits else None)
        if rc != 0:
            raise ValueError("token outside the vocabulary or context full")
        return out


def synthetic_decode_oracle(cfg, seed, context, mid, mid_embed, mid_head):
    """DecodeOracle of the engine's synthetic model: every matrix generated on
    the fly from (seed, mid(layer, slot)), norms 1, conv 0.1, A_log and
    dt_bias 0 (the reference's synthetic constants, src/engine/synthetic.rs:220-225)."""
    o = DecodeOracle(dict(cfg, context=context))
    H, F = cfg["hidden"], cfg["inter"]
    KD, VD = cfg["lin_key_heads"] * cfg["lin_key_dim"], cfg["lin_value_heads"] * cfg["lin_value_dim"]
    QD, KVD = cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    o.set_synth(-1, "embed", seed, mid_embed, cfg["vocab"], H)
    o.set_synth(-1, "head", seed, mid_head, cfg["vocab"], H)
    ones_h, ones_v = np.ones(H, np.float32), np.ones(cfg["lin_value_dim"], np.float32)
    ones_d = np.ones(cfg["head_dim"], np.float32)
    conv = np.full((2 * KD + VD) * cfg["conv_width"], 0.1, np.float32)
    zeros = np.zeros(cfg["lin_value_heads"], np.float32)
    o.set_vector(-1, None, ones_h)
    for l, att in enumerate(cfg["is_attn"]):
        o.set_vector(l, "input_norm", ones_h)
        o.set_vector(l, "post_norm", ones_h)
        o.set_synth(l, "gate", seed, mid(l, "gate"), F, H)
        o.set_synth(l, "up", seed, mid(l, "up"), F, H)
        o.set_synth(l, "down", seed, mid(l, "down"), H, F)
        if att:
            o.set_synth(l, "q", seed, mid(l, "q"), 2 * QD, H)
            o.set_synth(l, "k", seed, mid(l, "k"), KVD, H)
            o.set_synth(l, "v", seed, mid(l, "v"), KVD, H)
            o.set_synth(l, "o", seed, mid(l, "o"), H, QD)
            o.set_vector(l, "q_norm", ones_d)
            o.set_vector(l, "k_norm", ones_d)
        else:
            o.set_synth(l, "qkv", seed, mid(l, "qkv"), 2 * KD + VD, H)
            o.set_synth(l, "z", seed, mid(l, "z"), VD, H)
            o.set_synth(l, "a", seed, mid(l, "a"), cfg["lin_value_heads"], H)
            o.set_synth(l, "b", seed, mid(l, "b"), cfg["lin_value_heads"], H)
            o.set_synth(l, "out", seed, mid(l, "out"), H, VD)
            o.set_vector(l, "conv", conv)
            o.set_vector(l, "A_log", zeros)
            o.set_vector(l, "dt_bias", zeros)
            o.set_vector(l, "delta_norm", ones_v)
    return o
